"""GPU parity: Q8_K quantization and packed-row dots against the reference's
golden vectors and the CPU oracle (bit-exact).

Follows crates/bridge-quant-layout/tests/oracle_vectors.rs:142-182 and
tests/q8_k.rs:62-94; the per-super-block int32 sums are compared one by one.
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
import synth
from conftest import read_golden
from gpu_helpers import bits, clean_status, ctx, dev, expect_status, host, matrix, planar_dev

pytestmark = pytest.mark.gpu

TYPES = [("q4-k", orc.TYPE_Q4_K, 144), ("q5-k", orc.TYPE_Q5_K, 176), ("iq2-s", orc.TYPE_IQ2_S, 82), ("iq3-s", orc.TYPE_IQ3_S, 110)]


def test_q8k_golden_fixture_byte_exact():
    x = np.frombuffer(read_golden("q8-k-activations.input-f32le.bin"), dtype="<f4").copy()
    want = np.frombuffer(read_golden("q8-k-activations.output-q8-k.bin"), dtype=np.uint8)
    q8 = torch.full((want.size,), 0xA5, dtype=torch.uint8, device="cuda")
    ctx().quantize_q8k(dev(x), q8)
    clean_status()
    np.testing.assert_array_equal(host(q8), want)


def edge_rows(rng):
    rows = [rng.standard_normal(4096).astype(np.float32)]
    z = np.zeros(512, np.float32)
    z[300] = -3.0  # block 0 all zero, block 1 one negative value
    rows.append(z)
    t = rng.standard_normal(256).astype(np.float32)
    t[10], t[200] = 5.0, -5.0  # max-abs tie: first index wins, keeps its sign
    rows.append(t)
    t2 = rng.standard_normal(256).astype(np.float32)
    t2[7], t2[9] = -7.5, 7.5
    rows.append(t2)
    rows.append((rng.standard_normal(1024) * 1e-30).astype(np.float32))  # subnormal scales
    rows.append((rng.standard_normal(768) * 1e30).astype(np.float32))
    rows.append(np.full(256, -0.0, np.float32))
    rows.append((rng.integers(-3, 4, 2048) * 0.5).astype(np.float32))  # many exact .5 ties
    return rows


def test_q8k_edge_rows_match_oracle():
    rng = np.random.default_rng(7)
    for x in edge_rows(rng):
        want = orc.quantize_q8k(x)
        q8 = torch.zeros(want.size, dtype=torch.uint8, device="cuda")
        ctx().quantize_q8k(dev(x), q8)
        clean_status()
        np.testing.assert_array_equal(host(q8), want)


@pytest.mark.parametrize("idx", [0, 127, 255, 256, 511])
def test_q8k_non_finite_rejected_before_any_write(idx):
    for bad in [np.inf, -np.inf, np.float32(np.nan)]:
        x = np.zeros(512, np.float32)
        x[idx] = bad
        x[idx + 1 if idx < 511 else 0] = np.nan  # a later/earlier bad lane too
        sentinel = (np.arange(584) * 37 + 11).astype(np.uint8)
        q8 = dev(sentinel)
        ctx().quantize_q8k(dev(x), q8)
        d = expect_status(8)
        first = min(idx, idx + 1 if idx < 511 else 0)
        assert d.index == first
        np.testing.assert_array_equal(host(q8), sentinel)


@pytest.mark.parametrize("layout", [lbk.LAYOUT_GGUF, lbk.LAYOUT_PLANAR])
@pytest.mark.parametrize("name,ty,bb", TYPES)
def test_dot_golden_fixture_bit_exact(name, ty, bb, layout):
    enc = np.frombuffer(read_golden(f"decode-{name}.input.bin"), dtype=np.uint8).copy()
    q8 = np.frombuffer(read_golden("q8-k-activations.output-q8-k.bin"), dtype=np.uint8).copy()
    want = np.frombuffer(read_golden(f"dot-{name}-q8-k.output-f32le.bin"), dtype="<u4")[0]
    w = planar_dev(ty, enc, 768) if layout == lbk.LAYOUT_PLANAR else dev(enc)
    out = torch.full((1,), float("nan"), device="cuda")
    sums = torch.zeros(27, dtype=torch.int32, device="cuda")
    ctx().vec_dot(matrix(ty, 768, 1, w, layout), dev(q8), out, sums)
    clean_status()
    assert bits(host(out))[0] == want
    per = 9 if ty in (orc.TYPE_Q4_K, orc.TYPE_Q5_K) else 1
    np.testing.assert_array_equal(host(sums)[: 3 * per], orc.block_sums(ty, enc, q8, 768))


@pytest.mark.parametrize("layout", [lbk.LAYOUT_GGUF, lbk.LAYOUT_PLANAR])
@pytest.mark.parametrize("ty", [orc.TYPE_Q4_K, orc.TYPE_Q5_K, orc.TYPE_IQ2_S, orc.TYPE_IQ3_S])
@pytest.mark.parametrize("k,rows", [(256, 1), (768, 7), (1536, 33), (4096, 64), (8192, 3)])
def test_block_sums_and_dots_match_oracle(ty, k, rows, layout):
    rng = np.random.default_rng(k * 31 + rows + ty)
    w = synth.packed_np(rng, ty, k, rows)
    q8 = orc.quantize_q8k(rng.standard_normal(k).astype(np.float32))
    wd = planar_dev(ty, w, k) if layout == lbk.LAYOUT_PLANAR else dev(w)
    out = torch.zeros(rows, device="cuda")
    per = 9 if ty in (orc.TYPE_Q4_K, orc.TYPE_Q5_K) else 1
    sums = torch.zeros(rows * k // 256 * per, dtype=torch.int32, device="cuda")
    ctx().vec_dot(matrix(ty, k, rows, wd, layout), dev(q8), out, sums)
    clean_status()
    rb = k // 256 * synth.BLOCK_BYTES[ty]
    got_sums = host(sums).reshape(rows, -1)
    got = bits(host(out))
    for r in range(rows):
        row = w[r * rb : (r + 1) * rb]
        np.testing.assert_array_equal(got_sums[r], orc.block_sums(ty, row, q8, k), err_msg=f"row {r}")
        assert got[r] == bits([orc.vec_dot(ty, row, q8, k, simd=True)])[0], f"row {r}"


def test_non_finite_q8_scale_reported():
    q8 = np.zeros(292, np.uint8)
    q8[0:4] = np.frombuffer(np.float32(np.nan).tobytes(), np.uint8)
    w = synth.packed_np(np.random.default_rng(1), orc.TYPE_Q4_K, 256, 1)
    out = torch.full((1,), 7.0, device="cuda")
    ctx().vec_dot(matrix(orc.TYPE_Q4_K, 256, 1, dev(w)), dev(q8), out)
    expect_status(9)
    assert host(out)[0] == 7.0
