"""GPU parity of the device decode (lbk_decode_rows) with the reference's
golden decode vectors (bridge-quant-layout/tests/fixtures: decode-*.input.bin
-> decode-*.output-f32le.bin, oracle_vectors.rs:82-120) and the CPU oracle's
decode_row_into on seeded matrices, bit for bit, plus validate-before-write on
a non-finite scale (k_quants.rs:178-208).
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
import synth
from conftest import read_golden
from gpu_helpers import bits, clean_status, ctx, dev, expect_status, host, matrix

pytestmark = pytest.mark.gpu

FIXTURES = [("q4-k", orc.TYPE_Q4_K, 144), ("q5-k", orc.TYPE_Q5_K, 176), ("iq2-s", orc.TYPE_IQ2_S, 82),
            ("iq3-s", orc.TYPE_IQ3_S, 110)]


@pytest.mark.parametrize("name,ty,bb", FIXTURES)
def test_golden_decode_vectors_on_device(name, ty, bb):
    enc = np.frombuffer(read_golden(f"decode-{name}.input.bin"), dtype=np.uint8).copy()
    want = np.frombuffer(read_golden(f"decode-{name}.output-f32le.bin"), dtype="<u4")
    nblk = enc.size // bb
    ed = dev(enc)
    # the three blocks as one row of 768 lanes, and as three rows of one block
    for in_w, rows in ((256 * nblk, 1), (256, nblk)):
        out = torch.full((in_w * rows,), float("nan"), device="cuda")
        ctx().decode_rows(matrix(ty, in_w, rows, ed), 0, rows, out)
        clean_status()
        np.testing.assert_array_equal(bits(host(out)), want)
    # a sub-range of rows: block 1 alone
    out = torch.full((256,), float("nan"), device="cuda")
    ctx().decode_rows(matrix(ty, 256, nblk, ed), 1, 1, out)
    clean_status()
    np.testing.assert_array_equal(bits(host(out)), want[256:512])


def test_golden_f32_decode_is_a_bit_copy():
    enc = np.frombuffer(read_golden("decode-f32.input.bin"), dtype=np.uint8).copy()
    want = np.frombuffer(read_golden("decode-f32.output-f32le.bin"), dtype="<u4")
    n = enc.size // 4
    out = torch.zeros(n, device="cuda")
    ed = dev(enc)
    ctx().decode_rows(lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, n, 1, ed.data_ptr(), enc.size), 0, 1, out)
    clean_status()
    np.testing.assert_array_equal(bits(host(out)), want)


@pytest.mark.parametrize("ty", [orc.TYPE_Q4_K, orc.TYPE_Q5_K, orc.TYPE_IQ2_S, orc.TYPE_IQ3_S])
def test_seeded_rows_match_oracle_decode(ty):
    rng = np.random.default_rng(ty + 900)
    in_w, rows = 4096, 37
    w = synth.packed_np(rng, ty, in_w, rows)
    rb = in_w // 256 * synth.BLOCK_BYTES[ty]
    out = torch.full((in_w * 30,), float("nan"), device="cuda")
    wd = dev(w)
    ctx().decode_rows(matrix(ty, in_w, rows, wd), 5, 30, out)
    clean_status()
    got = host(out).reshape(30, in_w)
    for r in range(30):
        want = orc.decode_row(ty, w[(5 + r) * rb:(6 + r) * rb].copy(), in_w)
        np.testing.assert_array_equal(bits(got[r]), bits(want), err_msg=f"row {5 + r}")


def test_non_finite_scale_is_reported_and_nothing_written():
    rng = np.random.default_rng(3)
    ty, in_w, rows = orc.TYPE_Q4_K, 1024, 4
    w = synth.packed_np(rng, ty, in_w, rows)
    w[(2 * 4 + 1) * 144 + 2: (2 * 4 + 1) * 144 + 4] = np.array([0x00, 0x7C], np.uint8)  # row 2, block 1: dmin = +inf
    sentinel = np.full(in_w * 3, -3.0, np.float32)
    out = dev(sentinel)
    wd = dev(w)
    ctx().decode_rows(matrix(ty, in_w, rows, wd), 1, 3, out)
    d = expect_status(7)  # NonFiniteScale
    assert d.index == 4 + 1  # block 1 of the range's second row
    np.testing.assert_array_equal(host(out), sentinel)
    with pytest.raises(lbk.LbkError) as e:
        ctx().decode_rows(matrix(ty, in_w, rows, wd), 3, 2, out)
    assert e.value.status == 10  # the range runs past the matrix
