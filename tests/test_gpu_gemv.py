"""GPU parity: GEMV and scaled accumulation against the CPU oracle, bit-exact,
including BASELINE configs 1 (Q4_K 4096x4096) and 2 (IQ2_S / IQ3_S
6144x4096), the checkpoint's output projection (Q5_K, 120832 rows of
4096) and a block's attention projections at full size, and the
validate-before-write behaviour of
bridge-kernels-reference/tests/gemv.rs:110-262.
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
import synth
from gpu_helpers import bits, clean_status, ctx, dev, expect_status, host, matrix, planar_dev

pytestmark = pytest.mark.gpu

ALL = [orc.TYPE_Q4_K, orc.TYPE_Q5_K, orc.TYPE_IQ2_S, orc.TYPE_IQ3_S]


def run_gemv(ty, k, rows, w, x, layout):
    wd = planar_dev(ty, w, k) if layout == lbk.LAYOUT_PLANAR else dev(w)
    y = torch.full((rows,), float("nan"), device="cuda")
    q8 = torch.zeros(k // 256 * 292, dtype=torch.uint8, device="cuda")
    ctx().gemv(matrix(ty, k, rows, wd, layout), dev(x), y, q8)
    clean_status()
    return host(y), host(q8)


@pytest.mark.parametrize("layout", [lbk.LAYOUT_GGUF, lbk.LAYOUT_PLANAR])
@pytest.mark.parametrize("ty", ALL)
# rows of 17-32 blocks (4352, 6144, 8192 wide) take the two-pass bulk-copy kernel in the planar layout;
# 5000 rows of 8192 give every warp two or more rows, so its tail batches flush more than once
@pytest.mark.parametrize("k,rows", [(256, 1), (512, 17), (768, 8), (1536, 130), (4096, 100), (3072, 5), (4352, 33),
                                    (6144, 70), (8192, 37), (8192, 5000)])
def test_gemv_matches_oracle(ty, k, rows, layout):
    rng = np.random.default_rng(1000 + k + rows + ty)
    w = synth.packed_np(rng, ty, k, rows)
    x = rng.standard_normal(k).astype(np.float32)
    y, q8 = run_gemv(ty, k, rows, w, x, layout)
    want, want_q8 = orc.gemv(ty, k, rows, w, x)
    np.testing.assert_array_equal(q8, want_q8)
    np.testing.assert_array_equal(bits(y), bits(want))


@pytest.mark.parametrize("layout", [lbk.LAYOUT_GGUF, lbk.LAYOUT_PLANAR])
@pytest.mark.parametrize(
    "ty,k,rows,seed,d_range",
    [
        (orc.TYPE_Q4_K, 4096, 4096, 0, (0.001, 0.02)),  # config 1
        (orc.TYPE_IQ2_S, 4096, 6144, 1, (0.001, 0.01)),  # config 2
        (orc.TYPE_IQ3_S, 4096, 6144, 1, (0.001, 0.01)),  # config 2, IQ3_S variant
        (orc.TYPE_Q5_K, 4096, 120832, 5, (0.001, 0.02)),  # the checkpoint's output.weight (vocabulary rows)
        # a Hy3 block's attention projections (schema.rs:120-170; profile.rs:22-29: hidden 4096,
        # 64 heads, 8 KV heads, key / value length 128)
        (orc.TYPE_IQ2_S, 4096, 8192, 6, (0.001, 0.01)),  # attn_q
        (orc.TYPE_IQ2_S, 4096, 1024, 7, (0.001, 0.01)),  # attn_k
        (orc.TYPE_Q4_K, 4096, 1024, 8, (0.001, 0.02)),   # attn_v
        (orc.TYPE_IQ3_S, 8192, 4096, 9, (0.001, 0.01)),  # attn_output (input 64 x 128)
    ],
)
def test_baseline_matvec_configs_bit_exact(ty, k, rows, seed, d_range, layout):
    rng = np.random.default_rng(seed)
    w = synth.packed_np(rng, ty, k, rows, d_range)
    x = rng.standard_normal(k).astype(np.float32)
    y, q8 = run_gemv(ty, k, rows, w, x, layout)
    want, want_q8 = orc.gemv(ty, k, rows, w, x)
    np.testing.assert_array_equal(q8, want_q8)
    np.testing.assert_array_equal(bits(y), bits(want))


@pytest.mark.parametrize("ty", ALL)
def test_accumulate_scaled_matches_oracle(ty):
    rng = np.random.default_rng(ty)
    k, rows = 1536, 4096
    w = synth.packed_np(rng, ty, k, rows)
    x = rng.standard_normal(k).astype(np.float32)
    y0 = rng.standard_normal(rows).astype(np.float32) * 10
    scale = np.float32(0.3721)
    yd = dev(y0)
    ctx().gemv_accumulate_scaled(matrix(ty, k, rows, dev(w)), dev(x), yd, float(scale))
    clean_status()
    want = orc.gemv_accumulate_scaled(ty, k, rows, w, x, y0.copy(), scale)
    np.testing.assert_array_equal(bits(host(yd)), bits(want))


def test_f32_gemv_sequential_bit_exact():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((192, 4096)) * 0.02).astype(np.float32)
    x = rng.standard_normal(4096).astype(np.float32)
    wd = dev(w.reshape(-1))
    y = torch.zeros(192, device="cuda")
    ctx().gemv(lbk.Matrix(lbk.TYPE_F32, 0, 4096, 192, wd.data_ptr(), wd.numel() * 4), dev(x), y)
    clean_status()
    np.testing.assert_array_equal(bits(host(y)), bits(orc.gemv_f32(4096, 192, w, x)))


def test_gemv_rejects_non_finite_input_without_writing():
    rng = np.random.default_rng(9)
    w = synth.packed_np(rng, orc.TYPE_IQ2_S, 4096, 1000)
    x = rng.standard_normal(4096).astype(np.float32)
    x[3000] = np.nan
    sentinel = np.full(1000, 123.5, np.float32)
    y = dev(sentinel)
    ctx().gemv(matrix(orc.TYPE_IQ2_S, 4096, 1000, dev(w)), dev(x), y)
    d = expect_status(8)
    assert d.index == 3000
    np.testing.assert_array_equal(host(y), sentinel)


def test_accumulate_rejects_non_finite_destination_without_writing():
    rng = np.random.default_rng(10)
    w = synth.packed_np(rng, orc.TYPE_Q4_K, 512, 300)
    x = rng.standard_normal(512).astype(np.float32)
    y0 = np.ones(300, np.float32)
    y0[123] = np.inf
    yd = dev(y0)
    ctx().gemv_accumulate_scaled(matrix(orc.TYPE_Q4_K, 512, 300, dev(w)), dev(x), yd, 0.5)
    d = expect_status(12)
    assert d.index == 123
    np.testing.assert_array_equal(host(yd), y0)


def test_non_finite_weight_scale_reported():
    rng = np.random.default_rng(11)
    w = synth.packed_np(rng, orc.TYPE_IQ3_S, 256, 4)
    w[2 * 110 : 2 * 110 + 2] = np.frombuffer(np.uint16(0x7C00).tobytes(), np.uint8)
    ctx().validate_matrix(matrix(orc.TYPE_IQ3_S, 256, 4, dev(w)))
    d = expect_status(7)
    assert d.index == 2 and d.bits == 0x7C00


@pytest.mark.parametrize("ty", ALL)
@pytest.mark.parametrize("k", [768, 1536, 4096])
def test_repack_matches_numpy_and_unpack_inverts(ty, k):
    rng = np.random.default_rng(20 + ty + k)
    rows = 37
    w = synth.packed_np(rng, ty, k, rows)
    src = dev(w)
    planar = torch.full((synth.planar_bytes(ty, k, rows),), 0xA5, dtype=torch.uint8, device="cuda")
    ctx().repack(matrix(ty, k, rows, src), planar)
    back = torch.zeros_like(src)
    ctx().unpack(matrix(ty, k, rows, planar, lbk.LAYOUT_PLANAR), back)
    clean_status()
    np.testing.assert_array_equal(host(planar), synth.planar_np(ty, w, k))  # pad bytes zeroed too
    np.testing.assert_array_equal(host(back), w)


@pytest.mark.parametrize("layout", [lbk.LAYOUT_GGUF, lbk.LAYOUT_PLANAR])
@pytest.mark.parametrize("H,F,gty,dty", [(4096, 1536, 22, 21), (2048, 512, 12, 12), (1024, 768, 22, 13)])
def test_expert_swiglu_accumulate_matches_oracle(H, F, gty, dty, layout):
    """expert_swiglu_accumulate_into (bridge-kernels-reference/src/activation.rs:104-144):
    dst += coef * down(swiglu(gate x, up x)), against the oracle's gemv_into ->
    apply_swiglu -> gemv_accumulate_scaled_into chain; bit for bit up to the
    exp of the SwiGLU (unpinned), held to 1e-5 relative element-wise."""
    rng = np.random.default_rng(H + F + gty + dty + layout)
    g = synth.packed_np(rng, gty, H, F)
    u = synth.packed_np(rng, gty, H, F)
    d = synth.packed_np(rng, dty, F, H)
    x = rng.standard_normal(H).astype(np.float32)
    dst0 = rng.standard_normal(H).astype(np.float32)
    coef = np.float32(-0.8125)
    gv, _ = orc.gemv(gty, H, F, g, x)
    uv, _ = orc.gemv(gty, H, F, u, x)
    hv = orc.swiglu(gv, uv)
    want = orc.gemv_accumulate_scaled(dty, F, H, d, hv, dst0.copy(), coef)

    def up(ty, b, in_w):
        return planar_dev(ty, b, in_w) if layout == lbk.LAYOUT_PLANAR else dev(b)

    keep = [up(gty, g, H), up(gty, u, H), up(dty, d, F)]
    e = lbk.Expert(matrix(gty, H, F, keep[0], layout), matrix(gty, H, F, keep[1], layout),
                   matrix(dty, F, H, keep[2], layout))
    ws = torch.zeros(ctx().expert_workspace_bytes(e), dtype=torch.uint8, device="cuda")
    dst = dev(dst0)
    ctx().expert_swiglu_accumulate(e, dev(x), dst, float(coef), ws)
    clean_status()
    got = host(dst)
    err = float(np.max(np.abs(got.astype(np.float64) - want) / np.maximum(np.abs(want), 1e-3 * np.abs(want).max())))
    assert err <= 1e-5, err
    print(f"expert SwiGLU accumulate H={H} F={F}: element-wise {err:.3e}, "
          f"{int(np.count_nonzero(got.view(np.uint32) != want.view(np.uint32)))} of {H} values differ in bits")
