"""C ABI checks that need no GPU: the library loads, exports every declared
entry point, and its host-side validation returns the reference's error for
the reference's bad inputs before touching the device (so a NULL context is
never reached). Mirrors the shape/length/order checks of
bridge-quant-layout/tests/q8_k.rs:11-60, tests/abi.rs:110-240,
bridge-kernels-reference/tests/gemv.rs:190-262 and
bridge-model-hy3/tests/routing.rs:123-235.
"""

import ctypes
import re

import lbk
import numpy as np
import pytest
import synth
from conftest import REPO

L = lbk.lib
NULL = None


def declared_symbols():
    text = (REPO / "include" / "lightbridge_kernels.h").read_text()
    return sorted(set(re.findall(r"\b(lbk_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(L, name), name
    assert set(names) == set(lbk.EXPORTED)


def test_abi_version_and_backend_name():
    assert L.lbk_abi_version() == 1
    assert L.lbk_backend_name() == b"cuda_sm100a_q8_k"


def test_context_create_without_device_reports_no_device():
    p = ctypes.c_void_p()
    st = L.lbk_context_create(0, ctypes.byref(p))
    assert st in (32, 0)  # NO_DEVICE on a CPU-only host
    if st == 0:
        L.lbk_context_destroy(p)


def test_required_q8k_bytes_and_matrix_bytes():
    n = ctypes.c_uint64()
    assert L.lbk_required_q8k_bytes(4096, ctypes.byref(n)) == 0 and n.value == 16 * 292
    assert L.lbk_required_q8k_bytes(0, ctypes.byref(n)) == 10
    assert L.lbk_required_q8k_bytes(255, ctypes.byref(n)) == 10
    for ty, bb in [(12, 144), (13, 176), (22, 82), (21, 110)]:
        assert L.lbk_matrix_bytes(ty, 4096, 3, ctypes.byref(n)) == 0 and n.value == 16 * bb * 3
    assert L.lbk_matrix_bytes(0, 7, 2, ctypes.byref(n)) == 0 and n.value == 56
    assert L.lbk_matrix_bytes(8, 256, 1, ctypes.byref(n)) == 1  # Q8_0: unsupported
    assert L.lbk_matrix_bytes(12, 255, 1, ctypes.byref(n)) == 10
    # planar rows are padded to 16 bytes: IQ3_S 6 blocks = 660 -> 672, IQ2_S 16 blocks = 1312
    assert L.lbk_planar_bytes(21, 1536, 5, ctypes.byref(n)) == 0 and n.value == 672 * 5
    assert L.lbk_planar_bytes(22, 4096, 3, ctypes.byref(n)) == 0 and n.value == 1312 * 3
    assert L.lbk_planar_bytes(0, 256, 1, ctypes.byref(n)) == 1  # F32 has no planar layout
    for ty in (12, 13, 21, 22):
        for k in (256, 768, 1536, 4096):
            assert L.lbk_planar_bytes(ty, k, 7, ctypes.byref(n)) == 0 and n.value == synth.planar_bytes(ty, k, 7)


def test_quantize_validation_order():
    # q8_k.rs:16-33: zero elements, divisibility, encoded length, then values
    assert L.lbk_quantize_q8k(NULL, NULL, 0, NULL, 292, NULL) == 2
    assert L.lbk_quantize_q8k(NULL, NULL, 255, NULL, 292, NULL) == 3
    for actual in (0, 291, 293):
        assert L.lbk_quantize_q8k(NULL, NULL, 256, NULL, actual, NULL) == 5
        d = lbk.last_error()
        assert (d.expected, d.actual) == (292, actual)
    assert L.lbk_quantize_q8k(NULL, NULL, 256, NULL, 292, NULL) == 15  # valid shape, null context


def fake_matrix(ty, in_w, out_w, nbytes=None, layout=0, data=0x1000):
    if nbytes is None:
        nbytes = synth.matrix_bytes(ty, in_w, out_w) if ty else in_w * out_w * 4
    return lbk.Matrix(ty, layout, in_w, out_w, data, nbytes)


def test_vec_dot_validation_order():
    # tests/q8_k.rs:96-153
    m = fake_matrix(0, 256, 1)
    assert L.lbk_vec_dot_q8k(NULL, ctypes.byref(m), NULL, 292, NULL, NULL, NULL) == 1
    m = fake_matrix(12, 0, 1, nbytes=0)
    assert L.lbk_vec_dot_q8k(NULL, ctypes.byref(m), NULL, 292, NULL, NULL, NULL) == 2
    m = fake_matrix(12, 1, 1, nbytes=0)
    assert L.lbk_vec_dot_q8k(NULL, ctypes.byref(m), NULL, 292, NULL, NULL, NULL) == 3
    m = fake_matrix(12, 256, 1, nbytes=143)
    assert L.lbk_vec_dot_q8k(NULL, ctypes.byref(m), NULL, 292, NULL, NULL, NULL) == 5
    m = fake_matrix(12, 256, 1)
    assert L.lbk_vec_dot_q8k(NULL, ctypes.byref(m), NULL, 291, NULL, NULL, NULL) == 5
    assert (lbk.last_error().expected, lbk.last_error().actual) == (292, 291)


def test_gemv_validation():
    # PackedMatrix / prepare_llama_q8k errors (matrix.rs, gemv.rs:245-272)
    m = fake_matrix(8, 256, 1, nbytes=34)
    assert L.lbk_gemv(NULL, ctypes.byref(m), 0x100, 0x200, NULL, 0, NULL) == 1
    m = fake_matrix(22, 100, 2, nbytes=82)
    assert L.lbk_gemv(NULL, ctypes.byref(m), 0x100, 0x200, NULL, 0, NULL) == 10
    m = fake_matrix(22, 256, 2, nbytes=163)
    assert L.lbk_gemv(NULL, ctypes.byref(m), 0x100, 0x200, NULL, 0, NULL) == 5
    m = fake_matrix(12, 256, 1)
    assert L.lbk_gemv(NULL, ctypes.byref(m), 0x100, 0x200, 0x300, 291, NULL) == 15  # null context first
    m = fake_matrix(12, 256, 1, data=0x1001)
    assert L.lbk_gemv(NULL, ctypes.byref(m), 0x100, 0x200, NULL, 0, NULL) == 15  # misaligned data
    m = fake_matrix(12, 256, 1)
    assert L.lbk_gemv_accumulate_scaled(NULL, ctypes.byref(m), 0x100, 0x200, float("inf"), NULL, 0, NULL) == 12
    assert L.lbk_gemv_accumulate_scaled(NULL, ctypes.byref(m), 0x100, 0x200, float("nan"), NULL, 0, NULL) == 12


def test_route_topk_validation():
    # routing.rs:25-56 via tests/routing.rs:123-235
    assert L.lbk_route_topk(NULL, 0x100, 0x200, 4, 1, 0, 1.0, 0x300, NULL) == 16
    assert L.lbk_route_topk(NULL, 0x100, 0x200, 4, 1, 5, 1.0, 0x300, NULL) == 16
    assert L.lbk_route_topk(NULL, 0x100, 0x200, 4, 1, 2, float("nan"), 0x300, NULL) == 18
    assert L.lbk_route_topk(NULL, 0x100, 0x200, 4, 1, 2, 1.0, 0x300, NULL) == 15  # null context


def test_expert_validation():
    # SwiGluExpert::new, activation.rs:13-22
    g = fake_matrix(22, 256, 512)
    u = fake_matrix(22, 256, 512)
    d = fake_matrix(21, 512, 256)
    e = lbk.Expert(g, u, d)
    n = ctypes.c_uint64()
    assert L.lbk_expert_workspace_bytes(ctypes.byref(e), ctypes.byref(n)) == 0 and n.value > 0
    e2 = lbk.Expert(g, fake_matrix(22, 256, 256), d)
    assert L.lbk_expert_workspace_bytes(ctypes.byref(e2), ctypes.byref(n)) == 10
    e3 = lbk.Expert(g, u, fake_matrix(21, 256, 256))
    assert L.lbk_expert_workspace_bytes(ctypes.byref(e3), ctypes.byref(n)) == 10
    assert L.lbk_expert_swiglu_accumulate(NULL, ctypes.byref(e), 0x100, 0x200, float("inf"), 0x400, 1 << 20, NULL) == 12


@pytest.mark.parametrize("ty", [synth.TYPE_IQ2_S, synth.TYPE_IQ3_S, synth.TYPE_Q4_K, synth.TYPE_Q5_K])
@pytest.mark.parametrize("k", [256, 768, 1536, 4096])
def test_planar_layout_round_trips(ty, k):
    rng = np.random.default_rng(ty + k)
    rows = 5
    w = synth.packed_np(rng, ty, k, rows)
    p = synth.planar_np(ty, w, k)
    rs = synth.planar_row_bytes(ty, k)
    assert rs % 16 == 0 and p.size == rs * rows
    raw = k // 256 * synth.BLOCK_BYTES[ty]
    assert not p.reshape(rows, rs)[:, raw:].any()  # zero pad
    if ty in (synth.TYPE_Q4_K, synth.TYPE_Q5_K):  # within a row: a pure byte permutation
        assert np.array_equal(np.sort(p.reshape(rows, rs)[:, :raw], axis=1), np.sort(w.reshape(rows, raw), axis=1))
    assert np.array_equal(synth.gguf_from_planar_np(ty, p, k), w)


def test_qh_transpose_moves_two_bit_cells():
    rng = np.random.default_rng(7)
    w = rng.integers(0, 1 << 32, size=4096, dtype=np.uint64).astype(np.uint32)
    t = synth.qh_transpose(w)
    assert np.array_equal(synth.qh_transpose(t), w)
    for r in range(4):
        for c in range(4):
            src = (w >> np.uint32(8 * r + 2 * c)) & np.uint32(3)
            dst = (t >> np.uint32(8 * c + 2 * r)) & np.uint32(3)
            assert np.array_equal(src, dst)
