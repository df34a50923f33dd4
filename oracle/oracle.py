"""ctypes binding of the CPU oracle (liblbk_oracle.so).

TEST INFRASTRUCTURE ONLY: the checker that the CUDA path is compared against,
and the timed CPU baseline. The product (lightbridge-engine_b200/) never
imports this module; only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference legs do.
"""

from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "liblbk_oracle.so"

TYPE_F32, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q8_K, TYPE_IQ3_S, TYPE_IQ2_S = 0, 12, 13, 15, 21, 22
BLOCK_BYTES = {TYPE_F32: 4, TYPE_Q4_K: 144, TYPE_Q5_K: 176, TYPE_IQ2_S: 82, TYPE_IQ3_S: 110}
Q8K_BLOCK_BYTES = 292


class Detail(ctypes.Structure):
    _fields_ = [
        ("status", ctypes.c_int32),
        ("index", ctypes.c_uint64),
        ("bits", ctypes.c_uint32),
        ("expected", ctypes.c_uint64),
        ("actual", ctypes.c_uint64),
    ]


class Matrix(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("input_width", ctypes.c_uint64),
        ("output_width", ctypes.c_uint64),
        ("data", ctypes.c_void_p),
        ("bytes", ctypes.c_uint64),
    ]


class Expert(ctypes.Structure):
    _fields_ = [("gate", Matrix), ("up", Matrix), ("down", Matrix)]


class Rope(ctypes.Structure):
    """Hy3RopeParams (bridge-kernels-reference/src/rope.rs:8-18)."""

    _fields_ = [
        ("head_dim", ctypes.c_uint64),
        ("context_length", ctypes.c_uint64),
        ("original_context", ctypes.c_uint64),
        ("base", ctypes.c_float),
        ("freq_scale", ctypes.c_float),
        ("ext_factor", ctypes.c_float),
        ("attn_factor", ctypes.c_float),
        ("beta_fast", ctypes.c_float),
        ("beta_slow", ctypes.c_float),
    ]


def build() -> None:
    """Compile the oracle library in place (make, no reference sources)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    P = ctypes.c_void_p
    U64 = ctypes.c_uint64
    I32 = ctypes.c_int32
    F = ctypes.c_float
    L.orc_last_detail.argtypes = [ctypes.POINTER(Detail)]
    L.orc_quantize_q8k.argtypes = [P, U64, P, U64]
    L.orc_decode_row.argtypes = [I32, P, U64, U64, P, U64]
    L.orc_vec_dot.argtypes = [I32, P, U64, P, U64, U64, I32, ctypes.POINTER(F)]
    L.orc_block_sums.argtypes = [I32, P, P, U64, P]
    L.orc_gemv.argtypes = [ctypes.POINTER(Matrix), P, P, P, I32, I32]
    L.orc_gemv_accumulate_scaled.argtypes = [ctypes.POINTER(Matrix), P, P, F, P, I32, I32]
    L.orc_gemv_f32.argtypes = [ctypes.POINTER(Matrix), P, P, I32]
    L.orc_route_experts.argtypes = [P, P, U64, U64, F, P, P]
    L.orc_swiglu.argtypes = [P, P, U64]
    L.orc_moe_routed.argtypes = [ctypes.POINTER(Expert), U64, ctypes.POINTER(Expert), P, P, U64, P, P, I32, I32, I32]
    L.orc_moe_token.argtypes = [
        ctypes.POINTER(Expert), U64, ctypes.POINTER(Expert), ctypes.POINTER(Matrix), P, U64, F, P, P, P, P, I32, I32, I32,
    ]
    L.orc_rms_norm.argtypes = [P, U64, P, U64, F, P, U64]
    L.orc_residual_add.argtypes = [P, U64, P, U64]
    L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.orc_f16_to_f32.restype = F
    L.orc_nearest_int.argtypes = [F]
    L.orc_expf.argtypes = [F]
    L.orc_expf.restype = F
    L.orc_table_bytes.argtypes = [I32, ctypes.POINTER(U64)]
    L.orc_table_bytes.restype = ctypes.POINTER(ctypes.c_uint8)
    L.orc_f32_to_f16.argtypes = [F]
    L.orc_f32_to_f16.restype = ctypes.c_uint16
    L.orc_hy3_fill_matrix.argtypes = [I32, U64, U64, U64, P, U64]
    L.orc_hy3_embeddings.argtypes = [P, U64]
    L.orc_hy3_embeddings.restype = None
    L.orc_hy3_norm_weights.argtypes = [U64, U64, P]
    L.orc_hy3_norm_weights.restype = None
    L.orc_gemv_dequant.argtypes = [ctypes.POINTER(Matrix), P, P]
    L.orc_gemv_dequant_accumulate_scaled.argtypes = [ctypes.POINTER(Matrix), P, P, F]
    L.orc_head_rms_norm.argtypes = [P, U64, P, U64, F]
    L.orc_rope_neox_yarn.argtypes = [P, U64, U64, ctypes.POINTER(Rope)]
    L.orc_gqa_attention.argtypes = [P, P, U64, U64, U64, U64, P, P, P, P]
    L.orc_softmax.argtypes = [P, U64, P]


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def last_detail() -> Detail:
    d = Detail()
    lib().orc_last_detail(ctypes.byref(d))
    return d


class OracleError(RuntimeError):
    def __init__(self, status: int):
        d = last_detail()
        super().__init__(f"oracle status {status} (index {d.index}, bits {d.bits:#x})")
        self.status = status
        self.detail = d


def _check(status: int) -> None:
    if status != 0:
        raise OracleError(status)


def matrix(ty: int, input_width: int, output_width: int, data: np.ndarray) -> Matrix:
    return Matrix(ty, input_width, output_width, _p(data), data.nbytes)


def quantize_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 256 * Q8K_BLOCK_BYTES, dtype=np.uint8)
    _check(lib().orc_quantize_q8k(_p(x), x.size, _p(out), out.size))
    return out


def quantize_q8k_status(x: np.ndarray, out: np.ndarray) -> int:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return lib().orc_quantize_q8k(_p(x) if x.size else None, x.size, _p(out) if out.size else None, out.size)


def decode_row(ty: int, enc: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    _check(lib().orc_decode_row(ty, _p(enc), enc.size, n, _p(out), out.size))
    return out


def vec_dot(ty: int, w: np.ndarray, q8: np.ndarray, n: int, simd: bool = False) -> np.float32:
    r = ctypes.c_float()
    _check(lib().orc_vec_dot(ty, _p(w), w.size, _p(q8), q8.size, n, int(simd), ctypes.byref(r)))
    return np.float32(r.value)


def block_sums(ty: int, w: np.ndarray, q8: np.ndarray, n: int) -> np.ndarray:
    nb = n // 256
    per = 9 if ty in (TYPE_Q4_K, TYPE_Q5_K) else 1
    out = np.zeros(nb * per, dtype=np.int32)
    _check(lib().orc_block_sums(ty, _p(w), _p(q8), n, _p(out)))
    return out


def gemv(ty: int, in_w: int, out_w: int, w: np.ndarray, x: np.ndarray, simd: bool = True, threads: int = 0):
    """Returns (y, q8) like gemv_into in CpuParallelQ8K mode."""
    m = matrix(ty, in_w, out_w, w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(out_w, dtype=np.float32)
    q8 = np.zeros(in_w // 256 * Q8K_BLOCK_BYTES, dtype=np.uint8)
    _check(lib().orc_gemv(ctypes.byref(m), _p(x), _p(y), _p(q8), int(simd), threads))
    return y, q8


def gemv_accumulate_scaled(ty, in_w, out_w, w, x, y, scale, simd=True, threads=0):
    m = matrix(ty, in_w, out_w, w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    q8 = np.zeros(in_w // 256 * Q8K_BLOCK_BYTES, dtype=np.uint8)
    _check(lib().orc_gemv_accumulate_scaled(ctypes.byref(m), _p(x), _p(y), float(scale), _p(q8), int(simd), threads))
    return y


def gemv_f32(in_w: int, out_w: int, w: np.ndarray, x: np.ndarray, threads: int = 0) -> np.ndarray:
    wb = np.ascontiguousarray(w, dtype=np.float32).view(np.uint8).reshape(-1)
    m = matrix(TYPE_F32, in_w, out_w, wb)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(out_w, dtype=np.float32)
    _check(lib().orc_gemv_f32(ctypes.byref(m), _p(x), _p(y), threads))
    return y


def route_experts(logits: np.ndarray, bias: np.ndarray, k: int, weight_scale: float):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    ids = np.zeros(k, dtype=np.uint32)
    coefs = np.zeros(k, dtype=np.float32)
    _check(lib().orc_route_experts(_p(logits), _p(bias), logits.size, k, float(weight_scale), _p(ids), _p(coefs)))
    return ids, coefs


def route_experts_status(logits, bias, k, weight_scale) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    ids = np.zeros(max(k, 1), dtype=np.uint32)
    coefs = np.zeros(max(k, 1), dtype=np.float32)
    return lib().orc_route_experts(_p(logits), _p(bias), logits.size, k, float(weight_scale), _p(ids), _p(coefs))


def rms_norm_status(x: np.ndarray, weight: np.ndarray, epsilon: float, out: np.ndarray) -> int:
    """weighted_rms_norm_into (norm.rs:5-18); `out` is left untouched on error."""
    x = np.ascontiguousarray(x, np.float32)
    weight = np.ascontiguousarray(weight, np.float32)
    return lib().orc_rms_norm(_p(x), x.size, _p(weight), weight.size, float(epsilon), _p(out), out.size)


def rms_norm(x: np.ndarray, weight: np.ndarray, epsilon: float) -> np.ndarray:
    out = np.empty(np.asarray(x).size, np.float32)
    _check(rms_norm_status(x, weight, epsilon, out))
    return out


def residual_add_status(dest: np.ndarray, src: np.ndarray) -> int:
    """residual_add_in_place (norm.rs:83-100) on `dest` (float32, in place)."""
    src = np.ascontiguousarray(src, np.float32)
    return lib().orc_residual_add(_p(dest), dest.size, _p(src), src.size)


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.array(gate, dtype=np.float32, copy=True)
    u = np.ascontiguousarray(up, dtype=np.float32)
    _check(lib().orc_swiglu(_p(g), _p(u), g.size))
    return g


class ExpertTable:
    """Host copy of a layer's expert table as oracle descriptors (keeps the
    numpy buffers alive)."""

    def __init__(self, experts, shared, router=None, hidden=None):
        # experts: list of (gate_ty, gate_bytes, up_ty, up_bytes, down_ty, down_bytes, hidden, ffn)
        self._keep = []
        arr = (Expert * len(experts))()
        for i, e in enumerate(experts):
            arr[i] = self._expert(*e)
        self.experts = arr
        self.shared = self._expert(*shared)
        self.count = len(experts)
        self.router = None
        if router is not None:
            rb = np.ascontiguousarray(router, dtype=np.float32).view(np.uint8).reshape(-1)
            self._keep.append(rb)
            self.router = matrix(TYPE_F32, hidden, router.shape[0], rb)

    def _expert(self, gty, gb, uty, ub, dty, db, hidden, ffn) -> Expert:
        self._keep += [gb, ub, db]
        return Expert(matrix(gty, hidden, ffn, gb), matrix(uty, hidden, ffn, ub), matrix(dty, ffn, hidden, db))


def moe_routed(table: ExpertTable, ids, coefs, x, preflight=False, simd=True, threads=0):
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    coefs = np.ascontiguousarray(coefs, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(table.shared.down.output_width, dtype=np.float32)
    _check(
        lib().orc_moe_routed(
            table.experts, table.count, ctypes.byref(table.shared), _p(ids), _p(coefs), ids.size, _p(x), _p(out),
            int(preflight), int(simd), threads,
        )
    )
    return out


def moe_token(table: ExpertTable, bias, k, weight_scale, x, preflight=False, simd=True, threads=0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    out = np.zeros(table.shared.down.output_width, dtype=np.float32)
    ids = np.zeros(k, dtype=np.uint32)
    coefs = np.zeros(k, dtype=np.float32)
    _check(
        lib().orc_moe_token(
            table.experts, table.count, ctypes.byref(table.shared), ctypes.byref(table.router), _p(bias), k,
            float(weight_scale), _p(x), _p(out), _p(ids), _p(coefs), int(preflight), int(simd), threads,
        )
    )
    return out, ids, coefs


def table_bytes(which: int) -> bytes:
    n = ctypes.c_uint64()
    ptr = lib().orc_table_bytes(which, ctypes.byref(n))
    return ctypes.string_at(ptr, n.value)


def hw_threads() -> int:
    return lib().orc_hw_threads()



# ---------------------------------------------------------------- reduced Hy3


def f32_to_f16(v: float) -> int:
    return int(lib().orc_f32_to_f16(float(v)))


def hy3_fill_matrix(ty: int, in_w: int, out_w: int, seed: int) -> np.ndarray:
    """OwnedMatrix::quantized (bridge-test-model/src/hy3.rs:68-117): GGUF bytes."""
    out = np.zeros(in_w // 256 * BLOCK_BYTES[ty] * out_w, dtype=np.uint8)
    _check(lib().orc_hy3_fill_matrix(ty, in_w, out_w, seed, _p(out), out.size))
    return out


def hy3_embeddings(n: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    lib().orc_hy3_embeddings(_p(out), n)
    return out


def hy3_norm_weights(length: int, seed: int) -> np.ndarray:
    out = np.zeros(length, dtype=np.float32)
    lib().orc_hy3_norm_weights(length, seed, _p(out))
    return out


def gemv_dequant(ty: int, in_w: int, out_w: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """gemv_into in DequantF32 mode (gemv.rs:33-41)."""
    m = matrix(ty, in_w, out_w, w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(out_w, dtype=np.float32)
    _check(lib().orc_gemv_dequant(ctypes.byref(m), _p(x), _p(y)))
    return y


def gemv_dequant_accumulate_scaled(ty, in_w, out_w, w, x, y, scale):
    m = matrix(ty, in_w, out_w, w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    _check(lib().orc_gemv_dequant_accumulate_scaled(ctypes.byref(m), _p(x), _p(y), float(scale)))
    return y


def head_rms_norm(values: np.ndarray, weight: np.ndarray, head_dim: int, epsilon: float) -> np.ndarray:
    v = np.array(values, dtype=np.float32, copy=True)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    _check(lib().orc_head_rms_norm(_p(v), v.size, _p(w), head_dim, float(epsilon)))
    return v


def rope_neox_yarn(values: np.ndarray, head_count: int, position: int, rope: Rope) -> np.ndarray:
    v = np.array(values, dtype=np.float32, copy=True)
    _check(lib().orc_rope_neox_yarn(_p(v), head_count, position, ctypes.byref(rope)))
    return v


def gqa_attention(cache_keys, cache_values, stored, q_heads, kv_heads, dim, q, k, v) -> np.ndarray:
    """One token of causal_gqa_attention_into (attention.rs:28-87) over
    `stored` cached [token][kv_head][dim] rows plus this token's k / v."""
    ck = np.ascontiguousarray(cache_keys, dtype=np.float32)
    cv = np.ascontiguousarray(cache_values, dtype=np.float32)
    q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
    out = np.zeros(q_heads * dim, dtype=np.float32)
    _check(lib().orc_gqa_attention(_p(ck), _p(cv), stored, q_heads, kv_heads, dim, _p(q), _p(k), _p(v), _p(out)))
    return out


def softmax(logits: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.zeros_like(x)
    _check(lib().orc_softmax(_p(x), x.size, _p(out)))
    return out
