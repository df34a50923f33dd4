"""ctypes binding of liblbk_b200.so (include/lightbridge_kernels.h).

A thin host-side mirror of the reference's operator API for the quantized
expert path -- gemv_into / gemv_accumulate_scaled_into / vec_dot_q8_k /
quantize_row_q8_k_into / route_experts_into / expert_swiglu_accumulate_into /
moe_routed_by_id_into -- over device memory held in torch tensors. Every call
goes through the C ABI into the sm_100a kernels; there is no CPU or PyTorch
fallback: if the library is missing, importing this module raises.
"""

from __future__ import annotations

import ctypes
import pathlib
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "liblbk_b200.so"

TYPE_F32, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q8_K, TYPE_IQ3_S, TYPE_IQ2_S = 0, 12, 13, 15, 21, 22
BLOCK_BYTES = {TYPE_F32: 4, TYPE_Q4_K: 144, TYPE_Q5_K: 176, TYPE_IQ2_S: 82, TYPE_IQ3_S: 110}
Q8K_BLOCK_BYTES = 292
LAYOUT_GGUF, LAYOUT_PLANAR = 0, 1
ROUTER_SEQUENTIAL, ROUTER_TREE = 0, 1

STATUS = {
    0: "OK", 1: "UNSUPPORTED_TYPE", 2: "ZERO_LOGICAL_ELEMENTS", 3: "LOGICAL_ELEMENTS_NOT_DIVISIBLE",
    4: "ARITHMETIC_OVERFLOW", 5: "ENCODED_LENGTH_MISMATCH", 6: "OUTPUT_LENGTH_MISMATCH", 7: "NON_FINITE_SCALE",
    8: "NON_FINITE_ACTIVATION", 9: "NON_FINITE_Q8_SCALE", 10: "DIMENSION_MISMATCH", 11: "SCRATCH_TOO_SMALL",
    12: "NON_FINITE_VALUE", 13: "ROUTED_EXPERT_ORDER", 14: "DUPLICATE_ROUTED_EXPERT", 15: "INVALID_PARAMETER",
    16: "ROUTING_TOPK", 17: "ROUTING_LENGTH", 18: "NON_FINITE_ROUTING_VALUE", 30: "CUDA_ERROR", 31: "TIMEOUT",
    32: "NO_DEVICE", 33: "FORMAT_ERROR", 34: "IO_ERROR",
}

# GGUF value types (lbk_gguf_value.type)
GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL = 0, 1, 2, 3, 4, 5, 6, 7
GGUF_STRING, GGUF_ARRAY, GGUF_U64, GGUF_I64, GGUF_F64 = 8, 9, 10, 11, 12


class ErrorDetail(ctypes.Structure):
    _fields_ = [
        ("status", ctypes.c_int32),
        ("cuda_error", ctypes.c_int32),
        ("index", ctypes.c_uint64),
        ("bits", ctypes.c_uint32),
        ("expected", ctypes.c_uint64),
        ("actual", ctypes.c_uint64),
        ("message", ctypes.c_char * 160),
    ]


class Matrix(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("input_width", ctypes.c_uint64),
        ("output_width", ctypes.c_uint64),
        ("data", ctypes.c_void_p),
        ("bytes", ctypes.c_uint64),
    ]


class Expert(ctypes.Structure):
    _fields_ = [("gate", Matrix), ("up", Matrix), ("down", Matrix)]


class EpExchange(ctypes.Structure):
    _fields_ = [("routing", ctypes.c_uint64), ("control", ctypes.c_uint64), ("q8", ctypes.c_uint64),
                ("dots", ctypes.c_uint64), ("total", ctypes.c_uint64), ("q8_bytes", ctypes.c_uint64)]


class Routed(ctypes.Structure):
    _fields_ = [("expert_id", ctypes.c_uint32), ("coefficient", ctypes.c_float)]


class MoeWeights(ctypes.Structure):
    _fields_ = [
        ("experts", ctypes.POINTER(Expert)),
        ("expert_count", ctypes.c_uint64),
        ("shared", Expert),
        ("router", Matrix),
        ("selection_bias", ctypes.c_void_p),
        ("top_k", ctypes.c_uint32),
        ("weight_scale", ctypes.c_float),
    ]


class GgufLimits(ctypes.Structure):
    _fields_ = [
        ("max_dimensions", ctypes.c_uint32),
        ("max_string_bytes", ctypes.c_uint64),
        ("max_array_elements", ctypes.c_uint64),
        ("max_tensors", ctypes.c_uint64),
        ("max_metadata_entries", ctypes.c_uint64),
        ("max_metadata_bytes", ctypes.c_uint64),
    ]


class GgufFileInfo(ctypes.Structure):
    _fields_ = [
        ("version", ctypes.c_uint32),
        ("big_endian", ctypes.c_uint32),
        ("alignment", ctypes.c_uint64),
        ("shard_count", ctypes.c_uint64),
        ("tensor_count", ctypes.c_uint64),
        ("metadata_count", ctypes.c_uint64),
        ("data_offset", ctypes.c_uint64),
        ("file_len", ctypes.c_uint64),
    ]


class GgufTensor(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("n_dims", ctypes.c_uint32),
        ("dims", ctypes.c_uint64 * 4),
        ("shard", ctypes.c_uint32),
        ("offset", ctypes.c_uint64),
        ("relative_offset", ctypes.c_uint64),
        ("bytes", ctypes.c_uint64),
        ("name_len", ctypes.c_uint64),
    ]

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(self.dims[: self.n_dims])


class GgufValue(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_uint32),
        ("element_type", ctypes.c_uint32),
        ("count", ctypes.c_uint64),
        ("u", ctypes.c_uint64),
        ("f", ctypes.c_double),
    ]


class LbkError(RuntimeError):
    def __init__(self, status: int, detail: ErrorDetail | None = None):
        self.status = status
        self.detail = detail
        msg = STATUS.get(status, str(status))
        if detail is not None:
            msg += f" (index={detail.index}, bits={detail.bits:#x}, expected={detail.expected}, actual={detail.actual}, {detail.message.decode(errors='replace')})"
        super().__init__(msg)


def build() -> None:
    """Compile liblbk_b200.so for sm_100a in place (nvcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-j8", "-C", str(HERE)], check=True)


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (or __graft_entry__.build())")
    L = ctypes.CDLL(str(LIB_PATH))
    P, U64, I32, U32, F = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32, ctypes.c_uint32, ctypes.c_float
    PM = ctypes.POINTER(Matrix)
    PE = ctypes.POINTER(Expert)
    sigs = {
        "lbk_abi_version": ([], I32),
        "lbk_backend_name": ([], ctypes.c_char_p),
        "lbk_context_create": ([I32, ctypes.POINTER(P)], I32),
        "lbk_context_destroy": ([P], I32),
        "lbk_context_sync_status": ([P, P, ctypes.POINTER(ErrorDetail)], I32),
        "lbk_last_error_detail": ([ctypes.POINTER(ErrorDetail)], None),
        "lbk_required_q8k_bytes": ([U64, ctypes.POINTER(U64)], I32),
        "lbk_matrix_bytes": ([I32, U64, U64, ctypes.POINTER(U64)], I32),
        "lbk_planar_bytes": ([I32, U64, U64, ctypes.POINTER(U64)], I32),
        "lbk_quantize_q8k": ([P, P, U64, P, U64, P], I32),
        "lbk_vec_dot_q8k": ([P, PM, P, U64, P, P, P], I32),
        "lbk_gemv": ([P, PM, P, P, P, U64, P], I32),
        "lbk_gemv_accumulate_scaled": ([P, PM, P, P, F, P, U64, P], I32),
        "lbk_router_logits": ([P, PM, P, U64, P, I32, P], I32),
        "lbk_route_topk": ([P, P, P, U64, U64, U32, F, P, P], I32),
        "lbk_expert_workspace_bytes": ([PE, ctypes.POINTER(U64)], I32),
        "lbk_expert_swiglu_accumulate": ([P, PE, P, P, F, P, U64, P], I32),
        "lbk_moe_layer_create": ([P, ctypes.POINTER(MoeWeights), P, ctypes.POINTER(P)], I32),
        "lbk_moe_layer_destroy": ([P], I32),
        "lbk_moe_layer_fused": ([P], I32),
        "lbk_moe_layer_set_grouping": ([P, U64], I32),
        "lbk_moe_layer_set_wait_limit": ([P, U32], I32),
        "lbk_moe_layer_set_tensor_cores": ([P, U64], I32),
        "lbk_moe_workspace_bytes": ([P, U64, ctypes.POINTER(U64)], I32),
        "lbk_moe_forward": ([P, P, U64, P, P, I32, P, U64, P], I32),
        "lbk_moe_routed": ([P, P, U64, P, P, P, U64, P], I32),
        "lbk_moe_forward_no_alloc": ([P, P, U64, P, P, I32, P], I32),
        "lbk_rms_norm": ([P, P, P, U64, U64, F, P, I32, P], I32),
        "lbk_residual_add": ([P, P, P, U64, P], I32),
        "lbk_moe_block_workspace_bytes": ([P, U64, ctypes.POINTER(U64)], I32),
        "lbk_moe_block_forward": ([P, P, P, F, U64, P, I32, P, U64, P], I32),
        "lbk_moe_block_route": ([P, P, P, F, U64, P, I32, P, U64, P], I32),
        "lbk_moe_block_finish": ([P, P, U64, P, P, U64, P], I32),
        "lbk_ep_layer_create": ([P, ctypes.POINTER(MoeWeights), U64, U64, P, ctypes.POINTER(P)], I32),
        "lbk_ep_q8_bytes": ([P, ctypes.POINTER(U64)], I32),
        "lbk_ep_workspace_bytes": ([P, U64, ctypes.POINTER(U64)], I32),
        "lbk_ep_route": ([P, P, U64, P, P, P, U64, P], I32),
        "lbk_ep_items_forward": ([P, P, P, U64, P, P, U64, P], I32),
        "lbk_ep_combine": ([P, P, U64, P, P, P, P, U64, P], I32),
        "lbk_peer_alloc": ([P, U64, ctypes.POINTER(P), ctypes.c_char_p], I32),
        "lbk_peer_free": ([P, P], I32),
        "lbk_peer_open": ([P, ctypes.c_char_p, ctypes.POINTER(P)], I32),
        "lbk_peer_close": ([P, P], I32),
        "lbk_ep_exchange_layout": ([P, U64, ctypes.POINTER(EpExchange)], I32),
        "lbk_ep_publish": ([P, P, U64, P, U64, P, U64, P], I32),
        "lbk_ep_gather": ([P, P, U32, U32, U64, P, P, P, P, U64, P], I32),
        "lbk_ep_items_forward_counted": ([P, P, P, P, U64, P, P, U64, P], I32),
        "lbk_ep_scatter": ([P, P, U32, U32, U64, P, P, P, U64, P], I32),
        "lbk_ep_shared": ([P, P, U64, U64, P, P, U64, P], I32),
        "lbk_ep_items_return": ([P, P, U32, U32, U64, P, P, P, P, U64, P, U64, P], I32),
        "lbk_tc_grouped_dots": ([P, I32, P, U32, P, U32, P, U64, P, P, U64, P], I32),
        "lbk_ep_combine_exchange": ([P, P, U32, U64, U64, P, P, P, U64, P], I32),
        "lbk_moe_layer_trace": ([P, I32], I32),
        "lbk_moe_layer_trace_read": ([P, ctypes.POINTER(ctypes.c_float)], I32),
        "lbk_repack": ([P, PM, P, U64, P], I32),
        "lbk_unpack": ([P, PM, P, U64, P], I32),
        "lbk_validate_matrix": ([P, PM, P], I32),
        "lbk_decode_rows": ([P, PM, U64, U64, P, P], I32),
        "lbk_gguf_default_limits": ([ctypes.POINTER(GgufLimits)], None),
        "lbk_gguf_open": ([ctypes.c_char_p, ctypes.POINTER(GgufLimits), ctypes.POINTER(P)], I32),
        "lbk_gguf_close": ([P], I32),
        "lbk_gguf_info": ([P, ctypes.POINTER(GgufFileInfo)], I32),
        "lbk_gguf_tensor_at": ([P, U64, ctypes.POINTER(GgufTensor), ctypes.c_char_p, U64], I32),
        "lbk_gguf_find_tensor": ([P, ctypes.c_char_p, ctypes.POINTER(U64)], I32),
        "lbk_gguf_metadata": ([P, ctypes.c_char_p, ctypes.POINTER(GgufValue)], I32),
        "lbk_gguf_metadata_string": ([P, ctypes.c_char_p, ctypes.c_char_p, U64, ctypes.POINTER(U64)], I32),
        "lbk_moe_layer_load": ([P, P, U32, U64, U64, P, ctypes.POINTER(P)], I32),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    return L


lib = _load()
EXPORTED = (
    "lbk_abi_version lbk_backend_name lbk_context_create lbk_context_destroy lbk_context_sync_status "
    "lbk_last_error_detail lbk_required_q8k_bytes lbk_matrix_bytes lbk_planar_bytes lbk_quantize_q8k lbk_vec_dot_q8k lbk_gemv "
    "lbk_gemv_accumulate_scaled lbk_router_logits lbk_route_topk lbk_expert_workspace_bytes "
    "lbk_expert_swiglu_accumulate lbk_moe_layer_create lbk_moe_layer_destroy lbk_moe_layer_fused lbk_moe_layer_set_grouping lbk_moe_layer_set_wait_limit "
    "lbk_moe_layer_set_tensor_cores "
    "lbk_moe_workspace_bytes lbk_moe_forward lbk_moe_routed lbk_moe_forward_no_alloc lbk_moe_layer_trace "
    "lbk_moe_layer_trace_read lbk_rms_norm lbk_residual_add lbk_moe_block_workspace_bytes lbk_moe_block_forward lbk_moe_block_route lbk_moe_block_finish "
    "lbk_ep_layer_create lbk_ep_q8_bytes lbk_ep_workspace_bytes lbk_ep_route "
    "lbk_ep_items_forward lbk_ep_combine lbk_peer_alloc lbk_peer_free lbk_peer_open lbk_peer_close "
    "lbk_ep_exchange_layout lbk_ep_publish lbk_ep_gather lbk_ep_items_forward_counted lbk_ep_scatter "
    "lbk_ep_shared lbk_ep_items_return lbk_ep_combine_exchange lbk_tc_grouped_dots "
    "lbk_repack lbk_unpack lbk_validate_matrix lbk_decode_rows "
    "lbk_gguf_default_limits lbk_gguf_open lbk_gguf_close lbk_gguf_info lbk_gguf_tensor_at lbk_gguf_find_tensor "
    "lbk_gguf_metadata lbk_gguf_metadata_string lbk_moe_layer_load"
).split()


def last_error() -> ErrorDetail:
    d = ErrorDetail()
    lib.lbk_last_error_detail(ctypes.byref(d))
    return d


def check(status: int) -> None:
    if status != 0:
        raise LbkError(status, last_error())


def tc_matrices(entries) -> "np.ndarray":
    """lbk_tc_matrix records (data pointer, rows, blocks, out_offset) packed
    into a uint8 array (24 bytes each) for a device copy."""
    import numpy as np

    rec = np.dtype([("data", "<u8"), ("rows", "<u4"), ("blocks", "<u4"), ("out_offset", "<u8")])
    arr = np.zeros(len(entries), dtype=rec)
    for i, (data, rows, blocks, off) in enumerate(entries):
        arr[i] = (data, rows, blocks, off)
    return arr.view(np.uint8)


def _ptr(t) -> int | None:
    if t is None:
        return None
    if isinstance(t, int):  # a raw device address (e.g. inside a PeerBuffer)
        return t
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    return stream


def matrix(ty: int, input_width: int, output_width: int, data, layout: int = LAYOUT_GGUF) -> Matrix:
    """Descriptor of a packed matrix held in a device tensor (uint8 / f32)."""
    nbytes = data.numel() * data.element_size()
    return Matrix(ty, layout, input_width, output_width, data.data_ptr(), nbytes)


class Context:
    """Per-device context (status word, codebooks). Mirrors the reference's
    CpuBackend (bridge-kernels-cpu/src/lib.rs:75-118): create once, reuse."""

    def __init__(self, device: int = 0):
        p = ctypes.c_void_p()
        check(lib.lbk_context_create(device, ctypes.byref(p)))
        self.ptr = p
        self.device = device

    def close(self) -> None:
        if self.ptr:
            lib.lbk_context_destroy(self.ptr)
            self.ptr = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def sync_status(self, stream=None) -> int:
        d = ErrorDetail()
        st = lib.lbk_context_sync_status(self.ptr, _stream(stream), ctypes.byref(d))
        self.last_detail = d
        return st

    def raise_status(self, stream=None) -> None:
        st = self.sync_status(stream)
        if st != 0:
            raise LbkError(st, self.last_detail)

    # -- kernels (device tensors) --------------------------------------
    def quantize_q8k(self, x, q8, stream=None) -> None:
        check(lib.lbk_quantize_q8k(self.ptr, _ptr(x), x.numel(), _ptr(q8), q8.numel(), _stream(stream)))

    def vec_dot(self, m: Matrix, q8, out, block_sums=None, stream=None) -> None:
        check(lib.lbk_vec_dot_q8k(self.ptr, ctypes.byref(m), _ptr(q8), q8.numel(), _ptr(out), _ptr(block_sums), _stream(stream)))

    def gemv(self, m: Matrix, x, y, q8_scratch=None, stream=None) -> None:
        n = 0 if q8_scratch is None else q8_scratch.numel()
        check(lib.lbk_gemv(self.ptr, ctypes.byref(m), _ptr(x), _ptr(y), _ptr(q8_scratch), n, _stream(stream)))

    def tc_grouped_dots(self, mats, nmat: int, jobs, njobs: int, q8, q8_row_bytes: int, pair_tokens, dots,
                        dots_stride: int, stream=None, type: int = TYPE_IQ2_S) -> None:
        """lbk_tc_grouped_dots: mats a device tensor of lbk_tc_matrix records
        (tc_matrices), jobs a device int32 [njobs, 4] tensor."""
        check(lib.lbk_tc_grouped_dots(self.ptr, type, _ptr(mats), nmat, _ptr(jobs), njobs, _ptr(q8), q8_row_bytes,
                                      _ptr(pair_tokens), _ptr(dots), dots_stride, _stream(stream)))

    def gemv_accumulate_scaled(self, m: Matrix, x, y, scale: float, q8_scratch=None, stream=None) -> None:
        n = 0 if q8_scratch is None else q8_scratch.numel()
        check(lib.lbk_gemv_accumulate_scaled(self.ptr, ctypes.byref(m), _ptr(x), _ptr(y), float(scale), _ptr(q8_scratch), n, _stream(stream)))

    def router_logits(self, router: Matrix, x, tokens: int, logits, mode: int = ROUTER_SEQUENTIAL, stream=None) -> None:
        check(lib.lbk_router_logits(self.ptr, ctypes.byref(router), _ptr(x), tokens, _ptr(logits), mode, _stream(stream)))

    def route_topk(self, logits, bias, expert_count: int, tokens: int, k: int, weight_scale: float, routed, stream=None) -> None:
        check(lib.lbk_route_topk(self.ptr, _ptr(logits), _ptr(bias), expert_count, tokens, k, float(weight_scale), _ptr(routed), _stream(stream)))

    def expert_workspace_bytes(self, e: Expert) -> int:
        n = ctypes.c_uint64()
        check(lib.lbk_expert_workspace_bytes(ctypes.byref(e), ctypes.byref(n)))
        return n.value

    def expert_swiglu_accumulate(self, e: Expert, x, dst, coef: float, workspace, stream=None) -> None:
        check(lib.lbk_expert_swiglu_accumulate(self.ptr, ctypes.byref(e), _ptr(x), _ptr(dst), float(coef), _ptr(workspace), workspace.numel(), _stream(stream)))

    def rms_norm(self, x, weight, n: int, rows: int, epsilon: float, out, mode: int = ROUTER_SEQUENTIAL,
                 stream=None) -> None:
        check(lib.lbk_rms_norm(self.ptr, _ptr(x), _ptr(weight), n, rows, float(epsilon), _ptr(out), mode,
                               _stream(stream)))

    def residual_add(self, dest, src, n: int, stream=None) -> None:
        check(lib.lbk_residual_add(self.ptr, _ptr(dest), _ptr(src), n, _stream(stream)))

    def repack(self, m: Matrix, dst, stream=None) -> None:
        check(lib.lbk_repack(self.ptr, ctypes.byref(m), _ptr(dst), dst.numel(), _stream(stream)))

    def unpack(self, m: Matrix, dst, stream=None) -> None:
        check(lib.lbk_unpack(self.ptr, ctypes.byref(m), _ptr(dst), dst.numel(), _stream(stream)))

    def decode_rows(self, m: Matrix, first_row: int, rows: int, out, stream=None) -> None:
        """decode_row_into (k_quants.rs:71-105) over a run of rows, into f32."""
        check(lib.lbk_decode_rows(self.ptr, ctypes.byref(m), first_row, rows, _ptr(out), _stream(stream)))

    def validate_matrix(self, m: Matrix, stream=None) -> None:
        check(lib.lbk_validate_matrix(self.ptr, ctypes.byref(m), _stream(stream)))


class MoeLayer:
    """A registered, HBM-resident MoE layer (lbk_moe_layer_create)."""

    def __init__(self, ctx: Context, experts: list[Expert], shared: Expert, router: Matrix, bias, top_k: int,
                 weight_scale: float, stream=None):
        self.ctx = ctx
        self._experts = (Expert * len(experts))(*experts)
        self._w = MoeWeights(
            ctypes.cast(self._experts, ctypes.POINTER(Expert)), len(experts), shared, router, bias.data_ptr(), top_k,
            float(weight_scale),
        )
        self._keep = [bias]
        p = ctypes.c_void_p()
        check(lib.lbk_moe_layer_create(ctx.ptr, ctypes.byref(self._w), _stream(stream), ctypes.byref(p)))
        self.ptr = p
        self.top_k = top_k
        self.hidden = shared.gate.input_width

    @property
    def fused(self) -> bool:
        return bool(lib.lbk_moe_layer_fused(self.ptr))

    def set_grouping(self, min_tokens: int) -> None:
        """Calls of at least `min_tokens` tokens run the grouped kernels (0: never)."""
        check(lib.lbk_moe_layer_set_grouping(self.ptr, min_tokens))

    def set_tensor_cores(self, min_pairs_per_expert: int) -> None:
        check(lib.lbk_moe_layer_set_tensor_cores(self.ptr, min_pairs_per_expert))

    def set_wait_limit(self, polls: int) -> None:
        check(lib.lbk_moe_layer_set_wait_limit(self.ptr, polls))

    def workspace_bytes(self, tokens: int) -> int:
        n = ctypes.c_uint64()
        check(lib.lbk_moe_workspace_bytes(self.ptr, tokens, ctypes.byref(n)))
        return n.value

    def forward(self, x, tokens: int, out, workspace, routed_out=None, router_mode: int = ROUTER_TREE, stream=None) -> None:
        check(lib.lbk_moe_forward(self.ptr, _ptr(x), tokens, _ptr(out), _ptr(routed_out), router_mode, _ptr(workspace), workspace.numel(), _stream(stream)))

    def routed(self, x, tokens: int, routed, out, workspace, stream=None) -> None:
        check(lib.lbk_moe_routed(self.ptr, _ptr(x), tokens, _ptr(routed), _ptr(out), _ptr(workspace), workspace.numel(), _stream(stream)))

    def block_workspace_bytes(self, tokens: int) -> int:
        n = ctypes.c_uint64()
        check(lib.lbk_moe_block_workspace_bytes(self.ptr, tokens, ctypes.byref(n)))
        return n.value

    def block_forward(self, hidden, ffn_norm, epsilon: float, tokens: int, workspace, routed_out=None,
                      router_mode: int = ROUTER_TREE, stream=None) -> None:
        check(lib.lbk_moe_block_forward(self.ptr, _ptr(hidden), _ptr(ffn_norm), float(epsilon), tokens, _ptr(routed_out),
                                        router_mode, _ptr(workspace), workspace.numel(), _stream(stream)))

    def block_route(self, hidden, ffn_norm, epsilon: float, tokens: int, workspace, routed_out=None,
                    router_mode: int = ROUTER_TREE, stream=None) -> None:
        """hy3_moe_route_token's FFN part (layer.rs:473-605): norm, router, top-k."""
        check(lib.lbk_moe_block_route(self.ptr, _ptr(hidden), _ptr(ffn_norm), float(epsilon), tokens, _ptr(routed_out),
                                      router_mode, _ptr(workspace), workspace.numel(), _stream(stream)))

    def block_finish(self, hidden, tokens: int, selected, workspace, stream=None) -> None:
        """hy3_moe_finish_token (layer.rs:610-659): identity check, experts, residual add."""
        check(lib.lbk_moe_block_finish(self.ptr, _ptr(hidden), tokens, _ptr(selected), _ptr(workspace), workspace.numel(),
                                       _stream(stream)))

    def trace(self, enable: bool = True) -> None:
        check(lib.lbk_moe_layer_trace(self.ptr, int(enable)))

    def trace_read(self) -> tuple[float, float, float]:
        ms = (ctypes.c_float * 3)()
        check(lib.lbk_moe_layer_trace_read(self.ptr, ms))
        return ms[0], ms[1], ms[2]

    def close(self) -> None:
        if self.ptr:
            lib.lbk_moe_layer_destroy(self.ptr)
            self.ptr = None


class EpLayer(MoeLayer):
    """One rank's share of an expert-parallel MoE layer (lbk_ep_layer_create):
    `experts` are the global experts [first_expert, first_expert + len) of a
    router over `global_experts`; the router and the shared expert are whole."""

    def __init__(self, ctx: Context, experts: list[Expert], shared: Expert, router: Matrix, bias, top_k: int,
                 weight_scale: float, global_experts: int, first_expert: int, stream=None):
        self.ctx = ctx
        self._experts = (Expert * len(experts))(*experts)
        self._w = MoeWeights(
            ctypes.cast(self._experts, ctypes.POINTER(Expert)), len(experts), shared, router, bias.data_ptr(), top_k,
            float(weight_scale),
        )
        self._keep = [bias]
        p = ctypes.c_void_p()
        check(lib.lbk_ep_layer_create(ctx.ptr, ctypes.byref(self._w), global_experts, first_expert, _stream(stream),
                                      ctypes.byref(p)))
        self.ptr = p
        self.top_k = top_k
        self.hidden = shared.gate.input_width
        self.global_experts = global_experts
        self.first_expert = first_expert
        self.local_experts = len(experts)

    @property
    def q8_bytes(self) -> int:
        n = ctypes.c_uint64()
        check(lib.lbk_ep_q8_bytes(self.ptr, ctypes.byref(n)))
        return n.value

    def workspace_bytes(self, count: int) -> int:
        n = ctypes.c_uint64()
        check(lib.lbk_ep_workspace_bytes(self.ptr, count, ctypes.byref(n)))
        return n.value

    def route(self, x, tokens: int, routed, q8, workspace, stream=None) -> None:
        check(lib.lbk_ep_route(self.ptr, _ptr(x), tokens, _ptr(routed), _ptr(q8), _ptr(workspace), workspace.numel(),
                               _stream(stream)))

    def items_forward(self, q8_items, items_routed, items: int, dots, workspace, stream=None) -> None:
        check(lib.lbk_ep_items_forward(self.ptr, _ptr(q8_items), _ptr(items_routed), items, _ptr(dots), _ptr(workspace),
                                       workspace.numel(), _stream(stream)))

    def combine(self, q8, tokens: int, routed, routed_dots, out, workspace, stream=None) -> None:
        check(lib.lbk_ep_combine(self.ptr, _ptr(q8), tokens, _ptr(routed), _ptr(routed_dots), _ptr(out),
                                 _ptr(workspace), workspace.numel(), _stream(stream)))

    # exchange over peer memory (lbk_ep_publish / gather / items_forward_counted / scatter / combine_exchange)
    def exchange_layout(self, cap: int) -> EpExchange:
        x = EpExchange()
        check(lib.lbk_ep_exchange_layout(self.ptr, cap, ctypes.byref(x)))
        return x

    def publish(self, x, tokens: int, xbuf: int, cap: int, workspace, stream=None) -> None:
        check(lib.lbk_ep_publish(self.ptr, _ptr(x), tokens, xbuf, cap, _ptr(workspace), workspace.numel(),
                                 _stream(stream)))

    def gather(self, peers, world: int, rank: int, cap: int, q8_items, items, returns, count, stream=None) -> None:
        check(lib.lbk_ep_gather(self.ptr, _ptr(peers), world, rank, cap, _ptr(q8_items), _ptr(items), _ptr(returns),
                                _ptr(count), items.shape[0], _stream(stream)))

    def items_forward_counted(self, q8_items, items, count, dots, workspace, stream=None) -> None:
        check(lib.lbk_ep_items_forward_counted(self.ptr, _ptr(q8_items), _ptr(items), _ptr(count), items.shape[0],
                                               _ptr(dots), _ptr(workspace), workspace.numel(), _stream(stream)))

    def scatter(self, peers, world: int, rank: int, cap: int, dots, returns, count, stream=None) -> None:
        check(lib.lbk_ep_scatter(self.ptr, _ptr(peers), world, rank, cap, _ptr(dots), _ptr(returns), _ptr(count),
                                 returns.shape[0], _stream(stream)))

    def items_return(self, peers, world: int, rank: int, cap: int, q8_items, items, returns, count, workspace,
                     stream=None) -> None:
        check(lib.lbk_ep_items_return(self.ptr, _ptr(peers), world, rank, cap, _ptr(q8_items), _ptr(items),
                                      _ptr(returns), _ptr(count), items.shape[0], _ptr(workspace), workspace.numel(),
                                      _stream(stream)))

    def shared(self, xbuf: int, cap: int, tokens: int, shared_dots, workspace, stream=None) -> None:
        check(lib.lbk_ep_shared(self.ptr, xbuf, cap, tokens, _ptr(shared_dots), _ptr(workspace), workspace.numel(),
                                _stream(stream)))

    def combine_exchange(self, xbuf: int, world: int, cap: int, tokens: int, out, workspace, shared_dots=None,
                         stream=None) -> None:
        check(lib.lbk_ep_combine_exchange(self.ptr, xbuf, world, cap, tokens, _ptr(shared_dots), _ptr(out),
                                          _ptr(workspace), workspace.numel(), _stream(stream)))


class PeerBuffer:
    """Device memory mapped into the other processes of the node
    (lbk_peer_alloc / lbk_peer_open): plain peer loads and stores."""

    def __init__(self, ctx: Context, nbytes: int):
        self.ctx = ctx
        p = ctypes.c_void_p()
        h = ctypes.create_string_buffer(64)
        check(lib.lbk_peer_alloc(ctx.ptr, nbytes, ctypes.byref(p), h))
        self.ptr = p.value
        self.handle = h.raw
        self.nbytes = nbytes
        self._opened: list[int] = []

    def open(self, handle: bytes) -> int:
        p = ctypes.c_void_p()
        check(lib.lbk_peer_open(self.ctx.ptr, handle, ctypes.byref(p)))
        self._opened.append(p.value)
        return p.value

    def close_opened(self) -> None:
        """Unmap the other processes' buffers opened here."""
        for q in self._opened:
            lib.lbk_peer_close(self.ctx.ptr, q)
        self._opened = []

    def close(self) -> None:
        self.close_opened()
        if self.ptr:
            lib.lbk_peer_free(self.ctx.ptr, self.ptr)
            self.ptr = None


class Gguf:
    """A GGUF split set opened by the native reader (lbk_gguf_open): the
    mirror of bridge-gguf-split's open_set / GgufSet and of GgufFile's typed
    metadata getters (bridge-gguf/src/reader.rs:55-168)."""

    def __init__(self, entry, limits: GgufLimits | None = None):
        p = ctypes.c_void_p()
        check(lib.lbk_gguf_open(str(entry).encode(), ctypes.byref(limits) if limits is not None else None,
                                ctypes.byref(p)))
        self.ptr = p

    @staticmethod
    def default_limits() -> GgufLimits:
        lim = GgufLimits()
        lib.lbk_gguf_default_limits(ctypes.byref(lim))
        return lim

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self) -> None:
        if self.ptr:
            lib.lbk_gguf_close(self.ptr)
            self.ptr = None

    def info(self) -> GgufFileInfo:
        out = GgufFileInfo()
        check(lib.lbk_gguf_info(self.ptr, ctypes.byref(out)))
        return out

    def tensors(self) -> list[tuple[str, GgufTensor]]:
        out = []
        for i in range(self.info().tensor_count):
            t = GgufTensor()
            check(lib.lbk_gguf_tensor_at(self.ptr, i, ctypes.byref(t), None, 0))
            name = ctypes.create_string_buffer(t.name_len + 1)
            check(lib.lbk_gguf_tensor_at(self.ptr, i, ctypes.byref(t), name, t.name_len + 1))
            out.append((name.value.decode(), t))
        return out

    def tensor(self, name: str) -> GgufTensor:
        i = ctypes.c_uint64()
        check(lib.lbk_gguf_find_tensor(self.ptr, name.encode(), ctypes.byref(i)))
        t = GgufTensor()
        check(lib.lbk_gguf_tensor_at(self.ptr, i.value, ctypes.byref(t), None, 0))
        return t

    def value(self, key: str) -> GgufValue:
        v = GgufValue()
        check(lib.lbk_gguf_metadata(self.ptr, key.encode(), ctypes.byref(v)))
        return v

    def metadata(self, key: str):
        """The primary shard's value for `key`: int, float, bool or str; for
        arrays the tuple ("array", element_type, count)."""
        v = self.value(key)
        if v.type == GGUF_STRING:
            n = ctypes.c_uint64()
            buf = ctypes.create_string_buffer(v.count + 1)
            check(lib.lbk_gguf_metadata_string(self.ptr, key.encode(), buf, v.count + 1, ctypes.byref(n)))
            return buf.raw[: n.value].decode()
        if v.type == GGUF_ARRAY:
            return ("array", v.element_type, v.count)
        if v.type in (GGUF_F32, GGUF_F64):
            return v.f
        if v.type == GGUF_BOOL:
            return bool(v.u)
        if v.type in (GGUF_I8, GGUF_I16, GGUF_I32, GGUF_I64):
            return ctypes.c_int64(v.u).value
        return v.u


def load_layer(ctx: Context, gguf: Gguf, block: int, first_expert: int = 0, expert_count: int = 0,
               stream=None) -> MoeLayer:
    """HBM-resident MoE layer of block `block` read from a Hy3 GGUF set
    (lbk_moe_layer_load): every routed expert (an MoeLayer), or the routed
    experts [first_expert, first_expert + expert_count) of an expert-parallel
    rank (an EpLayer)."""
    p = ctypes.c_void_p()
    check(lib.lbk_moe_layer_load(ctx.ptr, gguf.ptr, block, first_expert, expert_count, _stream(stream), ctypes.byref(p)))
    experts = gguf.metadata("hy_v3.expert_count")
    count = expert_count or experts - first_expert
    layer = object.__new__(MoeLayer if (first_expert, count) == (0, experts) else EpLayer)
    layer.ctx = ctx
    layer.ptr = p
    layer._keep = []
    layer.top_k = gguf.metadata("hy_v3.expert_used_count")
    layer.hidden = gguf.metadata("hy_v3.embedding_length")
    if isinstance(layer, EpLayer):
        layer.global_experts = experts
        layer.first_expert = first_expert
        layer.local_experts = count
    return layer
