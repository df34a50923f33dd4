// abi.cu -- the C ABI (include/lightbridge_kernels.h): contexts, host-side
// validation in the reference's order, and the launch sequences.
//
// Host validation mirrors the reference's checks so that a caller sees the
// same error for the same bad input: PackedMatrix / EncodedTensorView
// (bridge-kernels-reference/src/matrix.rs:26-150), required_q8_k_bytes
// (gemv.rs:18-31), prepare_llama_q8k (gemv.rs:245-272), quantize_row_q8_k_into
// (bridge-quant-layout/src/q8_k.rs:16-33), vec_dot validation (q8_k.rs:121-161),
// route_experts_into (bridge-model-hy3/src/routing.rs:25-56), SwiGluExpert::new
// (activation.rs:13-22) and the MoE structure checks (moe.rs:64-129).

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <utility>
#include <vector>

#include "lbk_iq_tables.h"
#include "lbk_kernels.h"
#include "lbk_host.h"
#include "lbk_moe.h"
#include "lbk_tc.h"

struct lbk_context {
    int device;
    int sm_count;
    lbk::DeviceStatus* status;          // device
    unsigned long long* scratch_min;    // device, 8 bytes
    uint64_t* iq2s;                     // device, 1024
    uint32_t* iq3s;                     // device, 512
    uint32_t* img_iq2;                  // replicated shared-memory images
    uint32_t* img_iq3;
    lbk::Tables tables() const {
        return lbk::Tables{reinterpret_cast<const uint4*>(img_iq2), reinterpret_cast<const uint4*>(img_iq3)};
    }
};

struct lbk_moe_layer {
    lbk_context* ctx;
    uint64_t E, H, F, k;
    // Resident routed experts: global IDs [first, first + E_local). A full
    // layer holds all E; an expert-parallel layer holds its rank's share.
    uint64_t E_local, first;
    float weight_scale;
    bool fused;
    lbk_moe_weights w;                   // host copy (experts pointer not kept)
    std::vector<lbk_expert> experts;     // host copy of the expert descriptors
    const uint8_t** d_gate;              // device pointer tables [E_local]
    const uint8_t** d_up;
    const uint8_t** d_down;
    int gate_type, down_type, sgate_type, sdown_type;
    cudaEvent_t trace[4];
    bool tracing;
    void* owned;                         // device memory freed with the layer (lbk_moe_layer_load)
    uint64_t group_min = 8;              // calls of at least this many tokens (items) run the grouped kernels; 0: never
    bool group_set = false;              // group_min set by lbk_moe_layer_set_grouping
    uint64_t tc_min = 4;                 // expert-parallel items: tensor cores from this many expected pairs per expert; 0: never
    uint32_t wait_limit = 1u << 20;      // polls of the down kernel's wait for the single-token routing flag
    // Block workspaces between lbk_moe_block_route and lbk_moe_block_finish,
    // with the routed call's token count (the reference keeps this phase in
    // its per-token scratch: Hy3BlockScratch::streaming_moe_pending).
    std::mutex phase_mu;
    std::map<const void*, uint64_t> pending;
};

namespace {

thread_local lbk_error_detail g_err;

int32_t ok() {
    std::memset(&g_err, 0, sizeof(g_err));
    return LBK_OK;
}

int32_t fail(int32_t status, const char* msg, uint64_t index = 0, uint64_t expected = 0, uint64_t actual = 0,
             uint32_t bits = 0) {
    std::memset(&g_err, 0, sizeof(g_err));
    g_err.status = status;
    g_err.index = index;
    g_err.expected = expected;
    g_err.actual = actual;
    g_err.bits = bits;
    std::snprintf(g_err.message, sizeof(g_err.message), "%s", msg);
    return status;
}

int32_t cuda_fail(cudaError_t e, const char* where) {
    int32_t s = fail(LBK_CUDA_ERROR, where);
    g_err.cuda_error = (int32_t)e;
    std::snprintf(g_err.message, sizeof(g_err.message), "%s: %s", where, cudaGetErrorString(e));
    return s;
}

uint32_t f32_bits(float v) {
    uint32_t b;
    std::memcpy(&b, &v, 4);
    return b;
}

uint64_t block_bytes(int32_t ty) {
    switch (ty) {
        case LBK_TYPE_F32: return 4;
        case LBK_TYPE_Q4_K: return 144;
        case LBK_TYPE_Q5_K: return 176;
        case LBK_TYPE_IQ2_S: return 82;
        case LBK_TYPE_IQ3_S: return 110;
        default: return 0;
    }
}

bool dot_type(int32_t ty) {
    return ty == LBK_TYPE_Q4_K || ty == LBK_TYPE_Q5_K || ty == LBK_TYPE_IQ2_S || ty == LBK_TYPE_IQ3_S;
}

bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

// PackedMatrix::new (matrix.rs:26-150) for a descriptor.
int32_t check_matrix(const lbk_matrix* m, const char* what) {
    if (m == nullptr) return fail(LBK_INVALID_PARAMETER, what);
    uint64_t bb = block_bytes(m->type);
    if (bb == 0) return fail(LBK_UNSUPPORTED_TYPE, "unsupported GGML type", (uint64_t)m->type);
    if (m->layout != LBK_LAYOUT_GGUF && m->layout != LBK_LAYOUT_PLANAR)
        return fail(LBK_INVALID_PARAMETER, "unknown layout", (uint64_t)m->layout);
    if (m->layout == LBK_LAYOUT_PLANAR && m->type == LBK_TYPE_F32)
        return fail(LBK_INVALID_PARAMETER, "F32 matrices have no planar layout");
    if (m->input_width == 0 || m->output_width == 0) return fail(LBK_DIMENSION_MISMATCH, "zero tensor dimension");
    uint64_t be = m->type == LBK_TYPE_F32 ? 1 : LBK_QK_K;
    if (m->input_width % be != 0)
        return fail(LBK_DIMENSION_MISMATCH, "block-aligned matrix input width", 0, be, m->input_width);
    uint64_t nb = m->input_width / be;
    if (nb > UINT64_MAX / bb || nb * bb > UINT64_MAX / m->output_width)
        return fail(LBK_ARITHMETIC_OVERFLOW, "tensor encoded byte length");
    const uint64_t row_bytes = m->layout == LBK_LAYOUT_PLANAR ? (nb * bb + 15) & ~(uint64_t)15 : nb * bb;
    if (row_bytes > UINT64_MAX / m->output_width) return fail(LBK_ARITHMETIC_OVERFLOW, "tensor encoded byte length");
    uint64_t expected = row_bytes * m->output_width;
    if (m->bytes != expected) return fail(LBK_ENCODED_LENGTH_MISMATCH, "tensor encoded length", 0, expected, m->bytes);
    if (m->data == nullptr) return fail(LBK_INVALID_PARAMETER, "null matrix data");
    if (!aligned(m->data, 16)) return fail(LBK_INVALID_PARAMETER, "matrix data must be 16-byte aligned");
    return LBK_OK;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int32_t set_device(lbk_context* ctx) {
    cudaError_t e = cudaSetDevice(ctx->device);
    return e == cudaSuccess ? LBK_OK : cuda_fail(e, "cudaSetDevice");
}

lbk::MatrixRef mref(const lbk_matrix* m) {
    return lbk::MatrixRef{reinterpret_cast<const uint8_t*>(m->data), m->output_width, (int)(m->input_width / LBK_QK_K)};
}

// Common GEMV launch (quantized matrices).
int32_t run_gemv(lbk_context* ctx, const lbk_matrix* w, const float* x, const uint8_t* q8_in, uint8_t* q8_out,
                 float* y, float scale, int mode, int32_t* block_sums, const uint8_t* const* mat_table,
                 const lbk_routed* sel, cudaStream_t stream, uint64_t mat_count = 0) {
    lbk::GemvArgs a{};
    a.mat_count = mat_count;
    a.w = mref(w);
    a.x = x;
    a.q8_in = q8_in;
    a.q8_out = q8_out;
    a.y = y;
    a.scale = scale;
    a.mode = mode;
    a.block_sums = block_sums;
    a.mat_table = mat_table;
    a.sel = sel;
    a.status = ctx->status;
    a.tables = ctx->tables();
    lbk::gemv_plan(w->type, a.w.nb, &a.tpr, &a.tail_slots);
    if (lbk::gemv_smem_required(w->type, a.w.nb, a.tail_slots) > lbk::kMaxSmem)
        return fail(LBK_INVALID_PARAMETER, "input_width too large for the shared-memory activation image", 0, 0,
                    (uint64_t)a.w.nb * LBK_QK_K);
    cudaError_t e = lbk::launch_gemv(w->type, w->layout, a, ctx->sm_count, stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "gemv launch");
}

int32_t run_f32_gemv(lbk_context* ctx, const lbk_matrix* w, const float* x, uint64_t tokens, float* y,
                     cudaStream_t stream) {
    lbk::RouterArgs r{};
    r.w = reinterpret_cast<const float*>(w->data);
    r.x = x;
    r.logits = y;
    r.hidden = w->input_width;
    r.experts = w->output_width;
    r.tokens = tokens;
    r.status = ctx->status;
    cudaError_t e = lbk::launch_router(r, LBK_ROUTER_SEQUENTIAL, ctx->sm_count, stream);
    return e == cudaSuccess ? ok() : cuda_fail(e, "router launch");
}

struct WsLayout {
    uint64_t rcounter, logits, partials, q8x, routed, h, hq, counters, dcounters, counter_words, dots, g, u, total;
    uint64_t grp_n, grp, grp_pairs;  // grouped kernels (T >= 2): group count, groups, grouped pairs
    uint64_t rflag, rreaders;        // single token: routing-published flag, and the down CTAs that have read it
    uint64_t tc_grp_n, tc_grp, tc_dots;  // expert-parallel items on the tensor cores: groups of <= 32, gate|up dots
};

// Groups of at most 32 pairs over E experts: each expert's pairs split into
// ceil(n_e / 32) runs, at most E + pairs / 32 in all.
uint64_t tc_groups_max(uint64_t experts, uint64_t pairs) { return experts + pairs / 32 + 1; }

uint64_t up256(uint64_t v) { return (v + 255) & ~(uint64_t)255; }

// Workspace of one MoE call. Bytes 0-15 sit at the same place for every
// layer and token count: the router's arrival counter (byte 0), the
// single-token routing flag (byte 4) and the count of down CTAs that have
// read it (byte 8). Each is back at zero when a call ends, so a workspace
// stays valid across calls of different shapes once it was zero-filled. The
// other arrival counters ([gate/up h blocks][down combine blocks]) move with
// the shape and are zeroed by the router kernel of every call.
WsLayout moe_ws(const lbk_moe_layer* L, uint64_t T, uint64_t k) {
    WsLayout o{};
    uint64_t slots = T * (k + 1);
    uint64_t nbh = L->H / LBK_QK_K, nbf = L->F / LBK_QK_K;
    o.rcounter = 0;
    o.rflag = 4;
    o.rreaders = 8;
    o.counters = 16;
    o.dcounters = o.counters + slots * nbf * 4;
    const uint64_t cend = o.dcounters + T * ((L->H + lbk::kMoeDownCombineRows - 1) / lbk::kMoeDownCombineRows) * 4;
    o.counter_words = (cend - o.counters) / 4;
    uint64_t off = up256(cend);
    o.dots = off;  // down row dots [T][k+1][H]
    off = up256(off + slots * L->H * 4);
    o.logits = off;
    off = up256(off + T * L->E * 4);
    o.partials = off;
    off = up256(off + lbk::router_partials_floats(L->H, L->E, T) * 4);
    o.q8x = off;
    off = up256(off + T * nbh * lbk::kQ8IBytes);  // internal Q8_K images
    o.routed = off;
    off = up256(off + T * (k ? k : 1) * sizeof(lbk_routed));
    o.h = off;
    off = up256(off + slots * L->F * 4);
    o.hq = off;
    off = up256(off + slots * nbf * lbk::kQ8IBytes);
    o.g = off;  // per-expert path: gate / up scratch, q8 scratch
    off = up256(off + L->F * 4);
    o.u = off;
    off = up256(off + L->F * 4 + (L->F > L->H ? L->F : L->H) / LBK_QK_K * LBK_Q8K_BLOCK_BYTES);
    if (T >= 2) {  // the grouping of a several-token call: [count][groups {expert, first, pairs, 0}][pairs]
        const uint64_t pairs = T * (k ? k : 1);
        o.grp_n = off;
        o.grp = off + 16;
        o.grp_pairs = o.grp + pairs * 16;
        off = up256(o.grp_pairs + pairs * 4);
        if (k == 1) {  // expert-parallel items: the tensor-core gate/up (groups of <= 32, dots [pairs][2F])
            o.tc_grp_n = off;
            o.tc_grp = off + 16;
            off = up256(o.tc_grp + tc_groups_max(L->E_local, pairs) * 16);
            o.tc_dots = off;
            off = up256(off + pairs * 2 * L->F * 4);
        }
    }
    o.total = off;
    return o;
}

__global__ void check_routed_kernel(const lbk_routed* routed, uint64_t tokens, uint64_t k, uint64_t experts,
                                    lbk::DeviceStatus* st) {
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < tokens; t += (uint64_t)gridDim.x * blockDim.x) {
        const lbk_routed* r = routed + t * k;
        for (uint64_t i = 0; i < k; i++) {  // moe.rs:282-304
            float c = r[i].coefficient;
            if (!isfinite(c)) {
                lbk::report(st, LBK_NON_FINITE_VALUE, t * k + i, __float_as_uint(c));
                return;
            }
            if (i > 0 && r[i].expert_id == r[i - 1].expert_id) {
                lbk::report(st, LBK_DUPLICATE_ROUTED_EXPERT, r[i].expert_id, 0);
                return;
            }
            if (i > 0 && r[i].expert_id < r[i - 1].expert_id) {
                lbk::report(st, LBK_ROUTED_EXPERT_ORDER, r[i].expert_id, r[i - 1].expert_id);
                return;
            }
            if (r[i].expert_id >= experts) {
                lbk::report(st, LBK_INVALID_PARAMETER, r[i].expert_id, 0);
                return;
            }
        }
    }
}

__global__ void fill_zero_kernel(float* p, uint64_t n, const lbk::DeviceStatus* st) {
    if (lbk::status_set(st)) return;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        p[i] = 0.0f;
}

std::mutex g_attr_mu;
std::set<std::pair<int, const void*>> g_attr_done;

// Records a trace event; inside a stream capture it becomes an event-record
// node of the graph (cudaEventRecordExternal), outside it is a plain record.
void trace_record(cudaEvent_t ev, cudaStream_t st, unsigned int capture_flags) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(ev, st, capture_flags);
    else
        cudaEventRecord(ev, st);
}

}  // namespace

namespace lbk {
cudaError_t ensure_max_smem(const void* kernel) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (g_attr_done.count({dev, kernel})) return cudaSuccess;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return e;
    // the per-block limit covers static + dynamic shared memory
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kMaxSmem - fa.sharedSizeBytes));
    if (e == cudaSuccess) g_attr_done.insert({dev, kernel});
    return e;
}
}  // namespace lbk

// ===================================================================== ABI

LBK_API int32_t lbk_abi_version(void) { return LBK_ABI_VERSION; }

LBK_API const char* lbk_backend_name(void) { return "cuda_sm100a_q8_k"; }

LBK_API void lbk_last_error_detail(lbk_error_detail* out) {
    if (out) *out = g_err;
}

LBK_API int32_t lbk_context_create(int32_t device, lbk_context** out) {
    if (out == nullptr) return fail(LBK_INVALID_PARAMETER, "null output pointer");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) return fail(LBK_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= count) return fail(LBK_INVALID_PARAMETER, "device index", (uint64_t)device);
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    if (prop.major != 10) return fail(LBK_NO_DEVICE, "this build targets sm_100a (B200)", 0, 100, (uint64_t)(prop.major * 10 + prop.minor));
    lbk_context* c = new lbk_context{};
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    void* p = nullptr;
    // [status 32 B][scratch_min 8 B .. 256][iq2s grid 8 KB][iq3s grid 2 KB]
    // [IQ2 code image 128 KB][IQ3 grid image 64 KB]
    static_assert(sizeof(lbk::DeviceStatus) <= 32, "status word layout");
    const size_t img_off = 256 + sizeof(lbk_iq2s_grid) + sizeof(lbk_iq3s_grid);
    const size_t total = img_off + lbk::kIq2CodeBytes + lbk::kIq3GridBytes;
    if ((e = cudaMalloc(&p, total)) != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaMalloc context");
    }
    uint8_t* base = static_cast<uint8_t*>(p);
    c->status = reinterpret_cast<lbk::DeviceStatus*>(base);
    c->scratch_min = reinterpret_cast<unsigned long long*>(base + 32);
    c->iq2s = reinterpret_cast<uint64_t*>(base + 256);
    c->iq3s = reinterpret_cast<uint32_t*>(base + 256 + sizeof(lbk_iq2s_grid));
    c->img_iq2 = reinterpret_cast<uint32_t*>(base + img_off);
    c->img_iq3 = reinterpret_cast<uint32_t*>(base + img_off + lbk::kIq2CodeBytes);
    e = cudaMemset(base, 0, 256);
    if (e == cudaSuccess) e = cudaMemcpy(c->iq2s, lbk_iq2s_grid, sizeof(lbk_iq2s_grid), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(c->iq3s, lbk_iq3s_grid, sizeof(lbk_iq3s_grid), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = lbk::launch_build_tables(c->iq2s, c->iq3s, c->img_iq2, c->img_iq3, nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        delete c;
        return cuda_fail(e, "upload codebooks");
    }
    *out = c;
    return ok();
}

LBK_API int32_t lbk_context_destroy(lbk_context* ctx) {
    if (ctx == nullptr) return ok();
    cudaSetDevice(ctx->device);
    cudaFree(ctx->status);
    delete ctx;
    return ok();
}

LBK_API int32_t lbk_context_sync_status(lbk_context* ctx, void* stream, lbk_error_detail* detail) {
    if (ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null context");
    if (int32_t s = set_device(ctx)) return s;
    cudaError_t e = cudaStreamSynchronize(as_stream(stream));
    if (e != cudaSuccess) return cuda_fail(e, "stream synchronize");
    lbk::DeviceStatus st;
    if ((e = cudaMemcpy(&st, ctx->status, sizeof(st), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "read status");
    if ((e = cudaMemset(ctx->status, 0, sizeof(st))) != cudaSuccess) return cuda_fail(e, "clear status");
    lbk_error_detail d{};
    d.status = st.status;
    d.index = st.index;
    d.bits = st.bits;
    if (st.status != 0) std::snprintf(d.message, sizeof(d.message), "device-detected status %d", st.status);
    if (detail) *detail = d;
    g_err = d;
    return st.status;
}

LBK_API int32_t lbk_required_q8k_bytes(uint64_t input_width, uint64_t* bytes) {
    if (bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null output pointer");
    if (input_width == 0 || input_width % LBK_QK_K != 0)
        return fail(LBK_DIMENSION_MISMATCH, "Q8_K input width", 0, LBK_QK_K, input_width);
    *bytes = input_width / LBK_QK_K * LBK_Q8K_BLOCK_BYTES;
    return ok();
}

LBK_API int32_t lbk_matrix_bytes(int32_t type, uint64_t input_width, uint64_t output_width, uint64_t* bytes) {
    if (bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null output pointer");
    uint64_t bb = block_bytes(type);
    if (bb == 0) return fail(LBK_UNSUPPORTED_TYPE, "unsupported GGML type", (uint64_t)type);
    uint64_t be = type == LBK_TYPE_F32 ? 1 : LBK_QK_K;
    if (input_width == 0 || output_width == 0 || input_width % be != 0)
        return fail(LBK_DIMENSION_MISMATCH, "block-aligned matrix input width", 0, be, input_width);
    *bytes = input_width / be * bb * output_width;
    return ok();
}

LBK_API int32_t lbk_planar_bytes(int32_t type, uint64_t input_width, uint64_t output_width, uint64_t* bytes) {
    if (bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null output pointer");
    if (!dot_type(type)) return fail(LBK_UNSUPPORTED_TYPE, "only packed types have a planar layout", (uint64_t)type);
    if (input_width == 0 || output_width == 0 || input_width % LBK_QK_K != 0)
        return fail(LBK_DIMENSION_MISMATCH, "block-aligned matrix input width", 0, LBK_QK_K, input_width);
    *bytes = ((input_width / LBK_QK_K * block_bytes(type) + 15) & ~(uint64_t)15) * output_width;
    return ok();
}

LBK_API int32_t lbk_quantize_q8k(lbk_context* ctx, const float* x, uint64_t n, uint8_t* q8, uint64_t q8_bytes,
                                 void* stream) {
    if (n == 0) return fail(LBK_ZERO_LOGICAL_ELEMENTS, "a row must contain at least one logical element");
    if (n % LBK_QK_K != 0) return fail(LBK_LOGICAL_ELEMENTS_NOT_DIVISIBLE, "logical elements not divisible", 0, LBK_QK_K, n);
    uint64_t expected = n / LBK_QK_K * LBK_Q8K_BLOCK_BYTES;
    if (q8_bytes != expected) return fail(LBK_ENCODED_LENGTH_MISMATCH, "Q8_K encoded row length", 0, expected, q8_bytes);
    if (ctx == nullptr || x == nullptr || q8 == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(q8, 4)) return fail(LBK_INVALID_PARAMETER, "q8 must be 4-byte aligned");
    if (int32_t s = set_device(ctx)) return s;
    cudaError_t e = lbk::launch_quantize_q8k_ws(x, n, q8, ctx->scratch_min, ctx->status, ctx->sm_count, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "quantize launch");
}

LBK_API int32_t lbk_vec_dot_q8k(lbk_context* ctx, const lbk_matrix* w, const uint8_t* q8, uint64_t q8_bytes, float* out,
                                int32_t* block_sums, void* stream) {
    if (w == nullptr) return fail(LBK_INVALID_PARAMETER, "null matrix");
    if (!dot_type(w->type)) return fail(LBK_UNSUPPORTED_TYPE, "unsupported dot type", (uint64_t)w->type);
    if (w->input_width == 0) return fail(LBK_ZERO_LOGICAL_ELEMENTS, "zero logical elements");
    if (w->input_width % LBK_QK_K != 0)
        return fail(LBK_LOGICAL_ELEMENTS_NOT_DIVISIBLE, "logical elements not divisible", 0, LBK_QK_K, w->input_width);
    if (int32_t s = check_matrix(w, "matrix")) return s;
    uint64_t expected = w->input_width / LBK_QK_K * LBK_Q8K_BLOCK_BYTES;
    if (q8_bytes != expected) return fail(LBK_ENCODED_LENGTH_MISMATCH, "packed dot Q8_K row length", 0, expected, q8_bytes);
    if (ctx == nullptr || q8 == nullptr || out == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(q8, 4)) return fail(LBK_INVALID_PARAMETER, "q8 must be 4-byte aligned");
    if (int32_t s = set_device(ctx)) return s;
    return run_gemv(ctx, w, nullptr, q8, nullptr, out, 0.0f, lbk::kGemvStore, block_sums, nullptr, nullptr,
                    as_stream(stream));
}

LBK_API int32_t lbk_gemv(lbk_context* ctx, const lbk_matrix* w, const float* x, float* y, uint8_t* q8_scratch,
                         uint64_t q8_scratch_bytes, void* stream) {
    if (int32_t s = check_matrix(w, "matrix")) return s;
    if (x == nullptr || y == nullptr || ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (w->type == LBK_TYPE_F32) {  // gemv_into on an F32 matrix: sequential f32 rows (gemv.rs:96-105)
        if (int32_t s = set_device(ctx)) return s;
        return run_f32_gemv(ctx, w, x, 1, y, as_stream(stream));
    }
    if (w->input_width % LBK_QK_K != 0)
        return fail(LBK_DIMENSION_MISMATCH, "Q8_K input width", 0, LBK_QK_K, w->input_width);
    uint64_t required = w->input_width / LBK_QK_K * LBK_Q8K_BLOCK_BYTES;
    if (q8_scratch != nullptr && q8_scratch_bytes < required)
        return fail(LBK_SCRATCH_TOO_SMALL, "Q8_K row scratch", 0, required, q8_scratch_bytes);
    if (!aligned(x, 16)) return fail(LBK_INVALID_PARAMETER, "x must be 16-byte aligned");
    if (q8_scratch != nullptr && !aligned(q8_scratch, 4)) return fail(LBK_INVALID_PARAMETER, "q8 scratch must be 4-byte aligned");
    if (int32_t s = set_device(ctx)) return s;
    return run_gemv(ctx, w, x, nullptr, q8_scratch, y, 0.0f, lbk::kGemvStore, nullptr, nullptr, nullptr,
                    as_stream(stream));
}

LBK_API int32_t lbk_gemv_accumulate_scaled(lbk_context* ctx, const lbk_matrix* w, const float* x, float* y, float scale,
                                           uint8_t* q8_scratch, uint64_t q8_scratch_bytes, void* stream) {
    if (!std::isfinite(scale)) return fail(LBK_NON_FINITE_VALUE, "accumulation scale", 0, 0, 0, f32_bits(scale));
    if (int32_t s = check_matrix(w, "matrix")) return s;
    if (x == nullptr || y == nullptr || ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (w->type == LBK_TYPE_F32) return fail(LBK_UNSUPPORTED_TYPE, "F32 accumulate is not on this path", LBK_TYPE_F32);
    uint64_t required = w->input_width / LBK_QK_K * LBK_Q8K_BLOCK_BYTES;
    if (q8_scratch != nullptr && q8_scratch_bytes < required)
        return fail(LBK_SCRATCH_TOO_SMALL, "Q8_K row scratch", 0, required, q8_scratch_bytes);
    if (!aligned(x, 16)) return fail(LBK_INVALID_PARAMETER, "x must be 16-byte aligned");
    if (int32_t s = set_device(ctx)) return s;
    return run_gemv(ctx, w, x, nullptr, q8_scratch, y, scale, lbk::kGemvAccumulate, nullptr, nullptr, nullptr,
                    as_stream(stream));
}

LBK_API int32_t lbk_router_logits(lbk_context* ctx, const lbk_matrix* router, const float* x, uint64_t tokens,
                                  float* logits, int32_t mode, void* stream) {
    if (int32_t s = check_matrix(router, "router")) return s;
    if (router->type != LBK_TYPE_F32) return fail(LBK_UNSUPPORTED_TYPE, "router must be F32", (uint64_t)router->type);
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    if (mode != LBK_ROUTER_SEQUENTIAL && mode != LBK_ROUTER_TREE) return fail(LBK_INVALID_PARAMETER, "router mode");
    if (ctx == nullptr || x == nullptr || logits == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = set_device(ctx)) return s;
    if (mode == LBK_ROUTER_SEQUENTIAL) return run_f32_gemv(ctx, router, x, tokens, logits, as_stream(stream));
    return fail(LBK_INVALID_PARAMETER, "tree order needs a workspace: use lbk_moe_forward");
}

LBK_API int32_t lbk_route_topk(lbk_context* ctx, const float* logits, const float* selection_bias, uint64_t expert_count,
                               uint64_t tokens, uint32_t k, float weight_scale, lbk_routed* routed, void* stream) {
    if (k == 0 || k > expert_count) return fail(LBK_ROUTING_TOPK, "expert_used_count", 0, expert_count, k);
    if (!std::isfinite(weight_scale))
        return fail(LBK_NON_FINITE_ROUTING_VALUE, "weight_scale", 0, 0, 0, f32_bits(weight_scale));
    if (expert_count > 1024 || k > 32) return fail(LBK_INVALID_PARAMETER, "this build routes at most 1024 experts, k <= 32");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    if (ctx == nullptr || logits == nullptr || selection_bias == nullptr || routed == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = set_device(ctx)) return s;
    lbk::TopkArgs a{logits, selection_bias, expert_count, tokens, k, weight_scale, routed, ctx->status};
    cudaError_t e = lbk::launch_topk(a, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "top-k launch");
}

namespace {

// SwiGluExpert::new (activation.rs:13-22) plus PackedMatrix checks.
int32_t check_expert(const lbk_expert* ex) {
    if (ex == nullptr) return fail(LBK_INVALID_PARAMETER, "null expert");
    if (int32_t s = check_matrix(&ex->gate, "gate")) return s;
    if (int32_t s = check_matrix(&ex->up, "up")) return s;
    if (int32_t s = check_matrix(&ex->down, "down")) return s;
    if (ex->gate.input_width != ex->up.input_width)
        return fail(LBK_DIMENSION_MISMATCH, "SwiGLU gate/up input width", 0, ex->gate.input_width, ex->up.input_width);
    if (ex->gate.output_width != ex->up.output_width)
        return fail(LBK_DIMENSION_MISMATCH, "SwiGLU gate/up hidden width", 0, ex->gate.output_width, ex->up.output_width);
    if (ex->gate.output_width != ex->down.input_width)
        return fail(LBK_DIMENSION_MISMATCH, "SwiGLU down input width", 0, ex->gate.output_width, ex->down.input_width);
    for (const lbk_matrix* m : {&ex->gate, &ex->up, &ex->down})
        if (!dot_type(m->type)) return fail(LBK_UNSUPPORTED_TYPE, "expert matrices must be quantized", (uint64_t)m->type);
    return LBK_OK;
}

// gate/up GEMVs, SwiGLU and the scaled down accumulation for one expert
// (activation.rs:104-144); the expert may be selected on the device.
int32_t expert_accumulate(lbk_context* ctx, const lbk_expert* ex, const float* x, float* dst, float coef, float* g,
                          float* u, uint8_t* q8, const uint8_t* const* tg, const uint8_t* const* tu,
                          const uint8_t* const* td, const lbk_routed* sel, cudaStream_t stream,
                          uint64_t table_count = 0) {
    if (int32_t s = run_gemv(ctx, &ex->gate, x, nullptr, q8, g, 0.0f, lbk::kGemvStore, nullptr, tg, sel, stream,
                             table_count))
        return s;
    if (int32_t s = run_gemv(ctx, &ex->up, x, nullptr, q8, u, 0.0f, lbk::kGemvStore, nullptr, tu, sel, stream,
                             table_count))
        return s;
    cudaError_t e = lbk::launch_swiglu(g, u, g, ex->gate.output_width, ctx->status, stream);
    if (e != cudaSuccess) return cuda_fail(e, "swiglu launch");
    return run_gemv(ctx, &ex->down, g, nullptr, q8, dst, coef, lbk::kGemvAccumulate, nullptr, td, sel, stream,
                    table_count);
}

}  // namespace

LBK_API int32_t lbk_expert_workspace_bytes(const lbk_expert* expert, uint64_t* bytes) {
    if (bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null output pointer");
    if (int32_t s = check_expert(expert)) return s;
    uint64_t F = expert->gate.output_width, H = expert->gate.input_width;
    uint64_t w = (F > H ? F : H) / LBK_QK_K;
    *bytes = up256(F * 4) * 2 + up256(w * LBK_Q8K_BLOCK_BYTES);
    return ok();
}

LBK_API int32_t lbk_expert_swiglu_accumulate(lbk_context* ctx, const lbk_expert* expert, const float* x, float* dst,
                                             float coefficient, void* workspace, uint64_t workspace_bytes,
                                             void* stream) {
    if (!std::isfinite(coefficient))
        return fail(LBK_NON_FINITE_VALUE, "expert coefficient", 0, 0, 0, f32_bits(coefficient));
    if (int32_t s = check_expert(expert)) return s;
    uint64_t need = 0;
    lbk_expert_workspace_bytes(expert, &need);
    if (workspace_bytes < need) return fail(LBK_SCRATCH_TOO_SMALL, "SwiGLU gate/up", 0, need, workspace_bytes);
    if (ctx == nullptr || x == nullptr || dst == nullptr || workspace == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(x, 16) || !aligned(workspace, 256)) return fail(LBK_INVALID_PARAMETER, "x 16-byte / workspace 256-byte alignment");
    if (int32_t s = set_device(ctx)) return s;
    uint64_t F = expert->gate.output_width;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* g = reinterpret_cast<float*>(ws);
    float* u = reinterpret_cast<float*>(ws + up256(F * 4));
    uint8_t* q8 = ws + 2 * up256(F * 4);
    return expert_accumulate(ctx, expert, x, dst, coefficient, g, u, q8, nullptr, nullptr, nullptr, nullptr,
                             as_stream(stream));
}

// ------------------------------------------------------------- MoE layer

namespace {

// A layer over the resident experts w->experts[0, expert_count), which are the
// global experts [first, first + expert_count) of a router over E_route.
int32_t layer_create(lbk_context* ctx, const lbk_moe_weights* w, uint64_t E_route, uint64_t first, void* stream,
                     lbk_moe_layer** out) {
    if (out == nullptr || w == nullptr || ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    *out = nullptr;
    if (w->expert_count == 0 || w->experts == nullptr) return fail(LBK_DIMENSION_MISMATCH, "expert count", 0, 1, 0);
    if (int32_t s = check_expert(&w->shared)) return s;
    if (int32_t s = check_matrix(&w->router, "router")) return s;
    if (w->router.type != LBK_TYPE_F32) return fail(LBK_UNSUPPORTED_TYPE, "router must be F32", (uint64_t)w->router.type);
    const uint64_t H = w->shared.gate.input_width, F = w->shared.gate.output_width, E = w->expert_count;
    if (first > E_route || E > E_route - first)
        return fail(LBK_DIMENSION_MISMATCH, "resident experts beyond the router's experts", first, E_route, first + E);
    if (w->router.input_width != H) return fail(LBK_DIMENSION_MISMATCH, "router input width", 0, H, w->router.input_width);
    if (w->router.output_width != E_route)
        return fail(LBK_DIMENSION_MISMATCH, "router output width", 0, E_route, w->router.output_width);
    if (w->shared.down.output_width != H) return fail(LBK_DIMENSION_MISMATCH, "MoE output", 0, H, w->shared.down.output_width);
    if (w->top_k == 0 || w->top_k > E_route) return fail(LBK_ROUTING_TOPK, "expert_used_count", 0, E_route, w->top_k);
    if (!std::isfinite(w->weight_scale))
        return fail(LBK_NON_FINITE_ROUTING_VALUE, "weight_scale", 0, 0, 0, f32_bits(w->weight_scale));
    if (E_route > 1024 || w->top_k > 32) return fail(LBK_INVALID_PARAMETER, "this build routes at most 1024 experts, k <= 32");
    if (w->selection_bias == nullptr) return fail(LBK_INVALID_PARAMETER, "null selection bias");
    if (H % LBK_QK_K != 0 || F % LBK_QK_K != 0) return fail(LBK_DIMENSION_MISMATCH, "Q8_K input width", 0, LBK_QK_K, H);
    for (uint64_t e = 0; e < E; e++) {
        const lbk_expert* ex = &w->experts[e];
        if (int32_t s = check_expert(ex)) {
            g_err.index = e;
            return s;
        }
        if (ex->gate.input_width != H) return fail(LBK_DIMENSION_MISMATCH, "routed expert input width", e, H, ex->gate.input_width);
        if (ex->down.output_width != H) return fail(LBK_DIMENSION_MISMATCH, "routed expert output width", e, H, ex->down.output_width);
        if (ex->gate.output_width != F) return fail(LBK_DIMENSION_MISMATCH, "routed expert hidden width", e, F, ex->gate.output_width);
    }
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);

    auto* L = new lbk_moe_layer{};
    L->ctx = ctx;
    L->E = E_route;
    L->E_local = E;
    L->first = first;
    L->H = H;
    L->F = F;
    L->k = w->top_k;
    L->weight_scale = w->weight_scale;
    L->w = *w;
    L->experts.assign(w->experts, w->experts + E);
    L->w.experts = nullptr;
    L->gate_type = w->experts[0].gate.type;
    L->down_type = w->experts[0].down.type;
    L->sgate_type = w->shared.gate.type;
    L->sdown_type = w->shared.down.type;
    bool uniform = true, planar = w->shared.gate.layout == LBK_LAYOUT_PLANAR && w->shared.up.layout == LBK_LAYOUT_PLANAR &&
                                  w->shared.down.layout == LBK_LAYOUT_PLANAR && w->shared.up.type == w->shared.gate.type;
    bool same_layout = true;
    for (uint64_t e = 0; e < E; e++) {
        const lbk_expert& ex = w->experts[e];
        uniform &= ex.gate.type == L->gate_type && ex.up.type == w->experts[0].up.type && ex.down.type == L->down_type;
        planar &= ex.gate.layout == LBK_LAYOUT_PLANAR && ex.up.layout == LBK_LAYOUT_PLANAR && ex.down.layout == LBK_LAYOUT_PLANAR;
        same_layout &= ex.gate.layout == w->experts[0].gate.layout && ex.up.layout == w->experts[0].up.layout &&
                       ex.down.layout == w->experts[0].down.layout;
    }
    // Routed experts are slices of one stacked tensor per projection in the
    // reference schema (bridge-model-hy3/src/schema.rs:219-243), so they share
    // types and layouts; the device-side expert selection relies on it.
    if (!uniform || !same_layout) {
        delete L;
        return fail(LBK_INVALID_PARAMETER, "routed experts must share each projection's type and layout");
    }
    uniform &= w->experts[0].up.type == L->gate_type;
    // the fused kernels: the register-streamed ones (any shape, top-k <= 8)
    // or the bulk-copy-staged ones, which also take the checkpoint's IQ
    // shared-expert types
    const bool staged = lbk::moe_gate_up_tma_supported(L->gate_type, L->sgate_type, (int)(H / LBK_QK_K)) &&
                        lbk::moe_down_tma_supported(L->down_type, L->sdown_type, (int)(F / LBK_QK_K)) && L->k <= 16;
    L->fused = uniform && planar &&
               ((lbk::moe_fused_supported(L->gate_type, L->sgate_type, L->down_type, L->sdown_type) &&
                 L->k + 1 <= (uint64_t)lbk::kMoeDownMaxSlots) ||
                staged);

    std::vector<const uint8_t*> ptrs(3 * E);
    for (uint64_t e = 0; e < E; e++) {
        ptrs[e] = static_cast<const uint8_t*>(w->experts[e].gate.data);
        ptrs[E + e] = static_cast<const uint8_t*>(w->experts[e].up.data);
        ptrs[2 * E + e] = static_cast<const uint8_t*>(w->experts[e].down.data);
    }
    void* d = nullptr;
    cudaError_t e = cudaMalloc(&d, 3 * E * sizeof(void*));
    if (e != cudaSuccess) {
        delete L;
        return cuda_fail(e, "cudaMalloc expert table");
    }
    L->d_gate = static_cast<const uint8_t**>(d);
    L->d_up = L->d_gate + E;
    L->d_down = L->d_gate + 2 * E;
    e = cudaMemcpyAsync(d, ptrs.data(), 3 * E * sizeof(void*), cudaMemcpyHostToDevice, st);
    // One scale scan per matrix (validate_scales), results gathered at the sync.
    auto scan = [&](const lbk_matrix& m) {
        if (e != cudaSuccess) return;
        e = lbk::launch_validate_scales(m.type, m.layout, static_cast<const uint8_t*>(m.data), m.output_width,
                                        (int)(m.input_width / LBK_QK_K), ctx->scratch_min, ctx->status, st);
    };
    for (uint64_t x = 0; x < E; x++) {
        scan(w->experts[x].gate);
        scan(w->experts[x].up);
        scan(w->experts[x].down);
    }
    scan(w->shared.gate);
    scan(w->shared.up);
    scan(w->shared.down);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        cudaFree(d);
        delete L;
        return cuda_fail(e, "layer registration");
    }
    lbk_error_detail det{};
    int32_t s = lbk_context_sync_status(ctx, stream, &det);
    if (s != LBK_OK) {
        cudaFree(d);
        delete L;
        g_err = det;
        return s;
    }
    *out = L;
    return ok();
}

}  // namespace

namespace lbk {

int32_t host_fail(int32_t status, const char* msg, uint64_t index, uint64_t expected, uint64_t actual, uint32_t bits) {
    return fail(status, msg, index, expected, actual, bits);
}

int32_t host_ok() { return ok(); }

int32_t host_set_device(lbk_context* ctx) { return set_device(ctx); }

int32_t layer_create_owned(lbk_context* ctx, const lbk_moe_weights* w, uint64_t global_experts, uint64_t first_expert,
                           void* stream, void* owned, lbk_moe_layer** out) {
    const int32_t s = layer_create(ctx, w, global_experts, first_expert, stream, out);
    if (s == LBK_OK) {
        (*out)->owned = owned;
        if ((*out)->E_local != (*out)->E) (*out)->group_min = 0;  // an expert-parallel share (see lbk_ep_layer_create)
    }
    return s;
}

}  // namespace lbk

LBK_API int32_t lbk_moe_layer_create(lbk_context* ctx, const lbk_moe_weights* w, void* stream, lbk_moe_layer** out) {
    return layer_create(ctx, w, w ? w->expert_count : 0, 0, stream, out);
}

LBK_API int32_t lbk_ep_layer_create(lbk_context* ctx, const lbk_moe_weights* w, uint64_t global_experts,
                                    uint64_t first_expert, void* stream, lbk_moe_layer** out) {
    const int32_t st = layer_create(ctx, w, global_experts, first_expert, stream, out);
    // The expert-parallel passes with host-known sizes (items without the
    // shared expert, the shared-only combine) measured no faster grouped: off
    // unless asked for. Device-counted items choose by their capacity per
    // expert (lbk_ep_items_forward_counted).
    if (st == LBK_OK && out != nullptr && *out != nullptr) (*out)->group_min = 0;
    return st;
}

LBK_API int32_t lbk_moe_layer_trace(lbk_moe_layer* layer, int32_t enable) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (int32_t s = set_device(layer->ctx)) return s;
    if (enable && !layer->tracing) {
        for (int i = 0; i < 4; i++) {
            cudaError_t e = cudaEventCreate(&layer->trace[i]);
            if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
        }
        layer->tracing = true;
    } else if (!enable && layer->tracing) {
        for (int i = 0; i < 4; i++) cudaEventDestroy(layer->trace[i]);
        layer->tracing = false;
    }
    return ok();
}

LBK_API int32_t lbk_moe_layer_trace_read(lbk_moe_layer* layer, float ms[3]) {
    if (layer == nullptr || ms == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!layer->tracing) return fail(LBK_INVALID_PARAMETER, "tracing is not enabled");
    if (int32_t s = set_device(layer->ctx)) return s;
    cudaError_t e = cudaEventSynchronize(layer->trace[3]);
    for (int i = 0; i < 3 && e == cudaSuccess; i++) e = cudaEventElapsedTime(&ms[i], layer->trace[i], layer->trace[i + 1]);
    return e == cudaSuccess ? ok() : cuda_fail(e, "trace read");
}

LBK_API int32_t lbk_moe_layer_destroy(lbk_moe_layer* layer) {
    if (layer == nullptr) return ok();
    cudaSetDevice(layer->ctx->device);
    lbk_moe_layer_trace(layer, 0);
    cudaFree(layer->d_gate);
    if (layer->owned) cudaFree(layer->owned);
    delete layer;
    return ok();
}

LBK_API int32_t lbk_moe_layer_fused(const lbk_moe_layer* layer) { return layer && layer->fused ? 1 : 0; }

LBK_API int32_t lbk_moe_layer_set_wait_limit(lbk_moe_layer* layer, uint32_t polls) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    layer->wait_limit = polls;
    return ok();
}

LBK_API int32_t lbk_moe_layer_set_tensor_cores(lbk_moe_layer* layer, uint64_t min_pairs_per_expert) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    layer->tc_min = min_pairs_per_expert;
    return ok();
}

LBK_API int32_t lbk_moe_layer_set_grouping(lbk_moe_layer* layer, uint64_t min_tokens) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    layer->group_min = min_tokens;
    layer->group_set = true;
    return ok();
}

LBK_API int32_t lbk_moe_workspace_bytes(const lbk_moe_layer* layer, uint64_t tokens, uint64_t* bytes) {
    if (layer == nullptr || bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    *bytes = moe_ws(layer, tokens, layer->k).total;
    return ok();
}

namespace {

// Per-warp time of one lane slot of a unit (one half block, microseconds, 16
// warps per SM), measured on B200 for the bulk-copy-staged kernels.
double hb_cost_us(int32_t ty) {
    switch (ty) {
        case LBK_TYPE_IQ2_S: return 0.034;
        case LBK_TYPE_IQ3_S: return 0.028;
        case LBK_TYPE_Q4_K: return 0.04;
        default: return 0.045;
    }
}

// The same for one lane slot of a gate/up unit (gate and up half blocks of a
// row decoded together), from per-warp globaltimer stamps of a config-3
// layer on B200: 0.91 us per IQ2_S unit, 1.52 us per Q4_K unit (32 slots).
double gu_hb_cost_us(int32_t ty) {
    switch (ty) {
        case LBK_TYPE_IQ2_S: return 0.0285;
        case LBK_TYPE_Q4_K: return 0.0476;
        default: return hb_cost_us(ty);
    }
}

// Routed CTAs out of `ctas` so that the routed and the shared role finish
// together: role time = fixed + work / (its warps).
long split_roles(unsigned ctas, int warps, double work_r, double fixed_r, double work_s, double fixed_s) {
    long best = 1;
    double best_t = 1e300;
    for (long r = 1; r < (long)ctas; r++) {
        const double tr = fixed_r + work_r / (double)(r * warps);
        const double ts = fixed_s + work_s / (double)((ctas - r) * warps);
        const double t = tr > ts ? tr : ts;
        if (t < best_t) {
            best_t = t;
            best = r;
        }
    }
    return best;
}

// What one fused expert stage computes.
struct MoeMode {
    uint64_t k;          // routed slots per token (the routing holds tokens * k entries)
    bool shared;         // also the shared expert (slot k)
    bool combine;        // form `out`; else leave the row dots in `dots`
    const uint8_t* q8x;  // the tokens' Q8_K images (null: the workspace's, from the router kernel)
    float* dots;         // row dots [T][dots_slots][H] (null: the workspace's)
    uint32_t dots_slots;
    const uint32_t* d_items = nullptr;  // items counted on the device (T is then the capacity)
    bool grouped = false;               // run the grouped kernels whatever the layer's rule
    bool tc = false;                    // grouped items: gate/up on the tensor cores (IQ2_S)
    // items returned in place: item t's row dots to its home buffer (see
    // MoeDownArgs::ret_addr), with no local dots
    const uint2* ret = nullptr;
    uint8_t* const* ret_peers = nullptr;
    uint64_t ret_off = 0;
};

MoeMode full_mode(const lbk_moe_layer* L) { return MoeMode{L->k, true, true, nullptr, nullptr, (uint32_t)(L->k + 1)}; }

// Share of a grouped item's per-half-block time spent decoding (once per
// group) rather than dotting (once per pair): IQ decode is most of a half
// block's work, a K-quant half block is dotted straight from its packed bytes.
double grp_decode_share(int32_t ty) { return ty == LBK_TYPE_IQ2_S || ty == LBK_TYPE_IQ3_S ? 0.6 : 0.15; }

// Expected routed groups of a call: pairs spread over the experts hit, cut
// into runs of at most gsize.
double grp_groups_est(double pairs, double experts, double gsize) {
    const double hit = experts * (1.0 - std::pow(1.0 - 1.0 / experts, pairs));
    const double runs = std::ceil(pairs / gsize);
    return 1.15 * (hit > runs ? hit : runs);
}

// The expert-parallel items' down projection on the tensor cores: IQ
// weights, one dots row per item, no shared expert, no combine.
bool tc_down_ok(const lbk_moe_layer* L, const MoeMode& m) {
    return m.tc && (L->down_type == LBK_TYPE_IQ3_S || L->down_type == LBK_TYPE_IQ2_S) &&
           (m.dots != nullptr || m.ret != nullptr) && m.dots_slots == 1 && !m.combine && !m.shared && m.k == 1;
}

// Expert stage of a several-token call on the grouped kernels: the routed
// pairs are grouped by expert, then gate/up + SwiGLU and down (+ combine) run
// with each weight half block decoded once per group. Same results, bit for
// bit, as the per-(token, slot) kernels.
int32_t moe_experts_grouped(lbk_moe_layer* L, uint64_t T, const lbk_routed* routed, float* out, uint8_t* ws,
                            const WsLayout& o, cudaStream_t st, const MoeMode& mode) {
    lbk_context* ctx = L->ctx;
    cudaError_t e = cudaSuccess;
    const uint64_t nbh = L->H / LBK_QK_K, nbf = L->F / LBK_QK_K;
    const uint64_t K = mode.k;
    const unsigned ctas = (unsigned)ctx->sm_count;
    const lbk::GrpShape sgu = lbk::moe_gate_up_grp_shape(L->gate_type, L->sgate_type);
    const lbk::GrpShape sdn = lbk::moe_down_grp_shape(L->down_type, L->sdown_type);
    const uint32_t gr = std::min(sgu.routed, sdn.routed), gs = std::min(sgu.shared, sdn.shared);
    uint32_t* grp_n = reinterpret_cast<uint32_t*>(ws + o.grp_n);
    const uint4* grp = reinterpret_cast<const uint4*>(ws + o.grp);
    uint32_t* grp_pairs = reinterpret_cast<uint32_t*>(ws + o.grp_pairs);
    if (K > 0 && !(mode.tc && tc_down_ok(L, mode))) {  // (groups for the dp4a kernels)
        lbk::MoeGroupArgs ga{routed, T, K, L->E_local, gr, grp_n, const_cast<uint4*>(grp), grp_pairs, ctx->status,
                             mode.d_items};
        if ((e = lbk::launch_moe_group(ga, st)) != cudaSuccess) return cuda_fail(e, "moe grouping launch");
    }
    const double pairs = (double)(T * K);
    const double groups_r = K ? grp_groups_est(pairs, (double)L->E_local, gr) : 0.0;
    const double groups_s = std::ceil((double)T / gs);
    auto role_work = [&](int32_t ty, double groups, double n) {
        const double d = grp_decode_share(ty);
        return hb_cost_us(ty) * (d * groups + (1.0 - d) * n);
    };

    int slots_unused = 0;
    if (mode.tc) {
        // Gate/up of the items on the tensor cores: the pairs grouped again in
        // runs of up to 32 (the same stable order, so the pair list is
        // shared), one CTA per (group, gate or up, 128-row tile); then SwiGLU
        // and Q8_K of h per pair; the down projection stays on the grouped
        // kernel below. Bit-identical to the dp4a gate/up.
        uint32_t* tgn = reinterpret_cast<uint32_t*>(ws + o.tc_grp_n);
        uint4* tgrp = reinterpret_cast<uint4*>(ws + o.tc_grp);
        float* tdots = reinterpret_cast<float*>(ws + o.tc_dots);
        lbk::MoeGroupArgs gt{routed, T, K, L->E_local, 32, tgn, tgrp, grp_pairs, ctx->status, mode.d_items};
        if ((e = lbk::launch_moe_group(gt, st)) != cudaSuccess) return cuda_fail(e, "moe grouping launch");
        lbk::TcDotsArgs ta{};
        ta.q8 = mode.q8x;
        ta.q8_row_bytes = nbh * lbk::kQ8IBytes;
        ta.pair_tokens = grp_pairs;
        ta.dots = tdots;
        ta.dots_stride = 2 * L->F;
        ta.status = ctx->status;
        ta.tables = ctx->tables();
        ta.groups = tgrp;
        ta.ngroups = tgn;
        ta.gate = L->d_gate;
        ta.up = L->d_up;
        ta.experts = (uint32_t)L->E_local;
        ta.rows = (uint32_t)L->F;
        ta.nb = (uint32_t)nbh;
        ta.mats_per_group = 2;
        const uint64_t tiles = (L->F + 127) / 128;
        const uint64_t ctas_tc = tc_groups_max(L->E_local, T * K) * 2 * tiles;
        if ((e = lbk::launch_tc_dots(L->gate_type, ta, (uint32_t)ctas_tc, st)) != cudaSuccess)
            return cuda_fail(e, "tensor-core gate/up launch");
        lbk::TcSwigluArgs sa{tdots, grp_pairs, mode.d_items, (uint32_t)(T * K), (uint32_t)L->F, (uint32_t)nbf,
                             (uint32_t)(K + 1), ws + o.hq, ctx->status};
        if ((e = lbk::launch_tc_swiglu_quant(sa, ctx->sm_count, st)) != cudaSuccess) return cuda_fail(e, "SwiGLU launch");
        if (L->tracing) trace_record(L->trace[2], st, cudaEventRecordExternal);
        if (tc_down_ok(L, mode)) {
            // the down projection on the tensor cores too: per (group, 128-row
            // tile), each pair's h image against the expert's down rows, the
            // row dots scattered to the pair's item
            lbk::TcDotsArgs da = ta;
            da.q8 = ws + o.hq;
            da.q8_row_bytes = (K + 1) * nbf * lbk::kQ8IBytes;
            da.dots = mode.dots;
            da.dots_stride = L->H;
            da.gate = L->d_down;
            da.up = nullptr;
            da.rows = (uint32_t)L->H;
            da.nb = (uint32_t)nbf;
            da.mats_per_group = 1;
            da.out_by_token = true;
            da.ret_addr = mode.ret;
            da.ret_peers = mode.ret_peers;
            da.ret_off = mode.ret_off;
            const uint64_t dtiles = (L->H + 127) / 128;
            const uint64_t dctas = tc_groups_max(L->E_local, T * K) * dtiles;
            if ((e = lbk::launch_tc_dots(L->down_type, da, (uint32_t)dctas, st)) != cudaSuccess)
                return cuda_fail(e, "tensor-core down launch");
            if (L->tracing) trace_record(L->trace[3], st, cudaEventRecordExternal);
            return ok();
        }
    } else {
        lbk::MoeGateUpArgs g{};
        g.hidden = L->H;
        g.ffn = L->F;
        g.nb_h = (int)nbh;
        g.nb_f = (int)nbf;
        lbk::gemv_plan(L->gate_type, (int)nbh, &g.tpr_h, &slots_unused);
        g.tokens = T;
        g.k = K;
        g.experts = L->E_local;
        g.gate = L->d_gate;
        g.up = L->d_up;
        g.sgate = static_cast<const uint8_t*>(L->w.shared.gate.data);
        g.sup = static_cast<const uint8_t*>(L->w.shared.up.data);
        g.routed = routed;
        g.q8x = mode.q8x ? mode.q8x : ws + o.q8x;
        g.has_shared = mode.shared ? 1 : 0;
        g.h = reinterpret_cast<float*>(ws + o.h);
        g.hq = ws + o.hq;
        g.counters = reinterpret_cast<unsigned int*>(ws + o.counters);
        g.grp_n = grp_n;
        g.grp = grp;
        g.grp_pairs = grp_pairs;
        g.gsize_r = gr;
        g.gsize_s = gs;
        g.status = ctx->status;
        g.tables = ctx->tables();
        {
            const double hb = 2.0 * nbh * 2.0 * L->F;  // half blocks of one slot (gate + up)
            const long rc = K == 0 ? 0
                            : !mode.shared ? (long)ctas
                                           : split_roles(ctas, (int)sgu.warps, hb * role_work(L->gate_type, groups_r, pairs),
                                                         1.5, hb * role_work(L->sgate_type, groups_s, (double)T), 1.0);
            g.routed_ctas = (uint32_t)rc;
        }
        if ((e = lbk::launch_moe_gate_up_grp(L->gate_type, L->sgate_type, g, ctas, st)) != cudaSuccess)
            return cuda_fail(e, "moe grouped gate/up launch");
        if (L->tracing) trace_record(L->trace[2], st, cudaEventRecordExternal);
    }

    lbk::MoeDownArgs d{};
    d.hidden = L->H;
    d.ffn = L->F;
    d.nb_f = (int)nbf;
    lbk::gemv_plan(L->down_type, (int)nbf, &d.tpr_f, &slots_unused);
    d.tokens = T;
    d.k = K;
    d.experts = L->E_local;
    d.down = L->d_down;
    d.sdown = static_cast<const uint8_t*>(L->w.shared.down.data);
    d.routed = routed;
    d.hq = ws + o.hq;
    d.out = out;
    d.dots = mode.dots ? mode.dots : reinterpret_cast<float*>(ws + o.dots);
    d.dots_slots = mode.dots_slots;
    d.combine = mode.combine ? 1 : 0;
    d.has_shared = mode.shared ? 1 : 0;
    d.counters = reinterpret_cast<unsigned int*>(ws + o.dcounters);
    d.grp_n = grp_n;
    d.grp = grp;
    d.grp_pairs = grp_pairs;
    d.gsize_r = gr;
    d.gsize_s = gs;
    d.ret_addr = mode.ret;
    d.ret_peers = mode.ret_peers;
    d.ret_off = mode.ret_off;
    d.status = ctx->status;
    d.tables = ctx->tables();
    {
        const double lanes = (double)L->H * d.tpr_f;  // lane slots of one slot's rows
        const long rc = K == 0 ? 0
                        : !mode.shared ? (long)ctas
                                       : split_roles(ctas, (int)sdn.warps, lanes * role_work(L->down_type, groups_r, pairs),
                                                     2.0, lanes * role_work(L->sdown_type, groups_s, (double)T), 1.5);
        d.routed_ctas = (uint32_t)rc;
    }
    if ((e = lbk::launch_moe_down_grp(L->down_type, L->sdown_type, d, ctas, st)) != cudaSuccess)
        return cuda_fail(e, "moe grouped down launch");
    if (L->tracing) trace_record(L->trace[3], st, cudaEventRecordExternal);
    return ok();
}

// Expert stage of one MoE call for `tokens` tokens with routing in `routed`.
// With defer_topk (single token, fused kernels) the routing is computed by the
// gate/up kernel from the router's chunk partials and stored into `routed`.
// A mode other than the full one (expert-parallel items and shared-expert
// passes) needs the bulk-copy kernels.
int32_t moe_experts(lbk_moe_layer* L, const float* x, uint64_t T, const lbk_routed* routed, float* out, uint8_t* ws,
                    const WsLayout& o, cudaStream_t st, bool defer_topk, const MoeMode& mode) {
    lbk_context* ctx = L->ctx;
    cudaError_t e = cudaSuccess;
    const uint64_t nbh = L->H / LBK_QK_K, nbf = L->F / LBK_QK_K;
    const uint64_t K = mode.k;
    const bool full = mode.shared && mode.combine && K == L->k && mode.q8x == nullptr && mode.dots == nullptr;
    if (!full && !(L->fused && lbk::moe_gate_up_tma_supported(L->gate_type, L->sgate_type, (int)nbh) &&
                   lbk::moe_down_tma_supported(L->down_type, L->sdown_type, (int)nbf)))
        return fail(LBK_INVALID_PARAMETER, "expert-parallel calls need planar layers with hidden 2048 or 4096");
    if (L->fused && !defer_topk && (mode.grouped || (L->group_min != 0 && T >= L->group_min)) && T >= 2 &&
        L->E_local <= 1024 &&
        T * K <= 8192 &&
        lbk::moe_grouped_supported(L->gate_type, L->sgate_type, L->down_type, L->sdown_type, (int)nbh, (int)nbf))
        return moe_experts_grouped(L, T, routed, out, ws, o, st, mode);
    if (L->fused) {
        lbk::MoeGateUpArgs g{};
        g.defer_topk = defer_topk ? 1 : 0;
        g.partials = reinterpret_cast<const float*>(ws + o.partials);
        g.chunks = lbk::router_partials_floats(L->H, 1, 1);
        g.bias = L->w.selection_bias;
        g.weight_scale = L->weight_scale;
        g.routed_store = const_cast<lbk_routed*>(routed);
        g.hidden = L->H;
        g.ffn = L->F;
        g.nb_h = (int)nbh;
        g.nb_f = (int)nbf;
        int slots_unused = 0;
        lbk::gemv_plan(L->gate_type, (int)nbh, &g.tpr_h, &slots_unused);
        g.tokens = T;
        g.k = K;
        g.experts = L->E_local;
        g.gate = L->d_gate;
        g.up = L->d_up;
        g.sgate = static_cast<const uint8_t*>(L->w.shared.gate.data);
        g.sup = static_cast<const uint8_t*>(L->w.shared.up.data);
        g.routed = routed;
        g.q8x = mode.q8x ? mode.q8x : ws + o.q8x;
        g.d_items = mode.d_items;
        g.has_shared = mode.shared ? 1 : 0;
        g.h = reinterpret_cast<float*>(ws + o.h);
        g.hq = ws + o.hq;
        g.counters = reinterpret_cast<unsigned int*>(ws + o.counters);
        g.status = ctx->status;
        g.tables = ctx->tables();
        const int rps = 32 / g.tpr_h;
        if (lbk::moe_gate_up_tma_supported(L->gate_type, L->sgate_type, (int)nbh)) {
            // Split the SMs between routed and shared CTAs so that both roles
            // end together, then spread each role's rows over its warps.
            const unsigned ctas = (unsigned)ctx->sm_count;
            const double hb = 2.0 * nbh * 2.0 * L->F;  // half blocks of one slot (gate + up)
            const long rc = K == 0 ? 0
                            : !mode.shared ? (long)ctas
                                           : split_roles(ctas, lbk::kMoeGateUpTmaWarps, T * K * hb * gu_hb_cost_us(L->gate_type),
                                                         defer_topk ? 12.0 : 8.0, T * hb * gu_hb_cost_us(L->sgate_type), 8.0);
            g.routed_ctas = (uint32_t)rc;
            // single-token decode: the gate/up kernel publishes the routing for early down copies
            if (full && defer_topk && lbk::moe_down_tma_supported(L->down_type, L->sdown_type, (int)nbf))
                g.route_flag = reinterpret_cast<unsigned int*>(ws + o.rflag);
            if (full && T <= 4 && lbk::moe_down_tma_supported(L->down_type, L->sdown_type, (int)nbf)) {
                g.down = L->d_down;
                g.sdown = static_cast<const uint8_t*>(L->w.shared.down.data);
                g.down_rs = (uint32_t)((nbf * block_bytes(L->down_type) + 15) & ~(uint64_t)15);
                g.sdown_rs = (uint32_t)((nbf * block_bytes(L->sdown_type) + 15) & ~(uint64_t)15);
            }
            auto chunk_for = [&](uint64_t warps, uint64_t instances) {
                uint64_t per = instances ? warps / instances : 1;
                per = per < 1 ? 1 : per;
                uint64_t c = (L->F + per - 1) / per;
                return (c + rps - 1) / rps * rps;
            };
            g.chunk_r = chunk_for((uint64_t)rc * lbk::kMoeGateUpTmaWarps, T * K);
            g.chunk_s = chunk_for((uint64_t)(ctas - rc) * lbk::kMoeGateUpTmaWarps, T);
            g.chunks_r = (L->F + g.chunk_r - 1) / g.chunk_r;
            g.chunks_s = (L->F + g.chunk_s - 1) / g.chunk_s;
            e = lbk::launch_moe_gate_up_tma(L->gate_type, L->sgate_type, g, ctas, st);
            if (e != cudaSuccess) return cuda_fail(e, "moe gate/up launch");
        } else {
        // Balance bytes over ~ (SMs x 16) warps: routed and shared rows differ in size.
        const double br = 2.0 * (double)(nbh * block_bytes(L->gate_type)), bs = 2.0 * (double)(nbh * block_bytes(L->sgate_type));
        const double total = (double)T * L->F * ((double)L->k * br + bs);
        const double per_warp = total / (double)(ctx->sm_count * lbk::kMoeGateUpWarps);
        auto chunk_of = [&](double b) {
            uint64_t c = (uint64_t)(per_warp / b + 0.5);
            c = c < 1 ? 1 : c;
            c = (c + rps - 1) / rps * rps;
            return c > 256 ? (uint64_t)256 : c;
        };
        g.chunk_r = chunk_of(br);
        g.chunk_s = chunk_of(bs);
        g.chunks_r = (L->F + g.chunk_r - 1) / g.chunk_r;
        g.chunks_s = (L->F + g.chunk_s - 1) / g.chunk_s;
        // One CTA per SM (the tables fill shared memory): keep the grid to a
        // single wave by growing the chunks until every warp item fits.
        const uint64_t warp_cap = (uint64_t)ctx->sm_count * lbk::kMoeGateUpWarps;
        while (T * L->k * g.chunks_r + T * g.chunks_s > warp_cap && (g.chunk_r < 256 || g.chunk_s < 256)) {
            if (g.chunk_r < 256) g.chunk_r += rps;
            if (T * L->k * ((L->F + g.chunk_r - 1) / g.chunk_r) + T * g.chunks_s > warp_cap && g.chunk_s < 256)
                g.chunk_s += rps;
            g.chunks_r = (L->F + g.chunk_r - 1) / g.chunk_r;
            g.chunks_s = (L->F + g.chunk_s - 1) / g.chunk_s;
        }
        g.bmax_iq = 16 > rps ? 16 : rps;
        g.bmax_k = 2 > rps ? 2 : rps;
        const int kt_g = dot_type(L->gate_type) && (L->gate_type == LBK_TYPE_Q4_K || L->gate_type == LBK_TYPE_Q5_K) ? 9 : 1;
        const int kt_s = (L->sgate_type == LBK_TYPE_Q4_K || L->sgate_type == LBK_TYPE_Q5_K) ? 9 : 1;
        auto pf = [&](int kt) { return (uint64_t)(kt == 9 ? g.bmax_k : g.bmax_iq) * 2 * nbh * kt; };
        g.prod_floats = pf(kt_g) > pf(kt_s) ? pf(kt_g) : pf(kt_s);
        uint64_t dots = (uint64_t)2 * (g.bmax_iq > g.bmax_k ? g.bmax_iq : g.bmax_k);
        g.chain_floats = (dots * 9 + 64 + 3) & ~(uint64_t)3;
        if (lbk::moe_gate_up_fixed_smem(L->gate_type, L->sgate_type) +
                lbk::kMoeGateUpWarps * (g.prod_floats + g.chain_floats) * 4 >
            lbk::kMaxSmem - 8704)  // static top-k buffers
            return fail(LBK_INVALID_PARAMETER, "MoE gate/up shapes exceed shared memory");
        e = lbk::launch_moe_gate_up(L->gate_type, L->sgate_type, g, st);
        if (e != cudaSuccess) return cuda_fail(e, "moe gate/up launch");
        }
        if (L->tracing) trace_record(L->trace[2], st, cudaEventRecordExternal);

        lbk::MoeDownArgs d{};
        d.hidden = L->H;
        d.ffn = L->F;
        d.nb_f = (int)nbf;
        lbk::gemv_plan(L->down_type, (int)nbf, &d.tpr_f, &slots_unused);
        d.tokens = T;
        d.k = K;
        d.experts = L->E_local;
        d.down = L->d_down;
        d.sdown = static_cast<const uint8_t*>(L->w.shared.down.data);
        d.routed = routed;
        d.hq = ws + o.hq;
        d.out = out;
        d.status = ctx->status;
        d.tables = ctx->tables();
        if (lbk::moe_down_tma_supported(L->down_type, L->sdown_type, (int)nbf)) {
            // Split the SMs so that both roles end together, then spread each
            // role's rows over its warps (chunks in whole steps of 32 / tpr rows).
            const unsigned ctas = (unsigned)ctx->sm_count;
            const double lanes = (double)L->H * d.tpr_f;  // lane slots of one slot's rows
            const long rc = K == 0 ? 0
                            : !mode.shared ? (long)ctas
                                           : split_roles(ctas, lbk::kMoeDownTmaWarps, T * K * lanes * hb_cost_us(L->down_type),
                                                         4.0, T * lanes * hb_cost_us(L->sdown_type), 1.5);
            d.routed_ctas = (uint32_t)rc;
            const uint64_t R = 32 / d.tpr_f;
            auto chunk_for = [&](uint64_t warps, uint64_t instances) {
                uint64_t per = instances ? warps / instances : 1;
                per = per < 1 ? 1 : per;
                uint64_t c = (L->H + per - 1) / per;
                return (c + R - 1) / R * R;
            };
            d.chunk_r = chunk_for((uint64_t)rc * lbk::kMoeDownTmaWarps, T * K);
            d.chunk_s = chunk_for((uint64_t)(ctas - rc) * lbk::kMoeDownTmaWarps, T);
            d.chunks_r = (L->H + d.chunk_r - 1) / d.chunk_r;
            d.chunks_s = (L->H + d.chunk_s - 1) / d.chunk_s;
            d.dots = mode.dots ? mode.dots : reinterpret_cast<float*>(ws + o.dots);
            d.dots_slots = mode.dots_slots;
            d.combine = mode.combine ? 1 : 0;
            d.has_shared = mode.shared ? 1 : 0;
            d.counters = reinterpret_cast<unsigned int*>(ws + o.dcounters);
            d.route_flag = g.route_flag;
            d.d_items = mode.d_items;
            d.ret_addr = mode.ret;
            d.ret_peers = mode.ret_peers;
            d.ret_off = mode.ret_off;
            d.route_readers = g.route_flag ? reinterpret_cast<unsigned int*>(ws + o.rreaders) : nullptr;
            d.route_polls = L->wait_limit;
            e = lbk::launch_moe_down_tma(L->down_type, L->sdown_type, d, ctas, st);
            if (e != cudaSuccess) return cuda_fail(e, "moe down launch");
            if (L->tracing) trace_record(L->trace[3], st, cudaEventRecordExternal);
            return ok();
        }
        d.wps = 1;  // one warp per slot (the kernel's 288-thread bound covers top-k <= 8)
        const uint64_t rpsf = 32 / d.tpr_f;
        uint64_t ctas_x = (uint64_t)ctx->sm_count;
        uint64_t rows = (L->H + ctas_x - 1) / ctas_x;
        rows = (rows + d.wps * rpsf - 1) / (d.wps * rpsf) * (d.wps * rpsf);
        if (rows > 64 * d.wps) rows = 64 * d.wps;  // <= 64 dots per warp
        d.rows_per_cta = rows;
        const uint64_t dots_w = (rows + d.wps * rpsf - 1) / (d.wps * rpsf) * rpsf;
        const int kt_d = (L->down_type == LBK_TYPE_Q4_K || L->down_type == LBK_TYPE_Q5_K) ? 9 : 1;
        const int kt_sd = (L->sdown_type == LBK_TYPE_Q4_K || L->sdown_type == LBK_TYPE_Q5_K) ? 9 : 1;
        const int kt = kt_d > kt_sd ? kt_d : kt_sd;
        d.prod_floats = dots_w * nbf * kt;
        d.chain_floats = (dots_w * 9 + 64 + 3) & ~(uint64_t)3;
        d.status = ctx->status;
        d.tables = ctx->tables();
        const uint64_t warps = (L->k + 1) * d.wps;
        if (lbk::moe_down_fixed_smem(L->down_type, L->sdown_type) + (L->k + 1) * rows * 4 +
                warps * (d.prod_floats + d.chain_floats) * 4 >
            lbk::kMaxSmem)
            return fail(LBK_INVALID_PARAMETER, "MoE down shapes exceed shared memory");
        e = lbk::launch_moe_down(L->down_type, L->sdown_type, d, st);
        if (e != cudaSuccess) return cuda_fail(e, "moe down launch");
        if (L->tracing) trace_record(L->trace[3], st, cudaEventRecordExternal);
        return ok();
    }
    // Per-expert path: any types and layouts, one token at a time.
    float* g = reinterpret_cast<float*>(ws + o.g);
    float* u = reinterpret_cast<float*>(ws + o.u);
    uint8_t* q8 = ws + o.u + up256(L->F * 4);
    for (uint64_t t = 0; t < T; t++) {
        const float* xt = x + t * L->H;
        float* ot = out + t * L->H;
        fill_zero_kernel<<<(unsigned)((L->H + 255) / 256), 256, 0, st>>>(ot, L->H, ctx->status);
        for (uint64_t j = 0; j < L->k; j++) {
            const lbk_expert& proto = L->experts[0];
            if (int32_t s = expert_accumulate(ctx, &proto, xt, ot, 0.0f, g, u, q8, L->d_gate, L->d_up, L->d_down,
                                              routed + t * L->k + j, st, L->E))
                return s;
        }
        if (int32_t s = expert_accumulate(ctx, &L->w.shared, xt, ot, 1.0f, g, u, q8, nullptr, nullptr, nullptr, nullptr, st))
            return s;
    }
    return ok();
}

}  // namespace

namespace {
// Router logits and top-k of `tokens` tokens into `routed` (unless `defer`:
// then the gate/up kernel finishes the top-k), plus the tokens' Q8_K images
// for the fused kernels: the route step of hy3_moe_route_token
// (layer.rs:583-603; gemv_into on the router, route_experts_into).
int32_t launch_routing(lbk_moe_layer* layer, const float* x, uint64_t tokens, lbk_routed* routed, int32_t router_mode,
                       uint8_t* ws, const WsLayout& o, bool defer, cudaStream_t st) {
    lbk_context* ctx = layer->ctx;
    float* logits = reinterpret_cast<float*>(ws + o.logits);
    lbk::RouterFusedArgs f{};
    f.r.w = static_cast<const float*>(layer->w.router.data);
    f.r.x = x;
    f.r.logits = logits;
    f.r.hidden = layer->H;
    f.r.experts = layer->E;
    f.r.tokens = tokens;
    f.r.status = ctx->status;
    f.partials = reinterpret_cast<float*>(ws + o.partials);
    f.q8x = layer->fused ? ws + o.q8x : nullptr;
    f.counter = reinterpret_cast<unsigned int*>(ws + o.rcounter);
    f.zero = reinterpret_cast<unsigned int*>(ws + o.counters);
    f.zero_words = layer->fused ? o.counter_words : 0;
    f.bias = layer->w.selection_bias;
    f.k = (uint32_t)layer->k;
    f.weight_scale = layer->weight_scale;
    f.routed = routed;
    f.defer = defer ? 1 : 0;
    cudaError_t e;
    if (router_mode == LBK_ROUTER_TREE) {
        e = lbk::launch_router_fused(f, ctx->sm_count, st);
        if (e != cudaSuccess) return cuda_fail(e, "router launch");
    } else if (tokens <= 4 && layer->E <= 1024) {
        // sequential logits, the tokens' Q8_K and top-k in one launch
        if ((e = lbk::launch_router_seq_fused(f, ctx->sm_count, st)) != cudaSuccess) return cuda_fail(e, "router launch");
    } else {
        if (int32_t s = run_f32_gemv(ctx, &layer->w.router, x, tokens, logits, st)) return s;
        lbk::TopkArgs ta{logits, layer->w.selection_bias, layer->E, tokens, (uint32_t)layer->k, layer->weight_scale, routed,
                         ctx->status};
        if ((e = lbk::launch_topk(ta, st)) != cudaSuccess) return cuda_fail(e, "top-k launch");
        if (layer->fused) {  // quantize the tokens only
            lbk::RouterFusedArgs q = f;
            q.r.experts = 0;
            q.routed = nullptr;
            if ((e = lbk::launch_router_fused(q, ctx->sm_count, st)) != cudaSuccess) return cuda_fail(e, "quantize launch");
        }
    }
    return LBK_OK;
}

// Checks of lbk_moe_forward's arguments other than the workspace (shared
// with lbk_moe_forward_no_alloc, which runs them before any device work).
int32_t check_forward_args(const lbk_moe_layer* layer, const float* x, uint64_t tokens, const float* out,
                           int32_t router_mode) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (layer->E_local != layer->E) return fail(LBK_INVALID_PARAMETER, "an expert-parallel layer runs through lbk_ep_*");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    if (router_mode != LBK_ROUTER_SEQUENTIAL && router_mode != LBK_ROUTER_TREE) return fail(LBK_INVALID_PARAMETER, "router mode");
    if (x == nullptr || out == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(x, 16)) return fail(LBK_INVALID_PARAMETER, "x 16-byte / workspace 256-byte alignment");
    return LBK_OK;
}
}  // namespace

LBK_API int32_t lbk_moe_forward(lbk_moe_layer* layer, const float* x, uint64_t tokens, float* out,
                                lbk_routed* routed_out, int32_t router_mode, void* workspace, uint64_t workspace_bytes,
                                void* stream) {
    if (int32_t s = check_forward_args(layer, x, tokens, out, router_mode)) return s;
    WsLayout o = moe_ws(layer, tokens, layer->k);
    if (workspace_bytes < o.total) return fail(LBK_SCRATCH_TOO_SMALL, "MoE workspace", 0, o.total, workspace_bytes);
    if (workspace == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(workspace, 256)) return fail(LBK_INVALID_PARAMETER, "x 16-byte / workspace 256-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    lbk_routed* routed = routed_out ? routed_out : reinterpret_cast<lbk_routed*>(ws + o.routed);

    // Single-token decode on the fused kernels: the gate/up kernel finishes the
    // router (partials -> logits -> top-k) in every CTA's prologue.
    const bool defer = layer->fused && tokens == 1 && router_mode == LBK_ROUTER_TREE &&
                       (!lbk::moe_gate_up_tma_supported(layer->gate_type, layer->sgate_type, (int)(layer->H / LBK_QK_K)) ||
                        lbk::moe_gate_up_tma_defer_fits(layer->gate_type, layer->E,
                                                        lbk::router_partials_floats(layer->H, 1, 1)));
    if (layer->tracing) trace_record(layer->trace[0], st, cudaEventRecordExternal);
    if (int32_t s = launch_routing(layer, x, tokens, routed, router_mode, ws, o, defer, st)) return s;
    if (layer->tracing) trace_record(layer->trace[1], st, cudaEventRecordExternal);
    int32_t s = moe_experts(layer, x, tokens, routed, out, ws, o, st, defer, full_mode(layer));
    if (s == LBK_OK && layer->tracing && !layer->fused) {
        trace_record(layer->trace[2], st, cudaEventRecordExternal);
        trace_record(layer->trace[3], st, cudaEventRecordExternal);
    }
    return s;
}

LBK_API int32_t lbk_moe_routed(lbk_moe_layer* layer, const float* x, uint64_t tokens, const lbk_routed* routed,
                               float* out, void* workspace, uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (layer->E_local != layer->E) return fail(LBK_INVALID_PARAMETER, "an expert-parallel layer runs through lbk_ep_*");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "selected routed expert count", 0, 1, 0);
    WsLayout o = moe_ws(layer, tokens, layer->k);
    if (workspace_bytes < o.total) return fail(LBK_SCRATCH_TOO_SMALL, "MoE workspace", 0, o.total, workspace_bytes);
    if (x == nullptr || out == nullptr || workspace == nullptr || routed == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(x, 16) || !aligned(workspace, 256)) return fail(LBK_INVALID_PARAMETER, "x 16-byte / workspace 256-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    check_routed_kernel<<<(unsigned)((tokens + 127) / 128), 128, 0, st>>>(routed, tokens, layer->k, layer->E, ctx->status);
    if (layer->fused) {
        lbk::RouterFusedArgs q{};
        q.r.x = x;
        q.r.hidden = layer->H;
        q.r.experts = 0;
        q.r.tokens = tokens;
        q.r.status = ctx->status;
        q.q8x = ws + o.q8x;
        q.counter = reinterpret_cast<unsigned int*>(ws + o.rcounter);
        q.zero = reinterpret_cast<unsigned int*>(ws + o.counters);
        q.zero_words = o.counter_words;
        cudaError_t e = lbk::launch_router_fused(q, ctx->sm_count, st);
        if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
    }
    return moe_experts(layer, x, tokens, routed, out, ws, o, st, false, full_mode(layer));
}

// ------------------------------------------------ MoE block: norm, residual

namespace {

int32_t norm_params(uint64_t n, float epsilon) {
    // validate_norm_lengths / validate_epsilon (norm.rs:116-142)
    if (n == 0) return fail(LBK_INVALID_PARAMETER, "RMSNorm input must not be empty");
    if (!std::isfinite(epsilon)) return fail(LBK_NON_FINITE_VALUE, "RMSNorm epsilon", 0, 0, 0, f32_bits(epsilon));
    if (!(epsilon > 0.0f)) return fail(LBK_INVALID_PARAMETER, "RMSNorm epsilon must be greater than zero");
    return LBK_OK;
}

}  // namespace

LBK_API int32_t lbk_rms_norm(lbk_context* ctx, const float* x, const float* weight, uint64_t n, uint64_t rows,
                             float epsilon, float* out, int32_t mode, void* stream) {
    if (ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null context");
    if (int32_t s = norm_params(n, epsilon)) return s;
    if (rows == 0) return fail(LBK_DIMENSION_MISMATCH, "RMSNorm rows", 0, 1, 0);
    if (x == nullptr || weight == nullptr || out == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (mode != LBK_ROUTER_SEQUENTIAL && mode != LBK_ROUTER_TREE) return fail(LBK_INVALID_PARAMETER, "norm mode");
    if (mode == LBK_ROUTER_SEQUENTIAL && n * 4 > lbk::kMaxSmem)
        return fail(LBK_INVALID_PARAMETER, "sequential RMSNorm rows are staged in shared memory", 0, lbk::kMaxSmem / 4, n);
    if (int32_t s = set_device(ctx)) return s;
    lbk::NormArgs a{x, weight, epsilon, out, rows, n, mode == LBK_ROUTER_SEQUENTIAL ? 1 : 0, ctx->status};
    cudaError_t e = lbk::launch_rms_norm(a, ctx->sm_count, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "RMSNorm launch");
}

LBK_API int32_t lbk_residual_add(lbk_context* ctx, float* dest, const float* src, uint64_t n, void* stream) {
    if (ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null context");
    if (dest == nullptr || src == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (n == 0) return ok();
    if (int32_t s = set_device(ctx)) return s;
    cudaError_t e = lbk::launch_residual_add(dest, src, n, ctx->scratch_min, ctx->status, ctx->sm_count, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "residual add launch");
}

namespace {

// [normalized input T*H][MoE output T*H][routing T*k (route / finish)][lbk_moe_forward's workspace]
struct BlockWs {
    uint64_t normed, delta, routing, moe, total;
};
BlockWs block_ws(const lbk_moe_layer* L, uint64_t T) {
    const uint64_t a = moe_ws(L, T, L->k).total, b = moe_ws(L, 1, L->k).total;
    BlockWs w{};
    w.normed = 0;
    w.delta = up256(T * L->H * 4);
    w.routing = w.delta + up256(T * L->H * 4);
    w.moe = w.routing + up256(T * (L->k ? L->k : 1) * sizeof(lbk_routed));
    w.total = w.moe + (a > b ? a : b);
    return w;
}
uint64_t block_ws_bytes(const lbk_moe_layer* L, uint64_t T) { return block_ws(L, T).total; }

// Entry j of the caller's routing against the route phase's: expert ID and
// coefficient bits (layer.rs:631-640); the first mismatch is reported.
__global__ void routing_identity_kernel(const lbk_routed* selected, const lbk_routed* routing, uint64_t n,
                                        lbk::DeviceStatus* st) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const lbk_routed a = selected[i], b = routing[i];
        if (a.expert_id != b.expert_id || __float_as_uint(a.coefficient) != __float_as_uint(b.coefficient))
            lbk::report(st, LBK_INVALID_PARAMETER, i, __float_as_uint(a.coefficient));
    }
}

}  // namespace

LBK_API int32_t lbk_moe_block_workspace_bytes(const lbk_moe_layer* layer, uint64_t tokens, uint64_t* bytes) {
    if (layer == nullptr || bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    *bytes = block_ws_bytes(layer, tokens);
    return ok();
}

LBK_API int32_t lbk_moe_block_forward(lbk_moe_layer* layer, float* hidden, const float* ffn_norm, float epsilon,
                                      uint64_t tokens, lbk_routed* routed_out, int32_t router_mode, void* workspace,
                                      uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    if (int32_t s = norm_params(layer->H, epsilon)) return s;
    if (hidden == nullptr || ffn_norm == nullptr || workspace == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(hidden, 16) || !aligned(workspace, 256))
        return fail(LBK_INVALID_PARAMETER, "hidden 16-byte / workspace 256-byte alignment");
    const uint64_t need = block_ws_bytes(layer, tokens);
    if (workspace_bytes < need) return fail(LBK_SCRATCH_TOO_SMALL, "MoE block workspace", 0, need, workspace_bytes);
    if (router_mode != LBK_ROUTER_SEQUENTIAL && router_mode != LBK_ROUTER_TREE) return fail(LBK_INVALID_PARAMETER, "router mode");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const BlockWs bw = block_ws(layer, tokens);
    float* normed = reinterpret_cast<float*>(ws + bw.normed);
    float* delta = reinterpret_cast<float*>(ws + bw.delta);
    // hy3_moe_route_token's FFN norm (layer.rs:588-593)
    lbk::NormArgs na{hidden, ffn_norm, epsilon, normed, tokens, layer->H, router_mode == LBK_ROUTER_SEQUENTIAL ? 1 : 0,
                     ctx->status};
    cudaError_t e = lbk::launch_rms_norm(na, ctx->sm_count, st);
    if (e != cudaSuccess) return cuda_fail(e, "RMSNorm launch");
    // router, top-k, experts, combine
    if (int32_t s = lbk_moe_forward(layer, normed, tokens, delta, routed_out, router_mode, ws + bw.moe,
                                    workspace_bytes - bw.moe, stream))
        return s;
    // hy3_moe_finish_token's residual add (layer.rs:654)
    e = lbk::launch_residual_add(hidden, delta, tokens * layer->H, ctx->scratch_min, ctx->status, ctx->sm_count, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "residual add launch");
}

namespace {
int32_t block_args(const lbk_moe_layer* layer, const void* hidden, uint64_t tokens, const void* workspace,
                   uint64_t workspace_bytes) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (layer->E_local != layer->E) return fail(LBK_INVALID_PARAMETER, "an expert-parallel layer runs through lbk_ep_*");
    if (tokens == 0) return fail(LBK_DIMENSION_MISMATCH, "token count", 0, 1, 0);
    if (hidden == nullptr || workspace == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(hidden, 16) || !aligned(workspace, 256))
        return fail(LBK_INVALID_PARAMETER, "hidden 16-byte / workspace 256-byte alignment");
    const uint64_t need = block_ws_bytes(layer, tokens);
    if (workspace_bytes < need) return fail(LBK_SCRATCH_TOO_SMALL, "MoE block workspace", 0, need, workspace_bytes);
    return LBK_OK;
}
}  // namespace

LBK_API int32_t lbk_moe_block_route(lbk_moe_layer* layer, const float* hidden, const float* ffn_norm, float epsilon,
                                    uint64_t tokens, lbk_routed* routed_out, int32_t router_mode, void* workspace,
                                    uint64_t workspace_bytes, void* stream) {
    if (int32_t s = block_args(layer, hidden, tokens, workspace, workspace_bytes)) return s;
    if (int32_t s = norm_params(layer->H, epsilon)) return s;
    if (ffn_norm == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (router_mode != LBK_ROUTER_SEQUENTIAL && router_mode != LBK_ROUTER_TREE) return fail(LBK_INVALID_PARAMETER, "router mode");
    {
        std::lock_guard<std::mutex> lock(layer->phase_mu);
        if (layer->pending.count(workspace))  // layer.rs:488-493
            return fail(LBK_INVALID_PARAMETER,
                        "streaming MoE phase: the previous routed phase must be completed before routing again");
    }
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const BlockWs bw = block_ws(layer, tokens);
    float* normed = reinterpret_cast<float*>(ws + bw.normed);
    lbk_routed* routing = reinterpret_cast<lbk_routed*>(ws + bw.routing);
    // hy3_moe_route_token's FFN norm, router and top-k (layer.rs:588-603)
    lbk::NormArgs na{hidden, ffn_norm, epsilon, normed, tokens, layer->H, router_mode == LBK_ROUTER_SEQUENTIAL ? 1 : 0,
                     ctx->status};
    cudaError_t e = lbk::launch_rms_norm(na, ctx->sm_count, st);
    if (e != cudaSuccess) return cuda_fail(e, "RMSNorm launch");
    uint8_t* mws = ws + bw.moe;
    if (int32_t s = launch_routing(layer, normed, tokens, routing, router_mode, mws, moe_ws(layer, tokens, layer->k), false, st))
        return s;
    if (routed_out != nullptr) {
        e = cudaMemcpyAsync(routed_out, routing, tokens * layer->k * sizeof(lbk_routed), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "routing copy");
    }
    std::lock_guard<std::mutex> lock(layer->phase_mu);
    layer->pending[workspace] = tokens;
    return ok();
}

LBK_API int32_t lbk_moe_block_finish(lbk_moe_layer* layer, float* hidden, uint64_t tokens, const lbk_routed* selected,
                                     void* workspace, uint64_t workspace_bytes, void* stream) {
    if (int32_t s = block_args(layer, hidden, tokens, workspace, workspace_bytes)) return s;
    if (selected == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    {
        std::lock_guard<std::mutex> lock(layer->phase_mu);
        auto it = layer->pending.find(workspace);
        if (it == layer->pending.end())  // layer.rs:617-622
            return fail(LBK_INVALID_PARAMETER, "streaming MoE phase: routing must run exactly once before completion");
        if (it->second != tokens)  // layer.rs:624-630
            return fail(LBK_DIMENSION_MISMATCH, "streaming selected expert count", 0, it->second * layer->k,
                        tokens * layer->k);
    }
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const BlockWs bw = block_ws(layer, tokens);
    const float* normed = reinterpret_cast<const float*>(ws + bw.normed);
    float* delta = reinterpret_cast<float*>(ws + bw.delta);
    const lbk_routed* routing = reinterpret_cast<const lbk_routed*>(ws + bw.routing);
    // IDs and coefficient bits against the route phase (layer.rs:631-640),
    // before anything is written: a mismatch leaves delta and hidden untouched
    const uint64_t n = tokens * layer->k;
    routing_identity_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(selected, routing, n, ctx->status);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "routing check launch");
    // moe_selected_into and the residual add (layer.rs:648-656)
    if (int32_t s = lbk_moe_routed(layer, normed, tokens, selected, delta, ws + bw.moe, workspace_bytes - bw.moe, stream))
        return s;
    e = lbk::launch_residual_add(hidden, delta, tokens * layer->H, ctx->scratch_min, ctx->status, ctx->sm_count, st);
    if (e != cudaSuccess) return cuda_fail(e, "residual add launch");
    std::lock_guard<std::mutex> lock(layer->phase_mu);
    layer->pending.erase(workspace);
    return ok();
}

// --------------------------------------------------- expert parallelism
//
// A rank's layer (lbk_ep_layer_create) holds the whole router and the shared
// expert, and only its share of the routed experts. The MoE step of a token
// becomes: route on the token's home rank (lbk_ep_route: routing + Q8_K
// image); send each (token, slot) whose expert lives elsewhere to that rank;
// there, lbk_ep_items_forward computes the expert's row dots (down(SwiGLU(..))
// before the coefficient); send the dots home; lbk_ep_combine adds the shared
// expert and combines in ascending expert ID, the single-GPU order, so the
// result is bit-identical to lbk_moe_forward on one GPU.

namespace {

int32_t ep_check(const lbk_moe_layer* layer, uint64_t n, const void* ws, uint64_t ws_bytes, uint64_t need) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (n == 0) return fail(LBK_DIMENSION_MISMATCH, "token / item count", 0, 1, 0);
    if (ws_bytes < need) return fail(LBK_SCRATCH_TOO_SMALL, "expert-parallel workspace", 0, need, ws_bytes);
    if (ws == nullptr || !aligned(ws, 256)) return fail(LBK_INVALID_PARAMETER, "workspace null or not 256-byte aligned");
    if (!layer->fused || !lbk::moe_gate_up_tma_supported(layer->gate_type, layer->sgate_type, (int)(layer->H / LBK_QK_K)) ||
        !lbk::moe_down_tma_supported(layer->down_type, layer->sdown_type, (int)(layer->F / LBK_QK_K)))
        return fail(LBK_INVALID_PARAMETER, "expert parallelism needs planar layers with hidden 2048 or 4096");
    return LBK_OK;
}

uint64_t ep_ws_bytes(const lbk_moe_layer* L, uint64_t n) {
    uint64_t a = moe_ws(L, n, L->k).total, b = moe_ws(L, n, 1).total, c = moe_ws(L, n, 0).total + n * L->H * 4;
    uint64_t m = a > b ? a : b;
    return m > c ? m : c;
}

}  // namespace

LBK_API int32_t lbk_ep_q8_bytes(const lbk_moe_layer* layer, uint64_t* bytes) {
    if (layer == nullptr || bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    *bytes = layer->H / LBK_QK_K * lbk::kQ8IBytes;
    return ok();
}

LBK_API int32_t lbk_ep_workspace_bytes(const lbk_moe_layer* layer, uint64_t count, uint64_t* bytes) {
    if (layer == nullptr || bytes == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (count == 0) return fail(LBK_DIMENSION_MISMATCH, "token / item count", 0, 1, 0);
    *bytes = ep_ws_bytes(layer, count);
    return ok();
}

LBK_API int32_t lbk_ep_route(lbk_moe_layer* layer, const float* x, uint64_t tokens, lbk_routed* routed, uint8_t* q8,
                             void* workspace, uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (int32_t s = ep_check(layer, tokens, workspace, workspace_bytes, ep_ws_bytes(layer, tokens))) return s;
    if (x == nullptr || routed == nullptr || q8 == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(x, 16) || !aligned(q8, 16)) return fail(LBK_INVALID_PARAMETER, "x / q8 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    const WsLayout o = moe_ws(layer, tokens, layer->k);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    lbk::RouterFusedArgs f{};
    f.r.w = static_cast<const float*>(layer->w.router.data);
    f.r.x = x;
    f.r.logits = reinterpret_cast<float*>(ws + o.logits);
    f.r.hidden = layer->H;
    f.r.experts = layer->E;
    f.r.tokens = tokens;
    f.r.status = ctx->status;
    f.partials = reinterpret_cast<float*>(ws + o.partials);
    f.q8x = q8;
    f.counter = reinterpret_cast<unsigned int*>(ws + o.rcounter);
    f.bias = layer->w.selection_bias;
    f.k = (uint32_t)layer->k;
    f.weight_scale = layer->weight_scale;
    f.routed = routed;
    cudaError_t e = lbk::launch_router_fused(f, ctx->sm_count, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "router launch");
}

LBK_API int32_t lbk_ep_items_forward(lbk_moe_layer* layer, const uint8_t* q8_items, const lbk_routed* items_routed,
                                     uint64_t items, float* dots, void* workspace, uint64_t workspace_bytes,
                                     void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (int32_t s = ep_check(layer, items, workspace, workspace_bytes, ep_ws_bytes(layer, items))) return s;
    if (q8_items == nullptr || items_routed == nullptr || dots == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(q8_items, 16) || !aligned(dots, 16)) return fail(LBK_INVALID_PARAMETER, "q8 / dots 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    const WsLayout o = moe_ws(layer, items, 1);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + o.counters, 0, o.counter_words * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "zero counters");
    // one routed slot per item, the expert ID local to this layer; no shared expert, no combine
    return moe_experts(layer, nullptr, items, items_routed, nullptr, ws, o, st, false,
                       MoeMode{1, false, false, q8_items, dots, 1});
}

// ---------------------------------------------- peer memory (expert parallelism)

LBK_API int32_t lbk_peer_alloc(lbk_context* ctx, uint64_t bytes, void** ptr, uint8_t handle[64]) {
    if (ctx == nullptr || ptr == nullptr || handle == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (bytes == 0) return fail(LBK_DIMENSION_MISMATCH, "peer buffer bytes", 0, 1, 0);
    if (int32_t s = set_device(ctx)) return s;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc peer buffer");
    if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "zero peer buffer");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "cudaIpcGetMemHandle");
    }
    std::memcpy(handle, &h, 64);
    *ptr = p;
    return ok();
}

LBK_API int32_t lbk_peer_free(lbk_context* ctx, void* ptr) {
    if (ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null context");
    if (ptr == nullptr) return ok();
    if (int32_t s = set_device(ctx)) return s;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaFree peer buffer");
}

LBK_API int32_t lbk_peer_open(lbk_context* ctx, const uint8_t handle[64], void** ptr) {
    if (ctx == nullptr || handle == nullptr || ptr == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = set_device(ctx)) return s;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, 64);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    *ptr = p;
    return ok();
}

LBK_API int32_t lbk_peer_close(lbk_context* ctx, void* ptr) {
    if (ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null context");
    if (ptr == nullptr) return ok();
    if (int32_t s = set_device(ctx)) return s;
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? ok() : cuda_fail(e, "cudaIpcCloseMemHandle");
}

namespace {
lbk_ep_exchange ep_exchange(const lbk_moe_layer* L, uint64_t cap) {
    lbk_ep_exchange x{};
    const uint64_t q8b = L->H / LBK_QK_K * lbk::kQ8IBytes;
    x.routing = 0;
    x.control = up256(cap * L->k * sizeof(lbk_routed));
    x.q8 = x.control + 512;
    x.dots = up256(x.q8 + cap * q8b);
    x.total = up256(x.dots + cap * L->k * L->H * 4);
    x.q8_bytes = q8b;
    return x;
}

int32_t ep_check_ranks(uint32_t world, uint32_t rank, uint64_t cap) {
    if (world == 0 || world > lbk::kEpMaxRanks)
        return fail(LBK_DIMENSION_MISMATCH, "ranks", 0, lbk::kEpMaxRanks, world);
    if (rank >= world) return fail(LBK_DIMENSION_MISMATCH, "rank", 0, world - 1, rank);
    if (cap == 0) return fail(LBK_DIMENSION_MISMATCH, "tokens per rank", 0, 1, 0);
    return LBK_OK;
}
}  // namespace

LBK_API int32_t lbk_ep_exchange_layout(const lbk_moe_layer* layer, uint64_t cap, lbk_ep_exchange* out) {
    if (layer == nullptr || out == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (cap == 0) return fail(LBK_DIMENSION_MISMATCH, "tokens per rank", 0, 1, 0);
    *out = ep_exchange(layer, cap);
    return ok();
}

LBK_API int32_t lbk_ep_publish(lbk_moe_layer* layer, const float* x, uint64_t tokens, void* xbuf, uint64_t cap,
                               void* workspace, uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr || xbuf == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (tokens > cap) return fail(LBK_DIMENSION_MISMATCH, "tokens beyond the exchange capacity", 0, cap, tokens);
    if (!aligned(xbuf, 256)) return fail(LBK_INVALID_PARAMETER, "exchange buffer 256-byte alignment");
    const lbk_ep_exchange xl = ep_exchange(layer, cap);
    uint8_t* xb = static_cast<uint8_t*>(xbuf);
    if (tokens) {
        if (int32_t s = lbk_ep_route(layer, x, tokens, reinterpret_cast<lbk_routed*>(xb + xl.routing), xb + xl.q8,
                                     workspace, workspace_bytes, stream))
            return s;
    } else if (int32_t s = set_device(layer->ctx)) {
        return s;
    }
    cudaError_t e = lbk::launch_ep_publish(reinterpret_cast<lbk::EpControl*>(xb + xl.control), (uint32_t)tokens,
                                           as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "publish launch");
}

LBK_API int32_t lbk_ep_gather(lbk_moe_layer* layer, const void* const* peers, uint32_t world, uint32_t rank,
                              uint64_t cap, uint8_t* q8_items, lbk_routed* items, uint64_t* returns, uint32_t* count,
                              uint64_t cap_items, void* stream) {
    if (layer == nullptr || peers == nullptr || q8_items == nullptr || items == nullptr || returns == nullptr ||
        count == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = ep_check_ranks(world, rank, cap)) return s;
    if (cap_items < world * cap * layer->k)
        return fail(LBK_SCRATCH_TOO_SMALL, "item capacity", 0, world * cap * layer->k, cap_items);
    if (!aligned(q8_items, 16)) return fail(LBK_INVALID_PARAMETER, "q8 items 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    const lbk_ep_exchange xl = ep_exchange(layer, cap);
    lbk::EpGatherArgs a{reinterpret_cast<const uint8_t* const*>(peers), world, rank, (uint32_t)cap, (uint32_t)layer->k,
                        (uint32_t)xl.q8_bytes, xl.control, xl.q8, (uint32_t)layer->first, (uint32_t)layer->E_local,
                        q8_items, items, reinterpret_cast<uint2*>(returns), count, (uint32_t)cap_items,
                        layer->wait_limit, ctx->status};
    cudaError_t e = lbk::launch_ep_gather(a, ctx->sm_count, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "gather launch");
}

namespace {
// The kernels' choice for device-counted items of a capacity.
void items_rules(const lbk_moe_layer* layer, uint64_t cap_items, MoeMode& m) {
    // Grouped kernels decode a weight half block once per group of pairs: at
    // 21 items per expert (64 tokens per rank on 8 ranks, 24 experts each)
    // 23 % faster than one decode per item, equal at 2.7 per expert (one rank
    // holding all 192). Without a rule set on the layer, the capacity per
    // expert decides (the count itself is only known on the device).
    if (!layer->group_set) m.grouped = cap_items >= 4 * layer->E_local;
    // Gate/up and down on the tensor cores (grouped items): 3.0x the dp4a
    // grouped kernels at 21 pairs per expert, 1.2x at 5.3, even at 5.3 with
    // 24 experts, slower at 2.7. With every rank full, the pairs per local
    // expert are cap_items / E.
    m.tc = layer->tc_min != 0 && layer->gate_type == LBK_TYPE_IQ2_S && cap_items >= layer->tc_min * layer->E &&
           (m.grouped || (layer->group_min != 0 && cap_items >= layer->group_min));
}
}  // namespace

LBK_API int32_t lbk_ep_items_forward_counted(lbk_moe_layer* layer, const uint8_t* q8_items, const lbk_routed* items,
                                             const uint32_t* count, uint64_t cap_items, float* dots, void* workspace,
                                             uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (int32_t s = ep_check(layer, cap_items, workspace, workspace_bytes, ep_ws_bytes(layer, cap_items))) return s;
    if (q8_items == nullptr || items == nullptr || dots == nullptr || count == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(q8_items, 16) || !aligned(dots, 16)) return fail(LBK_INVALID_PARAMETER, "q8 / dots 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    const WsLayout o = moe_ws(layer, cap_items, 1);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + o.counters, 0, o.counter_words * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "zero counters");
    MoeMode m{1, false, false, q8_items, dots, 1};
    m.d_items = count;
    items_rules(layer, cap_items, m);
    if (layer->tracing) {  // no router here: its interval is empty, gate/up starts now
        trace_record(layer->trace[0], st, cudaEventRecordExternal);
        trace_record(layer->trace[1], st, cudaEventRecordExternal);
    }
    return moe_experts(layer, nullptr, cap_items, items, nullptr, ws, o, st, false, m);
}

LBK_API int32_t lbk_ep_items_return(lbk_moe_layer* layer, void* const* peers, uint32_t world, uint32_t rank,
                                    uint64_t cap, const uint8_t* q8_items, const lbk_routed* items,
                                    const uint64_t* returns, uint32_t* count, uint64_t cap_items, void* workspace,
                                    uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (int32_t s = ep_check_ranks(world, rank, cap)) return s;
    if (int32_t s = ep_check(layer, cap_items, workspace, workspace_bytes, ep_ws_bytes(layer, cap_items))) return s;
    if (peers == nullptr || q8_items == nullptr || items == nullptr || returns == nullptr || count == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(q8_items, 16)) return fail(LBK_INVALID_PARAMETER, "q8 items 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    const WsLayout o = moe_ws(layer, cap_items, 1);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + o.counters, 0, o.counter_words * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "zero counters");
    const lbk_ep_exchange xl = ep_exchange(layer, cap);
    MoeMode m{1, false, false, q8_items, nullptr, 1};
    m.d_items = count;
    m.ret = reinterpret_cast<const uint2*>(returns);
    m.ret_peers = reinterpret_cast<uint8_t* const*>(peers);
    m.ret_off = xl.dots;
    items_rules(layer, cap_items, m);
    if (layer->tracing) {
        trace_record(layer->trace[0], st, cudaEventRecordExternal);
        trace_record(layer->trace[1], st, cudaEventRecordExternal);
    }
    if (int32_t s = moe_experts(layer, nullptr, cap_items, items, nullptr, ws, o, st, false, m)) return s;
    lbk::EpScatterArgs a{reinterpret_cast<uint8_t* const*>(peers), world, rank, xl.control, xl.dots, nullptr,
                         reinterpret_cast<const uint2*>(returns), count, (uint32_t)cap_items, (uint32_t)layer->H};
    e = lbk::launch_ep_signal(a, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "signal launch");
}

LBK_API int32_t lbk_ep_scatter(lbk_moe_layer* layer, void* const* peers, uint32_t world, uint32_t rank, uint64_t cap,
                               const float* dots, const uint64_t* returns, uint32_t* count, uint64_t cap_items,
                               void* stream) {
    if (layer == nullptr || peers == nullptr || dots == nullptr || returns == nullptr || count == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = ep_check_ranks(world, rank, cap)) return s;
    if (!aligned(dots, 16) || layer->H % 4) return fail(LBK_INVALID_PARAMETER, "dots 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    const lbk_ep_exchange xl = ep_exchange(layer, cap);
    lbk::EpScatterArgs a{reinterpret_cast<uint8_t* const*>(peers), world, rank, xl.control, xl.dots, dots,
                         reinterpret_cast<const uint2*>(returns), count, (uint32_t)cap_items, (uint32_t)layer->H};
    cudaError_t e = lbk::launch_ep_scatter(a, ctx->sm_count, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "scatter launch");
}

namespace {
// The shared expert on a rank's published tokens: dots [tokens][H].
int32_t ep_shared_pass(lbk_moe_layer* layer, uint8_t* xb, const lbk_ep_exchange& xl, uint64_t tokens, float* dots,
                       uint8_t* ws, cudaStream_t st) {
    const WsLayout o = moe_ws(layer, tokens, 0);
    cudaError_t e = cudaMemsetAsync(ws + o.counters, 0, o.counter_words * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "zero counters");
    return moe_experts(layer, nullptr, tokens, reinterpret_cast<const lbk_routed*>(xb + xl.routing), nullptr, ws, o,
                       st, false, MoeMode{0, true, false, xb + xl.q8, dots, 1});
}
}  // namespace

LBK_API int32_t lbk_ep_shared(lbk_moe_layer* layer, void* xbuf, uint64_t cap, uint64_t tokens, float* shared_dots,
                              void* workspace, uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr || xbuf == nullptr || shared_dots == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (cap == 0) return fail(LBK_DIMENSION_MISMATCH, "tokens per rank", 0, 1, 0);
    if (tokens > cap) return fail(LBK_DIMENSION_MISMATCH, "tokens beyond the exchange capacity", 0, cap, tokens);
    if (!aligned(shared_dots, 16)) return fail(LBK_INVALID_PARAMETER, "shared dots 16-byte alignment");
    if (tokens == 0) return ok();
    if (int32_t s = ep_check(layer, tokens, workspace, workspace_bytes, ep_ws_bytes(layer, tokens))) return s;
    if (int32_t s = set_device(layer->ctx)) return s;
    return ep_shared_pass(layer, static_cast<uint8_t*>(xbuf), ep_exchange(layer, cap), tokens, shared_dots,
                          static_cast<uint8_t*>(workspace), as_stream(stream));
}

LBK_API int32_t lbk_ep_combine_exchange(lbk_moe_layer* layer, void* xbuf, uint32_t world, uint64_t cap,
                                        uint64_t tokens, const float* shared_dots, float* out, void* workspace,
                                        uint64_t workspace_bytes, void* stream) {
    if (layer == nullptr || xbuf == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = ep_check_ranks(world, 0, cap)) return s;
    if (tokens > cap) return fail(LBK_DIMENSION_MISMATCH, "tokens beyond the exchange capacity", 0, cap, tokens);
    if (tokens) {  // a rank without tokens only waits
        if (out == nullptr) return fail(LBK_INVALID_PARAMETER, "null output");
        if (int32_t s = ep_check(layer, tokens, workspace, workspace_bytes, ep_ws_bytes(layer, tokens))) return s;
    }
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    const lbk_ep_exchange xl = ep_exchange(layer, cap);
    uint8_t* xb = static_cast<uint8_t*>(xbuf);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (tokens && shared_dots == nullptr) {  // the shared expert here, in the workspace
        float* sd = reinterpret_cast<float*>(ws + moe_ws(layer, tokens, 0).total);
        if (int32_t s = ep_shared_pass(layer, xb, xl, tokens, sd, ws, st)) return s;
        shared_dots = sd;
    }
    cudaError_t e = lbk::launch_ep_combine_wait(reinterpret_cast<const lbk::EpControl*>(xb + xl.control), world,
                                                layer->wait_limit, reinterpret_cast<const lbk_routed*>(xb + xl.routing),
                                                reinterpret_cast<const float*>(xb + xl.dots), shared_dots, out, tokens,
                                                layer->k, layer->H, ctx->status, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "combine launch");
}

LBK_API int32_t lbk_ep_combine(lbk_moe_layer* layer, const uint8_t* q8, uint64_t tokens, const lbk_routed* routed,
                               const float* routed_dots, float* out, void* workspace, uint64_t workspace_bytes,
                               void* stream) {
    if (layer == nullptr) return fail(LBK_INVALID_PARAMETER, "null layer");
    if (int32_t s = ep_check(layer, tokens, workspace, workspace_bytes, ep_ws_bytes(layer, tokens))) return s;
    if (q8 == nullptr || routed == nullptr || routed_dots == nullptr || out == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(q8, 16)) return fail(LBK_INVALID_PARAMETER, "q8 16-byte alignment");
    lbk_context* ctx = layer->ctx;
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    const WsLayout o = moe_ws(layer, tokens, 0);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* shared_dots = reinterpret_cast<float*>(ws + o.total);  // [tokens][H] after the pass's own workspace
    cudaError_t e = cudaMemsetAsync(ws + o.counters, 0, o.counter_words * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "zero counters");
    if (int32_t s = moe_experts(layer, nullptr, tokens, routed, nullptr, ws, o, st, false,
                                MoeMode{0, true, false, q8, shared_dots, 1}))
        return s;
    e = lbk::launch_ep_combine(routed, routed_dots, shared_dots, out, tokens, layer->k, layer->H, ctx->status, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "combine launch");
}

// ------------------------------------------------- MoE forward, no allocation
//
// lbk_moe_forward_no_alloc runs lbk_moe_forward with its workspace in a fixed
// array of this library's device memory, so the caller allocates nothing and
// the call allocates nothing (no cudaMalloc / cudaFree, no allocating library
// routine). It serves callers that cannot allocate device memory: an FFI host
// that receives device pointers from another component and has no device
// allocator of its own to create the workspace, and decode loops in which a
// cudaMalloc / cudaFree would synchronize the device between layers.
//
// Limits: one array per device, shared by every call on that device, so calls
// that overlap in time (other streams, other host threads, other layers)
// race on it; serialize them (one stream, or events). Layers and token counts
// whose workspace exceeds kStaticScratchBytes are rejected with
// LBK_SCRATCH_TOO_SMALL. The workspace's first 16 bytes (the router's arrival
// counter, the routing flag and its reader count) must be zero when a call
// starts: the first call on a device zero-fills the whole array, and every
// call that runs to completion leaves those words at zero again.
namespace {

constexpr uint64_t kStaticScratchBytes = 1ull << 20;  // 1 MiB: hidden 4096 / ffn 1536 / top-8 decode up to 4 tokens
constexpr int kStaticScratchDevices = 64;

static __device__ __align__(256) uint8_t g_moe_scratch[kStaticScratchBytes];

std::mutex g_static_scratch_mu;
uint8_t* g_static_scratch[kStaticScratchDevices];

// Address of the array on `device`, which must be current. First call per
// device: symbol lookup plus a synchronous zero fill (setup work that belongs
// before any stream capture on that device).
int32_t static_scratch(int device, uint8_t** out) {
    if (device < 0 || device >= kStaticScratchDevices)
        return fail(LBK_INVALID_PARAMETER, "device ordinal beyond the static scratch table", 0,
                    (uint64_t)kStaticScratchDevices, (uint64_t)device);
    std::lock_guard<std::mutex> lock(g_static_scratch_mu);
    if (g_static_scratch[device] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_moe_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static MoE scratch)");
        if ((e = cudaMemset(p, 0, kStaticScratchBytes)) != cudaSuccess) return cuda_fail(e, "zero static MoE scratch");
        if ((e = cudaDeviceSynchronize()) != cudaSuccess) return cuda_fail(e, "zero static MoE scratch");
        g_static_scratch[device] = static_cast<uint8_t*>(p);
    }
    *out = g_static_scratch[device];
    return LBK_OK;
}

}  // namespace

LBK_API int32_t lbk_moe_forward_no_alloc(lbk_moe_layer* layer, const float* x, uint64_t tokens, float* out,
                                         lbk_routed* routed_out, int32_t router_mode, void* stream) {
    // every argument check runs before the first call's set-up touches the device
    if (int32_t s = check_forward_args(layer, x, tokens, out, router_mode)) return s;
    const uint64_t need = moe_ws(layer, tokens, layer->k).total;
    if (need > kStaticScratchBytes)
        return fail(LBK_SCRATCH_TOO_SMALL,
                    "static MoE scratch (1 MiB) is smaller than this layer's workspace for this token count; "
                    "use lbk_moe_forward with a caller workspace",
                    0, need, kStaticScratchBytes);
    if (int32_t s = set_device(layer->ctx)) return s;
    uint8_t* ws = nullptr;
    if (int32_t s = static_scratch(layer->ctx->device, &ws)) return s;
    return lbk_moe_forward(layer, x, tokens, out, routed_out, router_mode, ws, kStaticScratchBytes, stream);
}

// ------------------------------------------------------------ layout tools

namespace {
int32_t repack_common(lbk_context* ctx, const lbk_matrix* src, void* dst, uint64_t dst_bytes, int expect_layout,
                      int to_planar, void* stream) {
    if (int32_t s = check_matrix(src, "source")) return s;
    if (!dot_type(src->type)) return fail(LBK_UNSUPPORTED_TYPE, "only packed types have a planar layout", (uint64_t)src->type);
    if (src->layout != expect_layout) return fail(LBK_INVALID_PARAMETER, "source layout");
    uint64_t want = 0;
    if (to_planar) {
        if (int32_t s = lbk_planar_bytes(src->type, src->input_width, src->output_width, &want)) return s;
    } else {
        if (int32_t s = lbk_matrix_bytes(src->type, src->input_width, src->output_width, &want)) return s;
    }
    if (dst_bytes != want) return fail(LBK_ENCODED_LENGTH_MISMATCH, "destination length", 0, want, dst_bytes);
    if (ctx == nullptr || dst == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (!aligned(dst, 16)) return fail(LBK_INVALID_PARAMETER, "destination must be 16-byte aligned");
    if (int32_t s = set_device(ctx)) return s;
    lbk::RepackArgs a{static_cast<const uint8_t*>(src->data), static_cast<uint8_t*>(dst), src->output_width,
                      (int)(src->input_width / LBK_QK_K), src->type, to_planar};
    cudaError_t e = lbk::launch_repack(a, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "repack launch");
}
}  // namespace

LBK_API int32_t lbk_repack(lbk_context* ctx, const lbk_matrix* src_gguf, void* dst_planar, uint64_t dst_bytes, void* stream) {
    return repack_common(ctx, src_gguf, dst_planar, dst_bytes, LBK_LAYOUT_GGUF, 1, stream);
}

LBK_API int32_t lbk_unpack(lbk_context* ctx, const lbk_matrix* src_planar, void* dst_gguf, uint64_t dst_bytes, void* stream) {
    return repack_common(ctx, src_planar, dst_gguf, dst_bytes, LBK_LAYOUT_PLANAR, 0, stream);
}

LBK_API int32_t lbk_decode_rows(lbk_context* ctx, const lbk_matrix* w, uint64_t first_row, uint64_t rows, float* out,
                                void* stream) {
    if (int32_t s = check_matrix(w, "matrix")) return s;
    if (w->type != LBK_TYPE_F32 && !dot_type(w->type)) return fail(LBK_UNSUPPORTED_TYPE, "decode type", (uint64_t)w->type);
    if (w->layout != LBK_LAYOUT_GGUF)
        return fail(LBK_INVALID_PARAMETER, "decode takes the GGUF layout (lbk_unpack converts a planar matrix)");
    if (rows == 0) return fail(LBK_DIMENSION_MISMATCH, "decoded rows", 0, 1, 0);
    if (first_row > w->output_width || rows > w->output_width - first_row)
        return fail(LBK_DIMENSION_MISMATCH, "decoded row range", 0, w->output_width, first_row + rows);
    if (ctx == nullptr || out == nullptr) return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (int32_t s = set_device(ctx)) return s;
    cudaStream_t st = as_stream(stream);
    const uint64_t nb = w->input_width / LBK_QK_K;
    const uint64_t row_bytes = w->type == LBK_TYPE_F32 ? w->input_width * 4 : nb * block_bytes(w->type);
    const uint8_t* data = static_cast<const uint8_t*>(w->data) + first_row * row_bytes;
    cudaError_t e;
    if (w->type == LBK_TYPE_F32) {  // decode_f32_validated: the bits, unchanged
        e = cudaMemcpyAsync(out, data, rows * row_bytes, cudaMemcpyDeviceToDevice, st);
        return e == cudaSuccess ? ok() : cuda_fail(e, "f32 row copy");
    }
    e = lbk::launch_validate_scales(w->type, LBK_LAYOUT_GGUF, data, rows, (int)nb, ctx->scratch_min, ctx->status, st);
    if (e != cudaSuccess) return cuda_fail(e, "scale scan launch");
    lbk::DecodeArgs a{w->type, data, rows, (int)nb, out, ctx->iq2s, ctx->iq3s, ctx->status};
    e = lbk::launch_decode(a, ctx->sm_count, st);
    return e == cudaSuccess ? ok() : cuda_fail(e, "decode launch");
}

LBK_API int32_t lbk_validate_matrix(lbk_context* ctx, const lbk_matrix* w, void* stream) {
    if (int32_t s = check_matrix(w, "matrix")) return s;
    if (!dot_type(w->type)) return fail(LBK_UNSUPPORTED_TYPE, "only packed types carry binary16 scales", (uint64_t)w->type);
    if (ctx == nullptr) return fail(LBK_INVALID_PARAMETER, "null context");
    if (int32_t s = set_device(ctx)) return s;
    cudaError_t e = lbk::launch_validate_scales(w->type, w->layout, static_cast<const uint8_t*>(w->data), w->output_width,
                                                (int)(w->input_width / LBK_QK_K), ctx->scratch_min, ctx->status,
                                                as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "validate launch");
}

// ---------------------------------------------- tensor-core grouped dots

LBK_API int32_t lbk_tc_grouped_dots(lbk_context* ctx, int32_t type, const lbk_tc_matrix* mats, uint32_t nmat,
                                    const uint32_t* jobs, uint32_t njobs, const uint8_t* q8, uint64_t q8_row_bytes,
                                    const uint32_t* pair_tokens, float* dots, uint64_t dots_stride, void* stream) {
    if (type != LBK_TYPE_IQ2_S && type != LBK_TYPE_IQ3_S) return fail(LBK_UNSUPPORTED_TYPE, "tensor-core dots type");
    if (ctx == nullptr || mats == nullptr || jobs == nullptr || q8 == nullptr || pair_tokens == nullptr ||
        dots == nullptr)
        return fail(LBK_INVALID_PARAMETER, "null pointer");
    if (nmat == 0) return fail(LBK_DIMENSION_MISMATCH, "matrices", 0, 1, 0);
    if (!aligned(q8, 16) || q8_row_bytes % 16 != 0 || !aligned(jobs, 16))
        return fail(LBK_INVALID_PARAMETER, "q8 / jobs 16-byte alignment");
    if (int32_t s = set_device(ctx)) return s;
    lbk::TcDotsArgs a{reinterpret_cast<const lbk::TcMatrix*>(mats), nmat, reinterpret_cast<const uint4*>(jobs), q8,
                      q8_row_bytes, pair_tokens, dots, dots_stride, ctx->status, ctx->tables()};
    cudaError_t e = lbk::launch_tc_dots(type, a, njobs, as_stream(stream));
    return e == cudaSuccess ? ok() : cuda_fail(e, "tensor-core dots launch");
}
