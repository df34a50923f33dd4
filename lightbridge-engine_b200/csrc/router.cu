// router.cu -- router logits (F32 GEMV) and Hy3 top-k routing.
//
// Replaces the router step of hy3_moe_route_token
// (bridge-kernels-reference/src/layer.rs:583-603): gemv_into on the F32
// router matrix (gemv.rs:72-86, dot_f32_row :286-303) followed by
// route_experts_into (bridge-model-hy3/src/routing.rs:25-107).
//
// Two logit orders:
//  * sequential -- one lane per (token, expert) runs the reference's single
//    f32 chain over the hidden lanes from products the rest of its CTA forms
//    in shared memory: bit-identical, bound by the chain's latency;
//  * tree -- rows split into 512-lane chunks over many warps, each chunk a
//    fixed shuffle tree, chunks summed in chunk order: deterministic and
//    within 1e-5 of the sequential order. The tree kernel also quantizes the
//    tokens to Q8_K for the expert kernels and, in its last CTA, runs top-k.

#include "lbk_kernels.h"
#include "lbk_topk.cuh"

namespace lbk {

namespace {

constexpr int kRouterThreads = 512;
constexpr int kChunk = 512;     // hidden lanes per warp work item
constexpr int kTopkWarps = 4;  // per CTA; each holds 2 x 1024 floats of scratch

__global__ void topk_kernel(TopkArgs a) {
    __shared__ float s_tk[kTopkWarps][2][1024];
    const int warp = threadIdx.x >> 5;
    for (uint64_t t = (uint64_t)blockIdx.x * kTopkWarps + warp; t < a.tokens; t += (uint64_t)gridDim.x * kTopkWarps)
        topk_warp(a.logits + t * a.experts, a.bias, (int)a.experts, (int)a.k, a.weight_scale, a.routed + t * a.k,
                  a.status, t, s_tk[warp][0], s_tk[warp][1]);
}

// Sequential order: bit-identical to dot_f32_row (gemv.rs:286-303): for each
// (token, expert), sum = fl(sum + fl(w[j] * x[j])) over j in order. The
// products do not depend on one another: warps 1-7 of the CTA form them for
// kSeqExperts experts, one chunk of the row at a time, with every load of a
// chunk in flight at once, into one of two shared buffers; meanwhile lane e of
// warp 0 runs expert e0 + e's dependent additions over the previous chunk,
// four products per shared load. The chain itself (hidden dependent adds) is
// the floor of this order; the loads of the next chunk hide behind it.
constexpr int kSeqExperts = 2;                                  // experts per CTA (one summing lane each)
constexpr int kSeqChunk = 2048;                                 // lanes of a row per chunk (16 KB of products)
constexpr int kSeqThreads = 256;
constexpr int kSeqLoaders = kSeqThreads - 32;                   // warps 1-7
constexpr int kSeqPer = (kSeqExperts * kSeqChunk + kSeqLoaders - 1) / kSeqLoaders;  // products per loader

// One item of the sequential order: token t, experts e0 .. e0 + kSeqExperts - 1.
__device__ __forceinline__ void seq_item(const RouterArgs& a, uint64_t t, uint64_t e0,
                                         float (*s_p)[kSeqExperts][kSeqChunk]) {
    const int warp = threadIdx.x >> 5;
    {
        const int ne = (int)(a.experts - e0 < (uint64_t)kSeqExperts ? a.experts - e0 : kSeqExperts);
        const float* x = a.x + t * a.hidden;
        const uint64_t nchunks = (a.hidden + kSeqChunk - 1) / kSeqChunk;
        // The item's rows and x into L2 at once (bulk prefetches, 16-byte
        // aligned rows only): each chunk's loads then return from L2 within
        // the summing of the chunk before, instead of one HBM round trip per
        // chunk on the critical path.
        const uint64_t row_bytes = a.hidden * 4;
        if (warp == 0 && (row_bytes & 15) == 0 && row_bytes < (1ull << 31)) {
            const int lane = threadIdx.x & 31;
            const float* src = lane < ne ? a.w + (e0 + lane) * a.hidden : (lane == ne ? x : nullptr);
            if (src != nullptr && ((uintptr_t)src & 15) == 0) prefetch_l2(src, (uint32_t)row_bytes);
        }
        // chunk c's products into buffer c & 1 (loaders only)
        auto stage = [&](uint64_t c) {
            const uint64_t c0 = c * kSeqChunk;
            const int n = (int)(a.hidden - c0 < (uint64_t)kSeqChunk ? a.hidden - c0 : kSeqChunk);
            const int tid = (int)threadIdx.x - 32;
            float wv[kSeqPer], xv[kSeqPer];
#pragma unroll
            for (int m = 0; m < kSeqPer; m++) {  // every load of the chunk in flight
                const int i = tid + m * kSeqLoaders, e = i / kSeqChunk, j = i - e * kSeqChunk;
                const bool in = e < ne && j < n;
                wv[m] = in ? __ldcs(a.w + (e0 + e) * a.hidden + c0 + j) : 0.0f;
                xv[m] = in ? __ldg(x + c0 + j) : 0.0f;
            }
#pragma unroll
            for (int m = 0; m < kSeqPer; m++) {
                const int i = tid + m * kSeqLoaders, e = i / kSeqChunk, j = i - e * kSeqChunk;
                if (e < ne && j < n) {
                    if (!isfinite(wv[m]))
                        report(a.status, LBK_NON_FINITE_VALUE, (e0 + e) * a.hidden + c0 + j, __float_as_uint(wv[m]));
                    s_p[c & 1][e][j] = __fmul_rn(wv[m], xv[m]);
                }
            }
        };
        __syncthreads();  // the previous item's sums are done with both buffers
        if (warp != 0) stage(0);
        __syncthreads();
        float sum = 0.0f;  // lane e of warp 0: expert e0 + e
        for (uint64_t c = 0; c < nchunks; c++) {
            if (warp != 0) {
                if (c + 1 < nchunks) stage(c + 1);
            } else if (threadIdx.x < (unsigned)ne) {
                const uint64_t c0 = c * kSeqChunk;
                const int n = (int)(a.hidden - c0 < (uint64_t)kSeqChunk ? a.hidden - c0 : kSeqChunk);
                const float* p = s_p[c & 1][threadIdx.x];
                int j = 0;
                if ((n & 31) == 0) {
                    // software-pipelined: the next 32 products are loaded
                    // before the current 32 are added, so the shared loads
                    // never sit on the dependent chain
                    const float4* p4 = reinterpret_cast<const float4*>(p);
                    const int n4 = n / 4;
                    float4 cur[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) cur[u] = p4[u];
                    for (int j4 = 0; j4 < n4; j4 += 8) {
                        float4 nxt[8];
#pragma unroll
                        for (int u = 0; u < 8; u++) nxt[u] = j4 + 8 + u < n4 ? p4[j4 + 8 + u] : cur[u];
#pragma unroll
                        for (int u = 0; u < 8; u++)
                            sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, cur[u].x), cur[u].y), cur[u].z), cur[u].w);
#pragma unroll
                        for (int u = 0; u < 8; u++) cur[u] = nxt[u];
                    }
                    j = n;
                }
                for (; j < n; j++) sum = __fadd_rn(sum, p[j]);
            }
            __syncthreads();  // chunk c summed and chunk c + 1 staged
        }
        if (threadIdx.x < (unsigned)ne) a.logits[t * a.experts + e0 + threadIdx.x] = sum;
    }
}

__global__ void __launch_bounds__(kSeqThreads) router_seq_kernel(RouterArgs a) {
    __shared__ __align__(16) float s_p[2][kSeqExperts][kSeqChunk];
    const uint64_t groups = (a.experts + kSeqExperts - 1) / kSeqExperts;
    for (uint64_t gi = blockIdx.x; gi < groups * a.tokens; gi += gridDim.x)
        seq_item(a, gi / groups, (gi % groups) * kSeqExperts, s_p);
}

}  // namespace

namespace {

// Q8_K of one 256-lane block q (token q / nbq, block q % nbq) of the tokens
// into the expert kernels' image (one warp); a non-finite lane is reported
// and the block is left unwritten.
__device__ __forceinline__ void q8_item(const RouterFusedArgs& f, uint64_t q, uint64_t nbq, int lane) {
    const RouterArgs& a = f.r;
    uint64_t t = q / nbq, b = q % nbq;
    const float* xb = a.x + t * a.hidden + b * kQK + lane * 8;
    float v[8];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        v[i] = __ldg(xb + i);
        bad |= !isfinite(v[i]);
    }
    if (__ballot_sync(0xffffffffu, bad)) {
        if (bad) {
            for (int i = 0; i < 8; i++)
                if (!isfinite(v[i])) {
                    report(a.status, LBK_NON_FINITE_VALUE, t * a.hidden + b * kQK + lane * 8 + i, __float_as_uint(v[i]));
                    break;
                }
        }
        return;
    }
    Q8Block qb = quantize_q8k_warp(v, lane);
    int32_t pair = qb.pair_sum + __shfl_xor_sync(0xffffffffu, qb.pair_sum, 1);
    store_q8i(f.q8x + (t * nbq + b) * kQ8IBytes, qb, pair, lane);
}

// Chunk partials of one (expert, chunk) item for every token, kTB tokens at a time.
template <int kTB>
__device__ __forceinline__ void chunk_partials(const RouterArgs& a, const RouterFusedArgs& f, const float* wr,
                                               uint64_t j0, uint64_t e, uint64_t c, uint64_t chunks, int lane) {
    for (uint64_t t0 = 0; t0 < a.tokens; t0 += kTB) {
        float xr[kTB][16];
#pragma unroll
        for (int u = 0; u < kTB; u++)
#pragma unroll
            for (int q = 0; q < 16; q++) {
                uint64_t j = j0 + (uint64_t)q * 32 + lane;
                xr[u][q] = (t0 + u < a.tokens && j < a.hidden) ? __ldg(a.x + (t0 + u) * a.hidden + j) : 0.0f;
            }
#pragma unroll
        for (int u = 0; u < kTB; u++) {
            if (t0 + u >= a.tokens) break;
            float acc = 0.0f;
#pragma unroll
            for (int q = 0; q < 16; q++) acc = __fadd_rn(acc, __fmul_rn(wr[q], xr[u][q]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
            if (lane == 0) f.partials[((t0 + u) * a.experts + e) * chunks + c] = acc;
        }
    }
}

__global__ void __launch_bounds__(kRouterThreads) router_fused_kernel(RouterFusedArgs f) {
    const RouterArgs& a = f.r;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t chunks = (a.hidden + kChunk - 1) / kChunk;
    const uint64_t row_items = a.experts * chunks;
    const uint64_t nbq = f.q8x ? a.hidden / kQK : 0;
    const uint64_t items = row_items + a.tokens * nbq;
    const uint64_t nw = (uint64_t)gridDim.x * (kRouterThreads / 32);
    __shared__ bool s_last;
    // The gate/up kernel may launch now: it does its constant-data prologue
    // on free SMs and waits for this grid before reading its output.
    grid_dep_launch();
    // The arrival counters of the gate/up and down launches that follow sit
    // at call-dependent places in the workspace: zero them for this call.
    if (blockIdx.x == 0)
        for (uint64_t i = threadIdx.x; i < f.zero_words; i += kRouterThreads) f.zero[i] = 0u;

    for (uint64_t it = (uint64_t)blockIdx.x * (kRouterThreads / 32) + warp; it < items; it += nw) {
        if (it < row_items) {
            uint64_t e = it / chunks, c = it % chunks;
            uint64_t j0 = c * kChunk;
            const float* w = a.w + e * a.hidden;
            // All loads first: no store (partials, status) may sit between
            // them, or the compiler serializes the loads behind it.
            float wr[16];
#pragma unroll
            for (int q = 0; q < 16; q++) {
                uint64_t j = j0 + (uint64_t)q * 32 + lane;
                wr[q] = j < a.hidden ? __ldcs(w + j) : 0.0f;
            }
            // several tokens: four at a time, their loads in flight together
            // (a single token takes the one-token instance: no idle loads)
            if (a.tokens == 1) chunk_partials<1>(a, f, wr, j0, e, c, chunks, lane);
            else chunk_partials<4>(a, f, wr, j0, e, c, chunks, lane);
            int bad_q = -1;
            uint32_t bad_bits = 0;
#pragma unroll
            for (int q = 15; q >= 0; q--)
                if (!isfinite(wr[q])) {
                    bad_q = q;
                    bad_bits = __float_as_uint(wr[q]);
                }
            if (bad_q >= 0) report(a.status, LBK_NON_FINITE_VALUE, e * a.hidden + j0 + (uint64_t)bad_q * 32 + lane, bad_bits);
        } else {
            q8_item(f, it - row_items, nbq, lane);
        }
    }

    // The last CTA to finish sums the chunk partials in chunk order and routes
    // (unless the consumer kernel does both itself).
    if (f.defer || f.split) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned ticket = atomicAdd(f.counter, 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const uint64_t nlog = a.tokens * a.experts;
    for (uint64_t i = threadIdx.x; i < nlog; i += kRouterThreads) {
        const float* pp = f.partials + i * chunks;
        float sum = 0.0f;
        for (uint64_t c = 0; c < chunks; c++) sum = __fadd_rn(sum, __ldcg(pp + c));
        a.logits[i] = sum;
    }
    __syncthreads();
    if (f.routed != nullptr && warp < kTopkWarps) {
        __shared__ float s_tk[kTopkWarps][2][1024];
        for (uint64_t t = warp; t < a.tokens; t += kTopkWarps)
            topk_warp(a.logits + t * a.experts, f.bias, (int)a.experts, (int)f.k, f.weight_scale, f.routed + t * f.k,
                      a.status, t, s_tk[warp][0], s_tk[warp][1]);
    }
    if (threadIdx.x == 0) *f.counter = 0u;
}

// The sequential order for a layer call of at most kTopkWarps tokens, in one
// launch: CTAs [0, seq_ctas) run seq_item over the (token, expert group)
// items; the CTAs after them quantize the tokens to Q8_K for the expert
// kernels, one warp per block; CTA 0 zeroes the call's arrival counters; the
// last CTA to arrive runs top-k, one warp per token, in the shared memory of
// the product buffers (free by then).
__global__ void __launch_bounds__(kSeqThreads) router_seq_fused_kernel(RouterFusedArgs f, uint32_t seq_ctas) {
    __shared__ __align__(16) float s_p[2][kSeqExperts][kSeqChunk];
    static_assert(sizeof(s_p) >= sizeof(float) * kTopkWarps * 2 * 1024, "top-k scratch fits the product buffers");
    __shared__ bool s_last;
    const RouterArgs& a = f.r;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    grid_dep_launch();  // the gate/up kernel may start its prologue; it waits for this grid
    if (blockIdx.x == 0)
        for (uint64_t i = threadIdx.x; i < f.zero_words; i += kSeqThreads) f.zero[i] = 0u;
    if (blockIdx.x < seq_ctas) {
        const uint64_t groups = (a.experts + kSeqExperts - 1) / kSeqExperts;
        for (uint64_t gi = blockIdx.x; gi < groups * a.tokens; gi += seq_ctas)
            seq_item(a, gi / groups, (gi % groups) * kSeqExperts, s_p);
    } else {
        const uint64_t nbq = f.q8x ? a.hidden / kQK : 0;
        constexpr int kW = kSeqThreads / 32;
        for (uint64_t q = (uint64_t)(blockIdx.x - seq_ctas) * kW + warp; q < a.tokens * nbq;
             q += (uint64_t)(gridDim.x - seq_ctas) * kW)
            q8_item(f, q, nbq, lane);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        unsigned ticket = atomicAdd(f.counter, 1u);
        s_last = (ticket == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();  // every CTA's logits before the reads below
    if (f.routed != nullptr && warp < kTopkWarps) {
        float* tk = &s_p[0][0][0] + (size_t)warp * 2 * 1024;
        for (uint64_t t = warp; t < a.tokens; t += kTopkWarps)
            topk_warp(a.logits + t * a.experts, f.bias, (int)a.experts, (int)f.k, f.weight_scale, f.routed + t * f.k,
                      a.status, t, tk, tk + 1024);
    }
    if (threadIdx.x == 0) *f.counter = 0u;
}

// Several tokens: logits (chunk partials summed in chunk order, as the
// last-CTA pass does) and top-k, one warp per token over many CTAs, after
// the router grid (programmatic dependent launch).
__global__ void topk_partials_kernel(RouterFusedArgs f) {
    __shared__ float s_tk[kTopkWarps][2][1024];
    const RouterArgs& a = f.r;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t chunks = (a.hidden + kChunk - 1) / kChunk;
    grid_dep_launch();
    grid_dep_wait();  // the router's partials
    for (uint64_t t = (uint64_t)blockIdx.x * kTopkWarps + warp; t < a.tokens; t += (uint64_t)gridDim.x * kTopkWarps) {
        for (uint64_t e = lane; e < a.experts; e += 32) {
            const float* pp = f.partials + (t * a.experts + e) * chunks;
            float sum = 0.0f;
            for (uint64_t c = 0; c < chunks; c++) sum = __fadd_rn(sum, __ldcg(pp + c));
            a.logits[t * a.experts + e] = sum;
        }
        __syncwarp();
        topk_warp(a.logits + t * a.experts, f.bias, (int)a.experts, (int)f.k, f.weight_scale, f.routed + t * f.k,
                  a.status, t, s_tk[warp][0], s_tk[warp][1]);
    }
}

}  // namespace

size_t router_partials_floats(uint64_t hidden, uint64_t experts, uint64_t tokens) {
    return (size_t)tokens * experts * ((hidden + kChunk - 1) / kChunk);
}

cudaError_t launch_router_fused(const RouterFusedArgs& f, int sm_count, cudaStream_t stream) {
    const uint64_t chunks = (f.r.hidden + kChunk - 1) / kChunk;
    uint64_t items = f.r.experts * chunks + (f.q8x ? f.r.tokens * (f.r.hidden / kQK) : 0);
    uint64_t ctas = (items + (kRouterThreads / 32) - 1) / (kRouterThreads / 32);
    if (ctas > (uint64_t)sm_count) ctas = sm_count;
    if (ctas < 1) ctas = 1;
    RouterFusedArgs g = f;
    g.split = (!f.defer && f.r.experts > 0 && f.routed != nullptr && f.r.tokens > 1 && f.r.experts <= 1024) ? 1 : 0;
    router_fused_kernel<<<(unsigned)ctas, kRouterThreads, 0, stream>>>(g);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !g.split) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)((f.r.tokens + kTopkWarps - 1) / kTopkWarps));
    cfg.blockDim = dim3(kTopkWarps * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, topk_partials_kernel, g);
}

cudaError_t launch_router(const RouterArgs& a, int mode, int sm_count, cudaStream_t stream) {
    (void)mode;
    const uint64_t n = (a.experts + kSeqExperts - 1) / kSeqExperts * a.tokens;
    uint64_t grid = n;
    if (grid > (uint64_t)sm_count * 4) grid = (uint64_t)sm_count * 4;
    if (grid < 1) grid = 1;
    router_seq_kernel<<<(unsigned)grid, kSeqThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_router_seq_fused(const RouterFusedArgs& f, int sm_count, cudaStream_t stream) {
    if (f.r.tokens > (uint64_t)kTopkWarps || f.r.experts > 1024) return cudaErrorInvalidValue;
    const uint64_t groups = (f.r.experts + kSeqExperts - 1) / kSeqExperts;
    uint64_t seq = groups * f.r.tokens;
    if (seq > (uint64_t)sm_count * 4) seq = (uint64_t)sm_count * 4;
    if (seq < 1) seq = 1;
    const uint64_t qw = f.q8x ? f.r.tokens * (f.r.hidden / kQK) : 0;
    const uint64_t qc = (qw + kSeqThreads / 32 - 1) / (kSeqThreads / 32);
    router_seq_fused_kernel<<<(unsigned)(seq + qc), kSeqThreads, 0, stream>>>(f, (uint32_t)seq);
    return cudaGetLastError();
}

cudaError_t launch_topk(const TopkArgs& a, cudaStream_t stream) {
    uint64_t grid = (a.tokens + kTopkWarps - 1) / kTopkWarps;
    if (grid < 1) grid = 1;
    topk_kernel<<<(unsigned)grid, kTopkWarps * 32, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace lbk
