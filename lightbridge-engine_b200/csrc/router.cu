// router.cu -- router logits (F32 GEMV) and Hy3 top-k routing.
//
// Replaces the router step of hy3_moe_route_token
// (bridge-kernels-reference/src/layer.rs:583-603): gemv_into on the F32
// router matrix (gemv.rs:72-86, dot_f32_row :286-303) followed by
// route_experts_into (bridge-model-hy3/src/routing.rs:25-107).
//
// Two logit orders:
//  * sequential -- one thread per (token, expert) runs the reference's single
//    f32 chain over the hidden lanes, bit-identical, but latency-bound;
//  * tree -- rows split into 512-lane chunks over many warps, each chunk a
//    fixed shuffle tree, chunks summed in chunk order: deterministic and
//    within 1e-5 of the sequential order. The tree kernel also quantizes the
//    tokens to Q8_K for the expert kernels and, in its last CTA, runs top-k.

#include "lbk_kernels.h"

namespace lbk {

namespace {

constexpr int kRouterThreads = 512;
constexpr int kChunk = 512;     // hidden lanes per warp work item
constexpr int kMaxCand = 32;    // candidates per lane in top-k (E <= 1024)

__device__ __forceinline__ uint32_t ord_f32(float f) {
    if (f == 0.0f) f = 0.0f;  // -0 and +0 compare equal in the reference sort
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Top-k of one token by one warp (routing.rs:25-107).
__device__ void topk_warp(const float* logits, const float* bias, int E, int k, float weight_scale, lbk_routed* out,
                          DeviceStatus* st, uint64_t token) {
    const int lane = threadIdx.x & 31;
    float p[kMaxCand], s[kMaxCand];
    uint32_t bad_idx = 0xffffffffu, bad_bits = 0;
#pragma unroll
    for (int c = 0; c < kMaxCand; c++) {
        int i = c * 32 + lane;
        p[c] = 0.0f;
        s[c] = 0.0f;
        if (i < E) {
            float l = logits[i], b = bias[i];
            float pv = sigmoid_ref(l);
            float sv = __fadd_rn(pv, b);
            if (!isfinite(l) || !isfinite(b) || !isfinite(sv)) {
                if ((uint32_t)i < bad_idx) {
                    bad_idx = (uint32_t)i;
                    bad_bits = !isfinite(l) ? __float_as_uint(l) : (!isfinite(b) ? __float_as_uint(b) : __float_as_uint(sv));
                }
            }
            p[c] = pv;
            s[c] = sv;
        }
    }
    uint32_t min_bad = bad_idx;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) min_bad = min(min_bad, __shfl_xor_sync(0xffffffffu, min_bad, o));
    if (min_bad != 0xffffffffu) {
        if (bad_idx == min_bad) report(st, LBK_NON_FINITE_ROUTING_VALUE, token * (uint64_t)E + min_bad, bad_bits);
        return;
    }
    uint32_t taken = 0;  // bit c: candidate c of this lane selected
    uint32_t sel_id[32];
    float sel_p[32];
    for (int r = 0; r < k; r++) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int c = 0; c < kMaxCand; c++) {
            int i = c * 32 + lane;
            if (i < E && !((taken >> c) & 1u)) {
                unsigned long long key = ((unsigned long long)ord_f32(s[c]) << 32) | (0xffffffffu - (uint32_t)i);
                best = key > best ? key : best;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        uint32_t id = 0xffffffffu - (uint32_t)(best & 0xffffffffull);
        int owner = (int)(id & 31), c_sel = (int)(id >> 5);
        float pv = 0.0f;
#pragma unroll
        for (int c = 0; c < kMaxCand; c++)
            if (c == c_sel) pv = p[c];
        pv = __shfl_sync(0xffffffffu, pv, owner);
        if (lane == owner) taken |= 1u << c_sel;
        sel_id[r] = id;
        sel_p[r] = pv;
    }
    if (lane == 0) {
        float wsum = 0.0f;
        for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, sel_p[r]);
        const float floor_v = 0.000061035156f;  // 2^-14 (routing.rs:5)
        wsum = wsum < floor_v ? floor_v : wsum;
        // output sorted by expert ID (routing.rs:105)
        for (int i = 1; i < k; i++) {
            uint32_t id = sel_id[i];
            float pv = sel_p[i];
            int j = i - 1;
            while (j >= 0 && sel_id[j] > id) {
                sel_id[j + 1] = sel_id[j];
                sel_p[j + 1] = sel_p[j];
                j--;
            }
            sel_id[j + 1] = id;
            sel_p[j + 1] = pv;
        }
        for (int r = 0; r < k; r++) {
            lbk_routed o;
            o.expert_id = sel_id[r];
            o.coefficient = __fmul_rn(__fdiv_rn(sel_p[r], wsum), weight_scale);
            out[r] = o;
        }
    }
}

__global__ void topk_kernel(TopkArgs a) {
    const int warp = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    for (uint64_t t = (uint64_t)blockIdx.x * nw + warp; t < a.tokens; t += (uint64_t)gridDim.x * nw)
        topk_warp(a.logits + t * a.experts, a.bias, (int)a.experts, (int)a.k, a.weight_scale, a.routed + t * a.k,
                  a.status, t);
}

// Sequential order: bit-identical to dot_f32_row (gemv.rs:286-303).
__global__ void router_seq_kernel(RouterArgs a) {
    uint64_t n = a.experts * a.tokens;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t t = i / a.experts, e = i % a.experts;
        const float* w = a.w + e * a.hidden;
        const float* x = a.x + t * a.hidden;
        float sum = 0.0f;
        for (uint64_t j = 0; j < a.hidden; j++) {
            float wv = w[j];
            if (!isfinite(wv)) report(a.status, LBK_NON_FINITE_VALUE, e * a.hidden + j, __float_as_uint(wv));
            sum = __fadd_rn(sum, __fmul_rn(wv, x[j]));
        }
        a.logits[t * a.experts + e] = sum;
    }
}

}  // namespace

namespace {

__global__ void __launch_bounds__(kRouterThreads) router_fused_kernel(RouterFusedArgs f) {
    const RouterArgs& a = f.r;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t chunks = (a.hidden + kChunk - 1) / kChunk;
    const uint64_t row_items = a.experts * chunks;
    const uint64_t nbq = f.q8x ? a.hidden / kQK : 0;
    const uint64_t items = row_items + a.tokens * nbq;
    const uint64_t nw = (uint64_t)gridDim.x * (kRouterThreads / 32);
    __shared__ bool s_last;

    for (uint64_t it = (uint64_t)blockIdx.x * (kRouterThreads / 32) + warp; it < items; it += nw) {
        if (it < row_items) {
            uint64_t e = it / chunks, c = it % chunks;
            uint64_t j0 = c * kChunk;
            const float* w = a.w + e * a.hidden;
            float wr[16];
#pragma unroll
            for (int q = 0; q < 16; q++) {
                uint64_t j = j0 + (uint64_t)q * 32 + lane;
                wr[q] = j < a.hidden ? __ldcs(w + j) : 0.0f;
                if (j < a.hidden && !isfinite(wr[q])) report(a.status, LBK_NON_FINITE_VALUE, e * a.hidden + j, __float_as_uint(wr[q]));
            }
            for (uint64_t t = 0; t < a.tokens; t++) {
                const float* x = a.x + t * a.hidden;
                float acc = 0.0f;
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    uint64_t j = j0 + (uint64_t)q * 32 + lane;
                    float xv = j < a.hidden ? __ldg(x + j) : 0.0f;
                    acc = __fadd_rn(acc, __fmul_rn(wr[q], xv));
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
                if (lane == 0) f.partials[(t * a.experts + e) * chunks + c] = acc;
            }
        } else {
            uint64_t q = it - row_items;
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
                continue;
            }
            Q8Block qb = quantize_q8k_warp(v, lane);
            uint8_t* o = f.q8x + (t * nbq + b) * kQ8Bytes;
            uint32_t* ow = reinterpret_cast<uint32_t*>(o + 4);
            ow[lane * 2] = qb.q[0];
            ow[lane * 2 + 1] = qb.q[1];
            int32_t pair = qb.pair_sum + __shfl_xor_sync(0xffffffffu, qb.pair_sum, 1);
            if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(o + 260 + lane) = (int16_t)pair;
            if (lane == 0) *reinterpret_cast<float*>(o) = qb.d;
        }
    }

    // The last CTA to finish sums the chunk partials in chunk order and routes.
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
    if (f.routed != nullptr) {
        for (uint64_t t = warp; t < a.tokens; t += kRouterThreads / 32)
            topk_warp(a.logits + t * a.experts, f.bias, (int)a.experts, (int)f.k, f.weight_scale, f.routed + t * f.k,
                      a.status, t);
    }
    if (threadIdx.x == 0) *f.counter = 0u;
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
    router_fused_kernel<<<(unsigned)ctas, kRouterThreads, 0, stream>>>(f);
    return cudaGetLastError();
}

cudaError_t launch_router(const RouterArgs& a, int mode, int sm_count, cudaStream_t stream) {
    (void)mode;
    uint64_t n = a.experts * a.tokens;
    uint64_t grid = (n + 127) / 128;
    if (grid > (uint64_t)sm_count * 8) grid = (uint64_t)sm_count * 8;
    if (grid < 1) grid = 1;
    router_seq_kernel<<<(unsigned)grid, 128, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_topk(const TopkArgs& a, cudaStream_t stream) {
    uint64_t grid = (a.tokens + 7) / 8;
    if (grid < 1) grid = 1;
    topk_kernel<<<(unsigned)grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace lbk
