// lbk_topk.cuh -- Hy3 top-k routing of one token by one warp.
//
// Restates route_experts_into (bridge-model-hy3/src/routing.rs:25-107):
// validate every logit, bias and selection score in order (the first bad one
// is reported); p = sigmoid(logit); selection score = p + bias; k rounds of a
// warp arg-max over (score, lowest ID); weight sum over the selected p in
// selection order with the 2^-14 floor; coef = p / sum * weight_scale;
// output sorted by expert ID.
//
// Written as rolled loops over a scratch copy of the scores: the kernels that
// call it run it once per launch, so its code is fetched cold every time and
// code size, not instruction count, sets its latency.
#pragma once

#include "lbk_device.cuh"

namespace lbk {

__device__ __forceinline__ uint32_t ord_f32(float f) {
    if (f == 0.0f) f = 0.0f;  // -0 and +0 compare equal in the reference sort
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Selection key: score order, then the lower expert ID; 0 = removed (NaN).
__device__ __forceinline__ unsigned long long topk_key(float s, int i) {
    return isnan(s) ? 0ull : ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)i);
}

// Best key among this lane's candidates i = lane, lane + 32, ...
__device__ __forceinline__ unsigned long long topk_lane_best(const float* s_score, int E, int lane) {
    unsigned long long best = 0ull;
#pragma unroll 1
    for (int i = lane; i < E; i += 32) {
        const unsigned long long key = topk_key(s_score[i], i);
        best = key > best ? key : best;
    }
    return best;
}

// One token. s_score / s_p: scratch of E floats each, private to this warp
// (s_score may alias `logits`: element i is read before it is written, by
// the same lane).
static __device__ __noinline__ void topk_warp(const float* logits, const float* bias, int E, int k, float weight_scale,
                                       lbk_routed* out, DeviceStatus* st, uint64_t token, float* s_score, float* s_p) {
    const int lane = threadIdx.x & 31;
    uint32_t bad_idx = 0xffffffffu, bad_bits = 0;
#pragma unroll 1
    for (int i = lane; i < E; i += 32) {
        const float l = logits[i], b = bias[i];
        const float pv = sigmoid_ref(l);
        const float sv = __fadd_rn(pv, b);
        if ((!isfinite(l) || !isfinite(b) || !isfinite(sv)) && (uint32_t)i < bad_idx) {
            bad_idx = (uint32_t)i;
            bad_bits = !isfinite(l) ? __float_as_uint(l) : (!isfinite(b) ? __float_as_uint(b) : __float_as_uint(sv));
        }
        s_p[i] = pv;
        s_score[i] = sv;
    }
    const uint32_t min_bad = __reduce_min_sync(0xffffffffu, bad_idx);
    if (min_bad != 0xffffffffu) {
        if (bad_idx == min_bad) report(st, LBK_NON_FINITE_ROUTING_VALUE, token * (uint64_t)E + min_bad, bad_bits);
        return;
    }
    __syncwarp();
    // k rounds; a lane's best key changes only when its candidate is taken
    unsigned long long best = topk_lane_best(s_score, E, lane);
    uint32_t sel_id = 0;
    float sel_p = 0.0f;  // lane r holds the r-th selection
#pragma unroll 1
    for (int r = 0; r < k; r++) {
        const uint32_t hi = (uint32_t)(best >> 32);
        const uint32_t top = __reduce_max_sync(0xffffffffu, hi);
        const uint32_t lo = __reduce_max_sync(0xffffffffu, hi == top ? (uint32_t)best : 0u);
        const uint32_t id = 0xffffffffu - lo;
        if (lane == (int)(id & 31)) {
            s_score[id] = __int_as_float(0x7fffffff);
            best = topk_lane_best(s_score, E, lane);
        }
        if (lane == r) {
            sel_id = id;
            sel_p = s_p[id];
        }
    }
    // weight sum in selection order (lane order r = 0..k-1)
    float wsum = 0.0f;
#pragma unroll 1
    for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, sel_p, r));
    const float floor_v = 0.000061035156f;  // 2^-14 (routing.rs:5)
    wsum = wsum < floor_v ? floor_v : wsum;
    // rank of this selection by expert ID (IDs are distinct)
    int rank = 0;
#pragma unroll 1
    for (int r = 0; r < k; r++) rank += __shfl_sync(0xffffffffu, sel_id, r) < sel_id ? 1 : 0;
    if (lane < k) {
        lbk_routed o;
        o.expert_id = sel_id;
        o.coefficient = __fmul_rn(__fdiv_rn(sel_p, wsum), weight_scale);
        out[rank] = o;
    }
    __syncwarp();
}

// The same routing by every thread of a CTA: one thread per expert for the
// logit sums and p / score, then each expert's rank among all keys
// (a selected expert's rank is its selection round), then warp 0 finishes
// as topk_warp does. Shared scratch: s_key[E], s_p[E], s_sel[k], *s_bad.
// partials: [E][chunks] chunk sums of the router dot, added in chunk order.
// Every thread must call it; on a non-finite value it reports, zero-fills
// `out` and returns false.
static __device__ __noinline__ bool topk_cta(const float* partials, int chunks, const float* bias, int E, int k,
                                      float weight_scale, lbk_routed* out, DeviceStatus* st, unsigned long long* s_key,
                                      float* s_p, uint32_t* s_sel, int* s_bad) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) *s_bad = 0x7fffffff;
    __syncthreads();
#pragma unroll 1
    for (int i = tid; i < E; i += nt) {
        const float* pp = partials + (size_t)i * chunks;
        float l = 0.0f;
#pragma unroll 1
        for (int c = 0; c < chunks; c++) l = __fadd_rn(l, pp[c]);
        const float b = bias[i];
        const float pv = sigmoid_ref(l);
        const float sv = __fadd_rn(pv, b);
        if (!isfinite(l) || !isfinite(b) || !isfinite(sv)) atomicMin(s_bad, i);
        s_p[i] = pv;
        s_key[i] = topk_key(sv, i);
    }
    __syncthreads();
    const int bad = *s_bad;
    if (bad != 0x7fffffff) {
        if (tid == 0) {
            const float* pp = partials + (size_t)bad * chunks;
            float l = 0.0f;
            for (int c = 0; c < chunks; c++) l = __fadd_rn(l, pp[c]);
            const float b = bias[bad], sv = __fadd_rn(sigmoid_ref(l), b);
            report(st, LBK_NON_FINITE_ROUTING_VALUE, (uint64_t)bad,
                   !isfinite(l) ? __float_as_uint(l) : (!isfinite(b) ? __float_as_uint(b) : __float_as_uint(sv)));
        }
        if (tid < k) out[tid] = lbk_routed{0u, 0.0f};
        __syncthreads();
        return false;
    }
    // each expert's rank, counted by two adjacent threads over halves of the keys
    const int half = (E + 1) >> 1;
#pragma unroll 1
    for (int base = 0; base < 2 * E; base += nt) {
        const int i = base + tid, e = i >> 1, h = i & 1;
        int part = 0;
        if (i < 2 * E) {
            const unsigned long long key = s_key[e];
            const int j1 = h ? E : half;
#pragma unroll 8
            for (int j = h ? half : 0; j < j1; j++) part += s_key[j] > key ? 1 : 0;
        }
        const int rank = part + __shfl_xor_sync(0xffffffffu, part, 1);
        if (i < 2 * E && h == 0 && rank < k) s_sel[rank] = (uint32_t)e;
    }
    __syncthreads();
    if (tid < 32) {
        const int lane = tid;
        const uint32_t sel_id = lane < k ? s_sel[lane] : 0xffffffffu;
        const float sel_p = lane < k ? s_p[sel_id] : 0.0f;
        float wsum = 0.0f;
#pragma unroll 1
        for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, sel_p, r));
        const float floor_v = 0.000061035156f;  // 2^-14 (routing.rs:5)
        wsum = wsum < floor_v ? floor_v : wsum;
        int rank = 0;
#pragma unroll 1
        for (int r = 0; r < k; r++) rank += __shfl_sync(0xffffffffu, sel_id, r) < sel_id ? 1 : 0;
        if (lane < k) out[rank] = lbk_routed{sel_id, __fmul_rn(__fdiv_rn(sel_p, wsum), weight_scale)};
    }
    __syncthreads();
    return true;
}

}  // namespace lbk
