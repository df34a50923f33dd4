// lbk_topk.cuh -- Hy3 top-k routing of one token by one warp.
//
// Restates route_experts_into (bridge-model-hy3/src/routing.rs:25-107):
// validate every logit, bias and selection score in order (the first bad one
// is reported); p = sigmoid(logit); selection score = p + bias; k rounds of a
// warp arg-max over (score, lowest ID); weight sum over the selected p in
// selection order with the 2^-14 floor; coef = p / sum * weight_scale;
// output sorted by expert ID.
#pragma once

#include "lbk_device.cuh"

namespace lbk {

__device__ __forceinline__ uint32_t ord_f32(float f) {
    if (f == 0.0f) f = 0.0f;  // -0 and +0 compare equal in the reference sort
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// C = candidates per lane (E <= 32*C).
template <int C>
__device__ void topk_warp_c(const float* logits, const float* bias, int E, int k, float weight_scale, lbk_routed* out,
                            DeviceStatus* st, uint64_t token) {
    const int lane = threadIdx.x & 31;
    float p[C], s[C];
    uint32_t bad_idx = 0xffffffffu, bad_bits = 0;
#pragma unroll
    for (int c = 0; c < C; c++) {
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
    // per-lane keys, refreshed only on the lane that lost a candidate
    unsigned long long key[C];
#pragma unroll
    for (int c = 0; c < C; c++) {
        int i = c * 32 + lane;
        key[c] = i < E ? ((unsigned long long)ord_f32(s[c]) << 32) | (0xffffffffu - (uint32_t)i) : 0ull;
    }
    uint32_t sel_id = 0;
    float sel_p = 0.0f;  // lane r holds the r-th selection
    for (int r = 0; r < k; r++) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int c = 0; c < C; c++) best = key[c] > best ? key[c] : best;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        uint32_t id = 0xffffffffu - (uint32_t)(best & 0xffffffffull);
        int owner = (int)(id & 31), c_sel = (int)(id >> 5);
        float pv = 0.0f;
#pragma unroll
        for (int c = 0; c < C; c++)
            if (c == c_sel) pv = p[c];
        pv = __shfl_sync(0xffffffffu, pv, owner);
        if (lane == owner) {
#pragma unroll
            for (int c = 0; c < C; c++)
                if (c == c_sel) key[c] = 0ull;
        }
        if (lane == r) {
            sel_id = id;
            sel_p = pv;
        }
    }
    // weight sum in selection order (lane order r = 0..k-1)
    float wsum = 0.0f;
    for (int r = 0; r < k; r++) wsum = __fadd_rn(wsum, __shfl_sync(0xffffffffu, sel_p, r));
    const float floor_v = 0.000061035156f;  // 2^-14 (routing.rs:5)
    wsum = wsum < floor_v ? floor_v : wsum;
    // rank of this selection by expert ID (IDs are distinct)
    int rank = 0;
    for (int r = 0; r < k; r++) {
        uint32_t other = __shfl_sync(0xffffffffu, sel_id, r);
        rank += (r < k && other < sel_id) ? 1 : 0;
    }
    if (lane < k) {
        lbk_routed o;
        o.expert_id = sel_id;
        o.coefficient = __fmul_rn(__fdiv_rn(sel_p, wsum), weight_scale);
        out[rank] = o;
    }
}

__device__ __forceinline__ void topk_warp(const float* logits, const float* bias, int E, int k, float weight_scale,
                                          lbk_routed* out, DeviceStatus* st, uint64_t token) {
    if (E <= 64)
        topk_warp_c<2>(logits, bias, E, k, weight_scale, out, st, token);
    else if (E <= 256)
        topk_warp_c<8>(logits, bias, E, k, weight_scale, out, st, token);
    else
        topk_warp_c<32>(logits, bias, E, k, weight_scale, out, st, token);
}

}  // namespace lbk
