// moe.cu -- fused routed + shared SwiGLU expert FFN over HBM-resident tables.
//
// Replaces the per-token expert work of hy3_moe_finish_token
// (bridge-kernels-reference/src/layer.rs:610-659) -> moe_routed_by_id_into
// (moe.rs:64-147) -> expert_swiglu_accumulate_into (activation.rs:104-144) ->
// gemv_into / gemv_accumulate_scaled_into (gemv.rs:88-174):
//
//   gate/up kernel: for every (token, slot) -- slot j < k the j-th routed
//     expert in ascending ID, slot k the shared expert -- both projections of
//     the token's Q8_K activations, SwiGLU (activation.rs:170-178), and the
//     Q8_K quantization of the hidden vector, done per 256-row block by the
//     warp that completes the block (arrival counter, no grid barrier);
//   down kernel: every output row's k+1 down-projection dots, then
//     out = 0; out += c_j * dot_j (ascending ID); out += 1.0 * dot_shared --
//     the reference's exact f32 combine order (moe.rs:331-336).
//
// The reference runs every expert twice (a preflight pass into scratch, then
// the accepting pass); here validation is carried by the device status word
// instead: a non-finite SwiGLU value or scale is reported and the down kernel
// then leaves `out` untouched.

#include "lbk_kernels.h"
#include "lbk_moe.h"
#include "lbk_topk.cuh"

namespace lbk {

namespace {

// 8 warps per SM with deep per-warp prefetch: registers, not warps, carry
// the bytes in flight (about 80 KB per SM for IQ2_S gate/up).
constexpr int kGUThreads = kMoeGateUpWarps * 32;
constexpr int kGUWarps = kMoeGateUpWarps;
constexpr int kDownMaxThreads = kMoeDownMaxSlots * 32;  // one warp per slot, top-k <= 8

// Prefetch ring depth (steps of rps rows held in registers) per weight type.
template <int T>
struct RingDepth {
    static constexpr bool kIq = (T == LBK_TYPE_IQ2_S || T == LBK_TYPE_IQ3_S);
    static constexpr int kGateUp = kIq ? 4 : 1;  // two matrices per step
    static constexpr int kDown = 3;  // 9 warps share 4 SMSPs: <= 168 registers per thread
};

template <int T>
struct HBOf;
template <>
struct HBOf<LBK_TYPE_IQ2_S> {
    using type = Iq2HB;
};
template <>
struct HBOf<LBK_TYPE_IQ3_S> {
    using type = Iq3HB;
};
template <>
struct HBOf<LBK_TYPE_Q4_K> {
    using type = Q4HB;
};
template <>
struct HBOf<LBK_TYPE_Q5_K> {
    using type = Q5HB;
};

template <int T>
constexpr bool is_iq() {
    return T == LBK_TYPE_IQ2_S || T == LBK_TYPE_IQ3_S;
}

// Loads a thread's half block of a Q8_K row held in global memory in the
// internal image layout (store_q8i). The image was written by an earlier
// launch and every warp of the grid reads it: read-only loads through L1, so
// each SM fetches a line from L2 once instead of once per warp (thousands of
// warps on the same few lines would stall every other L2 request behind them).
template <bool kTr>
__device__ __forceinline__ void load_act_global(ActHB& a, const uint8_t* q8row, int b, int h, bool bsums) {
    const uint8_t* blk = q8row + (size_t)b * kQ8IBytes;
    const uint4* qw = reinterpret_cast<const uint4*>(blk + 128 * h);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint4 v = __ldg(qw + i);
        a.w[4 * i + 0] = v.x;
        a.w[4 * i + 1] = v.y;
        a.w[4 * i + 2] = v.z;
        a.w[4 * i + 3] = v.w;
    }
    if (kTr) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t n[8];
#pragma unroll
            for (int i = 0; i < 8; i++) n[i] = a.w[8 * j + i];
            transpose4(n[0], n[2], n[4], n[6], a.w[8 * j + 0], a.w[8 * j + 1], a.w[8 * j + 2], a.w[8 * j + 3]);
            transpose4(n[1], n[3], n[5], n[7], a.w[8 * j + 4], a.w[8 * j + 5], a.w[8 * j + 6], a.w[8 * j + 7]);
        }
    }
    a.d = __uint_as_float(__ldg(reinterpret_cast<const unsigned int*>(blk + 288)));
    uint4 bs = bsums ? __ldg(reinterpret_cast<const uint4*>(blk + 256 + 16 * h)) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < 8; i++) a.bsum[i] = (int32_t)(int16_t)((w32(bs, i >> 1) >> (16 * (i & 1))) & 0xffffu);
}

// Integer dot of one half block, dispatched on the weight type.
template <int T>
struct HBDot {
    // t0: shared-window address of this lane's copy of the type's table.
    template <class HB>
    __device__ __forceinline__ static void run(const HB& w, const ActHB& a, const uint32_t* na, uint32_t t0, int h,
                                               IqPart& ip, KPart& kp) {
        if constexpr (T == LBK_TYPE_IQ2_S) {
            ip = dot_hb(w, a, t0);
        } else if constexpr (T == LBK_TYPE_IQ3_S) {
            ip = dot_hb(w, a, na, t0);
        } else {
            kp = dot_hb(w, a, h);
        }
        (void)na;
        (void)h;
    }
};

// Tails of a warp's batch: prod[(row*nmat + mat)][nb][kTail] -> res[row*nmat + mat].
// Chains are spread over lanes (one lane per chain), so a batch costs about
// nb dependent adds regardless of its size.
template <int T>
__device__ __forceinline__ void warp_tails(const float* prod, int ndots, int nb, float* chains, float* res) {
    const int lane = threadIdx.x & 31;
    if constexpr (is_iq<T>()) {
        for (int c = lane; c < ndots; c += 32) {
            float v = iq_tail(prod + (size_t)c * nb, nb, 1, T == LBK_TYPE_IQ2_S);
            res[c] = v;
        }
    } else {
        for (int c = lane; c < ndots * 9; c += 32) {
            int d = c / 9, l = c % 9;
            const float* p = prod + (size_t)d * nb * 9 + l;
            float acc = 0.0f;
            if (l < 8) {
                for (int b = 0; b < nb; b++) acc = __fadd_rn(acc, p[b * 9]);
            } else {
                for (int b = 0; b < nb; b++) acc = __fsub_rn(acc, p[b * 9]);
            }
            chains[c] = acc;
        }
        __syncwarp();
        for (int d = lane; d < ndots; d += 32) {
            float sum = chains[d * 9 + 8];
#pragma unroll
            for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, chains[d * 9 + l]);
            res[d] = sum;
        }
    }
    __syncwarp();
}

// Per-row products of one half block pair, written into prod[dot][b][kTail]
// by the lane holding half 0 when `store`. Every lane computes them (no
// divergent branch); the store alone is predicated. The binary16 scales were
// checked when the layer was created (the reference's validate_scales,
// k_quants.rs:178-208, hoisted out of the call: the weights are immutable).
template <int T>
__device__ __forceinline__ void write_products(float* prod_dot, int b, int h, bool store, IqPart ip, KPart kp, float dx) {
    if constexpr (is_iq<T>()) {
        ip.sum += __shfl_xor_sync(0xffffffffu, ip.sum, 1);
        const float p = iq_block_product(ip, dx);
        if (store && h == 0) prod_dot[b] = p;
    } else {
#pragma unroll
        for (int l = 0; l < 8; l++) kp.lane[l] += __shfl_xor_sync(0xffffffffu, kp.lane[l], 1);
        kp.min_sum += __shfl_xor_sync(0xffffffffu, kp.min_sum, 1);
        float pr[9];
        k_block_products(kp, dx, pr);
        if (store && h == 0) {
#pragma unroll
            for (int i = 0; i < 9; i++) prod_dot[b * 9 + i] = pr[i];
        }
    }
}

// The routed role's work when the item count is read on the device
// (expert-parallel items; a.tokens is the capacity): the host's chunking
// (rows spread over the role's warps in whole steps of R rows) on the count.
struct RoleWork {
    uint32_t tokens, chunk, chunks;
};
__device__ __forceinline__ RoleWork device_work(const uint32_t* d_items, uint64_t cap, uint32_t slots, uint32_t warps,
                                                uint32_t rows, uint32_t R) {
    uint32_t n = __ldcg(d_items);
    n = n < cap ? n : (uint32_t)cap;
    uint32_t per = n ? warps / (n * slots) : 1u;
    per = per < 1u ? 1u : per;
    uint32_t c = (rows + per - 1) / per;
    c = (c + R - 1) / R * R;
    return RoleWork{n, c, (rows + c - 1) / c};
}

template <int T>
constexpr int table_bytes() {
    return T == LBK_TYPE_IQ2_S ? kIq2CodeBytes : (T == LBK_TYPE_IQ3_S ? kIq3GridBytes : 0);
}

template <int T>
__device__ __forceinline__ void fill_tables(uint32_t* tab, const Tables& t) {
    if constexpr (T == LBK_TYPE_IQ2_S) fill_iq2_codes(tab, t);
    if constexpr (T == LBK_TYPE_IQ3_S) fill_iq3_grid(tab, t);
}

__device__ __forceinline__ uint32_t lane_addr(const uint32_t* tab) {
    return (uint32_t)__cvta_generic_to_shared(tab + (threadIdx.x & 31));
}

// ---------------------------------------------------------------- gate / up

// One warp = one (token, slot, row chunk). Shared memory:
//   [routed-type table][shared-type table][sign table][per-warp prod][per-warp chains/results]
template <int TG, int TS>
struct GUSmem {
    static constexpr int kTabG = table_bytes<TG>();
    static constexpr int kTabS = (TS == TG) ? 0 : table_bytes<TS>();
    static constexpr int kFixed = kTabG + kTabS;
};

template <int T>
__device__ __forceinline__ void gate_up_rows(const MoeGateUpArgs& a, uint64_t t, uint64_t slot, const uint8_t* gmat,
                                             const uint8_t* umat, uint64_t r0, uint64_t r1, float* prod, float* chains,
                                             float* res, const uint32_t* tab) {
    using HB = typename HBOf<T>::type;
    constexpr bool kIq = is_iq<T>();
    const int lane = threadIdx.x & 31;
    const int nb = a.nb_h;
    const int tpr = a.tpr_h;
    const int rps = 32 / tpr;
    const int sub = lane / tpr, hb = lane % tpr;
    const int b = hb >> 1, h = hb & 1;
    const bool lane_on = hb < 2 * nb;
    constexpr int kTail = TypeInfo<T>::kTail;

    ActHB act;
    uint32_t nact[32];
    if (lane_on) {
        load_act_global<!kIq>(act, a.q8x + t * (uint64_t)nb * kQ8IBytes, b, h, !kIq);
        if constexpr (T == LBK_TYPE_IQ3_S) {
#pragma unroll
            for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
        }
    }
    const uint32_t t0 = lane_addr(tab);
    MatrixRef gm{gmat, a.ffn, nb}, um{umat, a.ffn, nb};

    // Rows stream through a ring of D prefetched steps held in registers
    // (the loads of step i+D are issued before step i is decoded); every
    // `bmax` rows (a multiple of rps) the batch's tails and SwiGLU are replayed.
    constexpr int D = RingDepth<T>::kGateUp;
    const int bmax = kIq ? a.bmax_iq : a.bmax_k;
    float* hrow = a.h + (t * (a.k + 1) + slot) * a.ffn;
    HB gbuf[D], ubuf[D];
#pragma unroll
    for (int i = 0; i < D; i++) {
        const uint64_t row = r0 + (uint64_t)i * rps + sub;
        if (lane_on && row < r1) {
            load_hb<LBK_LAYOUT_PLANAR>(gbuf[i], gm, row, b, h);
            load_hb<LBK_LAYOUT_PLANAR>(ubuf[i], um, row, b, h);
        }
    }
    uint64_t rb = r0;
    for (uint64_t base = r0; base < r1; base += (uint64_t)D * rps) {
#pragma unroll
        for (int i = 0; i < D; i++) {
            const uint64_t r = base + (uint64_t)i * rps;
            if (r >= r1) break;  // warp-uniform
            const uint64_t row = r + sub;
            const bool mine = lane_on && row < r1;
            const HB gw = gbuf[i], uw = ubuf[i];
            const uint64_t nrow = row + (uint64_t)D * rps;
            if (lane_on && nrow < r1) {
                load_hb<LBK_LAYOUT_PLANAR>(gbuf[i], gm, nrow, b, h);
                load_hb<LBK_LAYOUT_PLANAR>(ubuf[i], um, nrow, b, h);
            }
            IqPart gi{0, 0}, ui{0, 0};
            KPart gk, uk;
#pragma unroll
            for (int l = 0; l < 8; l++) gk.lane[l] = uk.lane[l] = 0;
            gk.min_sum = uk.min_sum = 0;
            gk.dm = uk.dm = 0;
            if (mine) {
                HBDot<T>::run(gw, act, nact, t0, h, gi, gk);
                HBDot<T>::run(uw, act, nact, t0, h, ui, uk);
            }
            const int ri = (int)(row - rb);
            float* pg = prod + (size_t)(ri * 2 + 0) * nb * kTail;
            float* pu = prod + (size_t)(ri * 2 + 1) * nb * kTail;
            write_products<T>(pg, b, h, mine, gi, gk, act.d);
            write_products<T>(pu, b, h, mine, ui, uk, act.d);
            const uint64_t rn = r + rps;
            if (rn - rb >= (uint64_t)bmax || rn >= r1) {
                const int nrows = (int)((rn < r1 ? rn : r1) - rb);
                __syncwarp();
                warp_tails<T>(prod, nrows * 2, nb, chains, res);
                // SwiGLU per row; one lane per row
                for (int q = lane; q < nrows; q += 32) {
                    float g = res[q * 2], u = res[q * 2 + 1];
                    float v = swiglu_ref(g, u);
                    if (!isfinite(v))
                        report(a.status, LBK_NON_FINITE_VALUE, (t * (a.k + 1) + slot) * a.ffn + rb + q,
                               __float_as_uint(v));
                    hrow[rb + q] = v;
                }
                __syncwarp();
                rb = rn;
            }
        }
    }
}

// Arrival counting on the 256-row Q8_K blocks of h; the completing warp
// quantizes the block (quantize_row_q8_k_into, q8_k.rs:35-73).
__device__ __forceinline__ void arrive_and_quantize(const MoeGateUpArgs& a, uint64_t t, uint64_t slot, uint64_t r0,
                                                   uint64_t r1) {
    const int lane = threadIdx.x & 31;
    const uint64_t sidx = t * (a.k + 1) + slot;
    for (uint64_t blk = r0 / kQK; blk * kQK < r1; blk++) {
        uint64_t lo = blk * kQK > r0 ? blk * kQK : r0;
        uint64_t hi = (blk + 1) * kQK < r1 ? (blk + 1) * kQK : r1;
        unsigned n = (unsigned)(hi - lo);
        unsigned int* cnt = a.counters + sidx * a.nb_f + blk;
        unsigned old = 0;
        __syncwarp();  // the lanes' h stores before lane 0's release
        if (lane == 0) old = atom_add_acq_rel_gpu(cnt, n);
        old = __shfl_sync(0xffffffffu, old, 0);
        __syncwarp();  // lane 0's acquire before the lanes' reads below
        if (old + n != (unsigned)kQK) continue;
        const float* hb = a.h + sidx * a.ffn + blk * kQK + lane * 8;
        float v[8];
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            v[i] = __ldcg(hb + i);
            bad |= !isfinite(v[i]);
        }
        if (lane == 0) *cnt = 0u;  // ready for the next launch
        if (__ballot_sync(0xffffffffu, bad)) continue;  // already reported by the SwiGLU check
        Q8Block q = quantize_q8k_warp(v, lane);
        int32_t pair = q.pair_sum + __shfl_xor_sync(0xffffffffu, q.pair_sum, 1);
        store_q8i(a.hq + (sidx * a.nb_f + blk) * kQ8IBytes, q, pair, lane);
    }
}

template <int TG, int TS>
__global__ void __launch_bounds__(kGUThreads, 1) moe_gate_up_kernel(MoeGateUpArgs a) {
    using S = GUSmem<TG, TS>;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tabG = reinterpret_cast<uint32_t*>(smem);
    uint32_t* tabS = S::kTabS ? reinterpret_cast<uint32_t*>(smem + S::kTabG) : tabG;
    float* prod_all = reinterpret_cast<float*>(smem + S::kFixed);
    const int warp = threadIdx.x >> 5;
    float* prod = prod_all + (size_t)warp * a.prod_floats;
    float* chains = prod_all + (size_t)kGUWarps * a.prod_floats + (size_t)warp * a.chain_floats;
    float* res = chains + a.chain_floats - 64;

    // Single-token decode: every CTA finishes the router itself (sum of the
    // chunk partials in chunk order, then top-k) while the other warps copy
    // the tables; CTA 0 publishes the routing for the down kernel.
    __shared__ float s_logits[1024];
    __shared__ float s_tkp[1024];
    __shared__ lbk_routed s_routed[32];
    if (a.defer_topk && warp == 0) {
        const int lane = threadIdx.x & 31;
        for (uint64_t e = lane; e < a.experts; e += 32) {
            const float* pp = a.partials + e * a.chunks;
            float sum = 0.0f;
            for (uint64_t c = 0; c < a.chunks; c++) sum = __fadd_rn(sum, __ldcg(pp + c));
            s_logits[e] = sum;
        }
        __syncwarp();
        topk_warp(s_logits, a.bias, (int)a.experts, (int)a.k, a.weight_scale, s_routed,
                  blockIdx.x == 0 ? a.status : nullptr, 0, s_logits, s_tkp);
        __syncwarp();
        if (blockIdx.x == 0 && lane < (int)a.k) a.routed_store[lane] = s_routed[lane];
    }
    fill_tables<TG>(tabG, a.tables);
    if constexpr (S::kTabS != 0) fill_tables<TS>(tabS, a.tables);
    __syncthreads();

    const uint64_t gw = (uint64_t)blockIdx.x * kGUWarps + warp;
    const uint64_t routed_items = a.tokens * a.k * a.chunks_r;
    const uint64_t shared_items = a.tokens * a.chunks_s;
    if (gw < routed_items) {
        uint64_t t = gw / (a.k * a.chunks_r);
        uint64_t rem = gw % (a.k * a.chunks_r);
        uint64_t j = rem / a.chunks_r, c = rem % a.chunks_r;
        uint32_t e = a.defer_topk ? s_routed[j].expert_id : a.routed[t * a.k + j].expert_id;
        if (e >= a.experts) {  // reported; compute on expert 0 so the arrival counts stay balanced
            if ((threadIdx.x & 31) == 0) report(a.status, LBK_INVALID_PARAMETER, e, 0);
            e = 0;
        }
        uint64_t r0 = c * a.chunk_r, r1 = r0 + a.chunk_r < a.ffn ? r0 + a.chunk_r : a.ffn;
        gate_up_rows<TG>(a, t, j, a.gate[e], a.up[e], r0, r1, prod, chains, res, tabG);
        arrive_and_quantize(a, t, j, r0, r1);
    } else if (gw < routed_items + shared_items) {
        uint64_t q = gw - routed_items;
        uint64_t t = q / a.chunks_s, c = q % a.chunks_s;
        uint64_t r0 = c * a.chunk_s, r1 = r0 + a.chunk_s < a.ffn ? r0 + a.chunk_s : a.ffn;
        gate_up_rows<TS>(a, t, a.k, a.sgate, a.sup, r0, r1, prod, chains, res, tabS);
        arrive_and_quantize(a, t, a.k, r0, r1);
    }
}

// ------------------------------------------------- gate / up, bulk-copy staged
//
// For planar weights with nb_h a multiple of 8 and at most 16: every planar
// field of a row is then a multiple of 16 bytes, and one warp step of
// 32/tpr rows covers exactly 32 half blocks. CTAs [0, routed_ctas) take the
// routed slots and hold the routed type's lookup tables; the other CTAs take
// the shared expert and hold none. Each warp owns one stage in shared memory:
// lane 0 fills it with bulk copies (one per planar field of gate and of up)
// completing on the warp's mbarrier; the lanes copy their half blocks into
// registers, lane 0 refills the stage with the next step's rows, and this
// step's decode overlaps that transfer.

constexpr int kGUTWarps = kMoeGateUpTmaWarps;
constexpr int kGUTThreads = kGUTWarps * 32;

// Shared-memory plan of one CTA role streaming type T.
template <int T>
struct GUTRole {
    static constexpr bool kIq = is_iq<T>();
    static constexpr int kBB = TypeInfo<T>::kBlockBytes;
    static constexpr int kMat = 16 * kBB;                 // 32 half blocks of one matrix (16-byte multiple)
    static constexpr int kStage = 2 * kMat;               // gate + up
    static constexpr int kBmax = kIq ? 8 : 4;             // rows per tail batch
    static constexpr int kTail = TypeInfo<T>::kTail;
    static constexpr int kProd = kBmax * 2 * 16 * kTail;  // floats per warp
    static constexpr int kChain = kIq ? 0 : kBmax * 2 * 9;
    static constexpr int kRes = 64;
    static constexpr int kTab = table_bytes<T>();
    static constexpr int kRingOff = kTab;
    static constexpr int kProdOff = kRingOff + kGUTWarps * kStage;
    static constexpr int kChainOff = kProdOff + kGUTWarps * kProd * 4;
    static constexpr int kResOff = kChainOff + kGUTWarps * kChain * 4;
    static constexpr int kBytes = kResOff + kGUTWarps * kRes * 4;
};

// Lane 0: rows [ra, ra+nr) of one matrix, one contiguous planar copy (rows
// at stride rs), into a stage.
__device__ __forceinline__ void gut_issue(uint32_t stage, uint32_t bar, const uint8_t* mat, uint32_t rs, uint32_t ra,
                                          uint32_t nr) {
    mbar_expect_tx(bar, nr * rs);
    bulk_g2s_stream(stage, mat + (uint64_t)ra * rs, nr * rs, bar, policy_evict_first());
}

// Lane 0: rows [ra, ra+nr) of gate and of up into the two halves of a stage,
// both completing on one mbarrier (one expected byte count).
__device__ __forceinline__ void gut_issue2(uint32_t stage, uint32_t bar, const uint8_t* gmat, const uint8_t* umat,
                                           uint32_t rs, uint32_t mat_bytes, uint32_t ra, uint32_t nr) {
    mbar_expect_tx(bar, 2 * nr * rs);
    const uint64_t pol = policy_evict_first();
    bulk_g2s_stream(stage, gmat + (uint64_t)ra * rs, nr * rs, bar, pol);
    bulk_g2s_stream(stage + mat_bytes, umat + (uint64_t)ra * rs, nr * rs, bar, pol);
}

// Wait for the phase with the given parity: one poll when the data is there
// (the common case), else the bounded wait. False when it ran out.
__device__ __forceinline__ bool stage_wait(uint32_t bar, uint32_t parity) {
    return mbar_try_wait(bar, parity) || mbar_wait(bar, parity);
}

// One role's items: (token, slot, chunk of rows) spread over the role's warps.
// Work step: R rows (32 half blocks) of gate and the same rows of up, one
// stage holding both and one mbarrier; the refill for the next step is issued
// as soon as the stage is copied to registers, so it lands while this step is
// decoded. dep_wait: the grid dependency (router output) is still to be
// waited for, after the first copies.
// s_ptr: the gate / up pointer tables staged in shared memory (gate at 0, up
// at kPtrMax), or null.
constexpr int kPtrMax = 256;

// This CTA's slice of every down matrix the call will read heads for L2:
// HBM streams it while the gate/up rows are being decoded. One matrix per
// warp (lane 0): a bulk prefetch can hold its thread while the SM's copy
// queue is full.
__device__ __forceinline__ void prefetch_down_rows(const MoeGateUpArgs& a, const lbk_routed* s_routed, uint32_t rcta) {
    const int warp = threadIdx.x >> 5;
    const uint64_t H = a.hidden, n = a.tokens * a.k;
    const uint64_t p0 = H * rcta / a.routed_ctas, p1 = H * (rcta + 1) / a.routed_ctas;
    for (uint64_t i = warp; p1 > p0 && i <= n; i += kGUTWarps) {
        if (i == n) {
            prefetch_l2(a.sdown + p0 * a.sdown_rs, (uint32_t)((p1 - p0) * a.sdown_rs));
        } else {
            const uint32_t e = a.defer_topk ? s_routed[i].expert_id : a.routed[i].expert_id;
            if (e < a.experts) prefetch_l2(a.down[e] + p0 * a.down_rs, (uint32_t)((p1 - p0) * a.down_rs));
        }
    }
}

template <int T, bool kRouted>
__device__ __forceinline__ void gut_run(const MoeGateUpArgs& a, uint8_t* smem, uint32_t bar0, const lbk_routed* s_routed,
                                        uint32_t role_warp, uint32_t role_warps, bool dep_wait,
                                        const uint8_t* const* s_ptr) {
    // the down rows are requested once this warp's first rows are in
    bool down_pf = kRouted && a.down != nullptr;
    using RL = GUTRole<T>;
    using HB = typename HBOf<T>::type;
    constexpr bool kIq = RL::kIq;
    constexpr int kTail = RL::kTail;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nb_h, tpr = a.tpr_h, R = 32 / tpr;
    const int sub = lane / tpr, hb = lane % tpr, b = hb >> 1, h = hb & 1;
    const bool lane_on = hb < 2 * nb;
    const uint32_t rs = planar_row_bytes(RL::kBB, nb);  // R * rs == kMat for nb in {8, 16}
    const uint8_t* stage = smem + RL::kRingOff + warp * RL::kStage;
    const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage);
    float* prod = reinterpret_cast<float*>(smem + RL::kProdOff) + warp * RL::kProd;
    float* chains = reinterpret_cast<float*>(smem + RL::kChainOff) + warp * RL::kChain;
    float* res = reinterpret_cast<float*>(smem + RL::kResOff) + warp * RL::kRes;
    const uint32_t t0 = lane_addr(reinterpret_cast<const uint32_t*>(smem));
    const StageOff so = stage_off<T>(nb, sub, b, h);
    const int pstride = 2 * nb * kTail;  // prod[(ri*2 + m)*nb + b][kTail]

    const uint32_t ffn = (uint32_t)a.ffn;
    const uint32_t slots = kRouted ? (uint32_t)a.k : 1u;
    RoleWork wk{(uint32_t)a.tokens, (uint32_t)(kRouted ? a.chunk_r : a.chunk_s), (uint32_t)(kRouted ? a.chunks_r : a.chunks_s)};
    if (kRouted && a.d_items != nullptr) wk = device_work(a.d_items, a.tokens, slots, role_warps, ffn, R);
    const uint32_t chunk = wk.chunk, chunks = wk.chunks;
    const uint32_t items = wk.tokens * slots * chunks;
    uint32_t phase = 0;  // parity of the stage's next phase
    bool live = true;  // false after a wait ran out: no further copies are issued
    for (uint32_t it = role_warp; it < items; it += role_warps) {
        const uint32_t t = it / (slots * chunks);
        const uint32_t rem = it - t * (slots * chunks);
        const uint32_t j = rem / chunks, c = rem - j * chunks;
        const uint32_t slot = kRouted ? j : (uint32_t)a.k;
        const uint32_t r0 = c * chunk, r1 = r0 + chunk < ffn ? r0 + chunk : ffn;
        if (r0 >= r1) continue;
        const uint32_t units = 2 * ((r1 - r0 + R - 1) / R);
        ActHB act;
        uint32_t nact[32];
        auto load_act = [&]() {
            if (lane_on) {
                load_act_global<!kIq>(act, a.q8x + (uint64_t)t * nb * kQ8IBytes, b, h, !kIq);
                if constexpr (T == LBK_TYPE_IQ3_S) {
#pragma unroll
                    for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
                }
            }
        };
        // the activations do not depend on the expert: in flight while it is resolved
        if (!dep_wait) load_act();
        const uint8_t* gmat = a.sgate;
        const uint8_t* umat = a.sup;
        if constexpr (kRouted) {
            uint32_t e = a.defer_topk ? s_routed[j].expert_id : a.routed[(uint64_t)t * a.k + j].expert_id;
            if (e >= a.experts) {  // reported; compute on expert 0 so the arrival counts stay balanced
                if (lane == 0) report(a.status, LBK_INVALID_PARAMETER, e, 0);
                e = 0;
            }
            gmat = s_ptr ? s_ptr[e] : a.gate[e];
            umat = s_ptr ? s_ptr[kPtrMax + e] : a.up[e];
        }
        if (lane == 0 && live) {
            // the first step's rows go straight to the stage, ahead of any prefetch
            gut_issue2(stage_s, bar0, gmat, umat, rs, RL::kMat, r0, r1 - r0 < (uint32_t)R ? r1 - r0 : R);
            // the next two steps' rows head for L2 (later ones as the steps go)
            const uint32_t rp = r0 + R, rq = r0 + 3 * R < r1 ? r0 + 3 * R : r1;
            if (rp < rq) {
                prefetch_l2_stream(gmat + (uint64_t)rp * rs, (rq - rp) * rs, policy_evict_first());
                prefetch_l2_stream(umat + (uint64_t)rp * rs, (rq - rp) * rs, policy_evict_first());
            }
        }
        if (dep_wait) {
            grid_dep_wait();
            dep_wait = false;
            load_act();
        }
        float* hrow = a.h + ((uint64_t)t * (a.k + 1) + slot) * a.ffn;
        uint32_t rb = r0;
        // one rolled loop over row steps (R rows of gate and of up, one stage
        // and one barrier): the lane decodes its half block of both matrices,
        // two independent chains on the same activations, with no branch on
        // the lane (rows past the chunk's end decode stale stage bytes and are
        // not stored); the decode is emitted once (its code is fetched cold
        // once per launch)
        const uint32_t steps = units >> 1;
#pragma unroll 1
        for (uint32_t q = 0; q < steps; q++) {
            const uint32_t ra = r0 + q * R;
            const uint32_t nr = r1 - ra < (uint32_t)R ? r1 - ra : (uint32_t)R;
            if (live && !stage_wait(bar0, phase)) {
                live = false;
                report(a.status, LBK_TIMEOUT, it, 0);
            }
            phase ^= 1u;
            HB wg, wu;
            load_stage(wg, stage, so);
            load_stage(wu, stage + RL::kMat, so);
            __syncwarp();
            const uint32_t rn = ra + R;
            if (lane == 0 && live && q + 1 < steps) {
                fence_proxy_async_smem();
                gut_issue2(stage_s, bar0, gmat, umat, rs, RL::kMat, rn, r1 - rn < (uint32_t)R ? r1 - rn : R);
                // the rows three steps ahead head for L2: a few requests per
                // step, so that no copy waits behind a long queue
                const uint32_t rp = ra + 3 * R;
                if (rp < r1) {
                    const uint32_t np = r1 - rp < (uint32_t)R ? r1 - rp : R;
                    prefetch_l2_stream(gmat + (uint64_t)rp * rs, np * rs, policy_evict_first());
                    prefetch_l2_stream(umat + (uint64_t)rp * rs, np * rs, policy_evict_first());
                }
            }
            if (q == 1 && down_pf) {
                if (lane == 0) prefetch_down_rows(a, s_routed, blockIdx.x);
                down_pf = false;
            }
            const uint32_t row = ra + sub;
            IqPart ipg{0, 0}, ipu{0, 0};
            KPart kpg, kpu;
            HBDot<T>::run(wg, act, nact, t0, h, ipg, kpg);
            HBDot<T>::run(wu, act, nact, t0, h, ipu, kpu);
            const bool store = (uint32_t)sub < nr;
            float* pr = prod + (int)(row - rb) * pstride;
            write_products<T>(pr, b, h, store, ipg, kpg, act.d);
            write_products<T>(pr + nb * kTail, b, h, store, ipu, kpu, act.d);
            if (rn - rb >= (uint32_t)RL::kBmax || rn >= r1) {
                const int nrows = (int)((rn < r1 ? rn : r1) - rb);
                __syncwarp();
                warp_tails<T>(prod, nrows * 2, nb, chains, res);
                for (int qq = lane; qq < nrows; qq += 32) {
                    float g = res[qq * 2], u = res[qq * 2 + 1];
                    float v = swiglu_ref(g, u);
                    if (!isfinite(v))
                        report(a.status, LBK_NON_FINITE_VALUE, ((uint64_t)t * (a.k + 1) + slot) * a.ffn + rb + qq,
                               __float_as_uint(v));
                    hrow[rb + qq] = v;
                }
                __syncwarp();
                rb = rn;
            }
        }
        arrive_and_quantize(a, t, slot, r0, r1);
    }
    if (down_pf && (threadIdx.x & 31) == 0) prefetch_down_rows(a, s_routed, blockIdx.x);  // a warp without items
}

// A shared-expert role of an IQ type holds that type's lookup table too:
// a bulk copy into the start of shared memory, waited for by every thread.
template <int T, int kTab>
__device__ __forceinline__ void load_role_tables(const Tables& t, uint8_t* smem, uint64_t* bar_word, DeviceStatus* st) {
    if constexpr (kTab != 0) {
        const uint32_t bar = (uint32_t)__cvta_generic_to_shared(bar_word);
        if (threadIdx.x == 0) {
            mbar_init(bar, 1);
            mbar_init_fence();
            mbar_expect_tx(bar, (uint32_t)kTab);
            const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
            bulk_g2s(base, T == LBK_TYPE_IQ2_S ? (const void*)t.iq2_codes : (const void*)t.iq3_grid, kTab, bar);
        }
        __syncthreads();
        if (!mbar_wait(bar, 0) && threadIdx.x == 0) report(st, LBK_TIMEOUT, 5, 0);
    }
}

template <int TG, int TS>
__global__ void __launch_bounds__(kGUTThreads, 1) moe_gate_up_tma_kernel(MoeGateUpArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[kGUTWarps * 2];  // two stages per warp
    __shared__ lbk_routed s_routed[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&s_bar[2 * warp]);
    grid_dep_launch();  // the down kernel may start on SMs this grid leaves
    if (lane == 0) {
        mbar_init(bar, 1);
        mbar_init(bar + 8, 1);
        mbar_init_fence();
    }
    __syncwarp();
    if (blockIdx.x < a.routed_ctas) {
        using RL = GUTRole<TG>;
        // Prologue by bulk copies: (single-token decode) the router's chunk
        // partials, then the lookup tables, land in shared memory; the whole
        // CTA finishes the router from the partials (logits in chunk order,
        // then top-k) while the tables arrive. CTA 0 publishes the routing
        // for the down kernel.
        __shared__ __align__(8) uint64_t s_pro[3];  // [0] partials, [1] tables, [2] selection bias
        __shared__ uint32_t s_sel[32];
        __shared__ int s_bad;
        const uint32_t bar_p = (uint32_t)__cvta_generic_to_shared(&s_pro[0]);
        const uint32_t bar_t = (uint32_t)__cvta_generic_to_shared(&s_pro[1]);
        const uint32_t bar_b = (uint32_t)__cvta_generic_to_shared(&s_pro[2]);
        // free until the rows start: [partials][keys][p]
        float* s_part = reinterpret_cast<float*>(smem + RL::kProdOff);
        const uint64_t pfloats = a.experts * a.chunks;
        unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_part + ((pfloats + 3) & ~(uint64_t)3));
        float* s_p = reinterpret_cast<float*>(s_key + a.experts);
        float* s_bias = s_p + a.experts;  // staged with the tables (constant data)
        const bool bulk_p = a.defer_topk && pfloats % 4 == 0;
        const bool stage_bias = a.defer_topk && a.experts % 4 == 0 && ((uintptr_t)a.bias & 15) == 0 &&
                                ((uintptr_t)s_bias & 15) == 0;
        // the experts' gate / up pointers, staged with the tables (16-byte copies)
        __shared__ __align__(16) const uint8_t* s_ptr[2 * kPtrMax];
        const bool stage_ptr = a.experts <= kPtrMax && a.experts % 2 == 0;
        const uint32_t tab_tx = (uint32_t)RL::kTab + (stage_ptr ? 16u * (uint32_t)a.experts : 0);
        if (threadIdx.x == 0) {
            mbar_init(bar_p, 1);
            mbar_init(bar_t, 1);
            mbar_init(bar_b, 1);
            mbar_init_fence();
            // constant data first: this part overlaps the router kernel's tail
            if (tab_tx != 0) mbar_expect_tx(bar_t, tab_tx);
            if constexpr (RL::kTab != 0) {
                const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
                bulk_g2s(base, TG == LBK_TYPE_IQ2_S ? (const void*)a.tables.iq2_codes : (const void*)a.tables.iq3_grid,
                         RL::kTab, bar_t);
            }
            if (stage_ptr) {
                const uint32_t ps = (uint32_t)__cvta_generic_to_shared(s_ptr);
                bulk_g2s(ps, a.gate, 8u * (uint32_t)a.experts, bar_t);
                bulk_g2s(ps + 8 * kPtrMax, a.up, 8u * (uint32_t)a.experts, bar_t);
            }
            if (stage_bias) {
                mbar_expect_tx(bar_b, 4u * (uint32_t)a.experts);
                bulk_g2s((uint32_t)__cvta_generic_to_shared(s_bias), a.bias, 4u * (uint32_t)a.experts, bar_b);
            }
        }
        grid_dep_wait();  // the router's partials, Q8_K image and zeroed counters
        if (threadIdx.x == 0 && bulk_p) {
            mbar_expect_tx(bar_p, (uint32_t)(pfloats * 4));
            bulk_g2s((uint32_t)__cvta_generic_to_shared(s_part), a.partials, (uint32_t)(pfloats * 4), bar_p);
        }
        __syncthreads();
        if (a.defer_topk) {
            if (bulk_p) {
                if (!mbar_wait(bar_p, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 0, 0);
            } else {
                for (uint64_t i = threadIdx.x; i < pfloats; i += blockDim.x) s_part[i] = __ldcg(a.partials + i);
                __syncthreads();
            }
            if (stage_bias) {
                if (!mbar_wait(bar_b, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 2, 0);
            }
            topk_cta(s_part, (int)a.chunks, stage_bias ? s_bias : a.bias, (int)a.experts, (int)a.k, a.weight_scale,
                     s_routed, blockIdx.x == 0 ? a.status : nullptr, s_key, s_p, s_sel, &s_bad);
            if (blockIdx.x == 0 && threadIdx.x < a.k) a.routed_store[threadIdx.x] = s_routed[threadIdx.x];
            // The down kernel may read the routing before its grid wait:
            // publish it (every writer's store, then the flag).
            if (blockIdx.x == 0 && a.route_flag != nullptr) {
                __threadfence();
                __syncthreads();
                if (threadIdx.x == 0) st_release_gpu(a.route_flag, 1u);
            }
        }
        if (tab_tx != 0) {
            if (!mbar_wait(bar_t, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 1, 0);
        }
        gut_run<TG, true>(a, smem, bar, s_routed, blockIdx.x * kGUTWarps + warp, a.routed_ctas * kGUTWarps, false,
                          stage_ptr ? s_ptr : nullptr);
    } else {
        __shared__ __align__(8) uint64_t s_stab;
        load_role_tables<TS, GUTRole<TS>::kTab>(a.tables, smem, &s_stab, a.status);
        // shared expert: its first rows are constant data, requested before
        // the wait for the router's output (inside gut_run)
        gut_run<TS, false>(a, smem, bar, nullptr, (blockIdx.x - a.routed_ctas) * kGUTWarps + warp,
                           (gridDim.x - a.routed_ctas) * kGUTWarps, true, nullptr);
    }
}

// -------------------------------------------------------------------- down

template <int TD, int TSD>
struct DownSmem {
    static constexpr int kTabD = table_bytes<TD>();
    static constexpr int kTabS = (TSD == TD) ? 0 : table_bytes<TSD>();
    static constexpr int kFixed = kTabD + kTabS;
};

template <int T>
__device__ __forceinline__ void down_rows(const MoeDownArgs& a, uint64_t t, uint64_t slot, const uint8_t* dmat,
                                          int wsub, uint64_t r0, uint64_t r1, float* prod, float* chains, float* res,
                                          float* dots, const uint32_t* tab) {
    using HB = typename HBOf<T>::type;
    constexpr bool kIq = is_iq<T>();
    constexpr int kTail = TypeInfo<T>::kTail;
    const int lane = threadIdx.x & 31;
    const int nb = a.nb_f;
    const int tpr = a.tpr_f;
    const int rps = 32 / tpr;
    const int sub = lane / tpr, hb = lane % tpr;
    const int b = hb >> 1, h = hb & 1;
    const bool lane_on = hb < 2 * nb;
    const uint64_t sidx = t * (a.k + 1) + slot;

    ActHB act;
    uint32_t nact[32];
    if (lane_on) {
        load_act_global<!kIq>(act, a.hq + sidx * (uint64_t)nb * kQ8IBytes, b, h, !kIq);
        if constexpr (T == LBK_TYPE_IQ3_S) {
#pragma unroll
            for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
        }
    }
    const uint32_t t0 = lane_addr(tab);
    MatrixRef dm{dmat, a.hidden, nb};
    // this warp's rows: r0 + wsub*rps + i*wps*rps + sub, through a ring of D
    // prefetched steps in registers
    constexpr int D = RingDepth<T>::kDown;
    const uint64_t stride = (uint64_t)a.wps * rps;
    const uint64_t first = r0 + (uint64_t)wsub * rps;
    int nd = 0;
    HB buf[D];
#pragma unroll
    for (int i = 0; i < D; i++) {
        const uint64_t row = first + (uint64_t)i * stride + sub;
        if (lane_on && row < r1) load_hb<LBK_LAYOUT_PLANAR>(buf[i], dm, row, b, h);
    }
    for (uint64_t base = first; base < r1; base += (uint64_t)D * stride) {
#pragma unroll
        for (int i = 0; i < D; i++) {
            const uint64_t r = base + (uint64_t)i * stride;
            if (r >= r1) break;  // warp-uniform
            const uint64_t row = r + sub;
            const bool mine = lane_on && row < r1;
            const HB w = buf[i];
            const uint64_t nrow = row + (uint64_t)D * stride;
            if (lane_on && nrow < r1) load_hb<LBK_LAYOUT_PLANAR>(buf[i], dm, nrow, b, h);
            IqPart ip{0, 0};
            KPart kp;
#pragma unroll
            for (int l = 0; l < 8; l++) kp.lane[l] = 0;
            kp.min_sum = 0;
            kp.dm = 0;
            if (mine) HBDot<T>::run(w, act, nact, t0, h, ip, kp);
            float* pd = prod + (size_t)(nd + sub) * nb * kTail;
            write_products<T>(pd, b, h, mine, ip, kp, act.d);
            nd += rps;
        }
    }
    __syncwarp();
    warp_tails<T>(prod, nd, nb, chains, res);
    // scatter results to dots[slot][row - r0]
    for (int d = lane; d < nd; d += 32) {
        uint64_t row = r0 + (uint64_t)wsub * rps + (uint64_t)(d / rps) * stride + (d % rps);
        if (row < r1) dots[slot * a.rows_per_cta + (row - r0)] = res[d];
    }
}

template <int TD, int TSD>
__global__ void __launch_bounds__(kDownMaxThreads, 1) moe_down_kernel(MoeDownArgs a) {
    using S = DownSmem<TD, TSD>;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* tabD = reinterpret_cast<uint32_t*>(smem);
    uint32_t* tabS = S::kTabS ? reinterpret_cast<uint32_t*>(smem + S::kTabD) : tabD;
    float* dots = reinterpret_cast<float*>(smem + S::kFixed);
    float* prod_all = dots + (a.k + 1) * a.rows_per_cta;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    float* prod = prod_all + (size_t)warp * a.prod_floats;
    float* chains = prod_all + (size_t)nwarps * a.prod_floats + (size_t)warp * a.chain_floats;
    float* res = chains + a.chain_floats - 64;

    fill_tables<TD>(tabD, a.tables);
    if constexpr (S::kTabS != 0) fill_tables<TSD>(tabS, a.tables);
    __syncthreads();

    const uint64_t t = blockIdx.y;
    const uint64_t r0 = (uint64_t)blockIdx.x * a.rows_per_cta;
    const uint64_t r1 = r0 + a.rows_per_cta < a.hidden ? r0 + a.rows_per_cta : a.hidden;
    const uint64_t slot = warp / a.wps;
    const int wsub = warp % a.wps;
    if (slot < a.k) {
        uint32_t e = a.routed[t * a.k + slot].expert_id;
        if (e < a.experts) down_rows<TD>(a, t, slot, a.down[e], wsub, r0, r1, prod, chains, res, dots, tabD);
    } else if (slot == a.k) {
        down_rows<TSD>(a, t, slot, a.sdown, wsub, r0, r1, prod, chains, res, dots, tabS);
    }
    __syncthreads();
    if (status_set(a.status)) return;  // validation failed upstream: leave out unchanged
    for (uint64_t i = threadIdx.x; i < r1 - r0; i += blockDim.x) {
        float acc = 0.0f;
        for (uint64_t j = 0; j < a.k; j++) {
            float c = a.routed[t * a.k + j].coefficient;
            acc = __fadd_rn(acc, __fmul_rn(c, dots[j * a.rows_per_cta + i]));
        }
        acc = __fadd_rn(acc, __fmul_rn(1.0f, dots[a.k * a.rows_per_cta + i]));
        a.out[t * a.hidden + r0 + i] = acc;
    }
}

// ---------------------------------------------------- down, bulk-copy staged
//
// Items (token, slot, chunk of output rows) over two CTA roles as in the
// gate/up kernel: CTAs [0, routed_ctas) take the routed slots (and hold the
// routed type's tables), the others the shared expert. A unit is R rows of
// one down matrix (32 half blocks at most), streamed through the warp's two
// stages. Each warp writes its rows' dots to `dots` and arrives on the
// 64-row combine blocks it touched; the last arrival of a block forms
// out = 0; += c_j * dot_j (routed, ascending ID); += 1.0 * dot_shared
// (moe.rs:331-336) for those rows, unless validation failed upstream.

constexpr int kDNWarps = kMoeDownTmaWarps;
constexpr int kDNThreads = kDNWarps * 32;
constexpr int kDNBlock = kMoeDownCombineRows;

template <int T>
struct DNRole {
    static constexpr bool kIq = is_iq<T>();
    static constexpr int kBB = TypeInfo<T>::kBlockBytes;
    static constexpr int kUnit = 16 * kBB + 256;  // R rows of <= 16 blocks, each padded to 16 bytes
    static constexpr int kStage = 2 * kUnit;
    static constexpr int kBmax = T == LBK_TYPE_IQ3_S ? 16 : 8;  // rows per tail batch (IQ2_S: tables leave less room)
    static constexpr int kTail = TypeInfo<T>::kTail;
    static constexpr int kProd = kBmax * 16 * kTail;  // a batch holds <= 16 blocks of rows (R * nb <= 16)
    static constexpr int kChain = kIq ? 0 : 16 * 9;   // a batch has <= max(kBmax, R) <= 16 rows
    static constexpr int kRes = 32;
    static constexpr int kTab = table_bytes<T>();
    static constexpr int kRingOff = kTab;
    static constexpr int kProdOff = kRingOff + kDNWarps * kStage;
    static constexpr int kChainOff = kProdOff + kDNWarps * kProd * 4;
    static constexpr int kResOff = kChainOff + kDNWarps * kChain * 4;
    static constexpr int kBytes = kResOff + kDNWarps * kRes * 4;
};

constexpr int kCombineK = 8;  // routed slots the combine holds in registers

// Arrivals on the combine blocks of rows [r0, r1) of slot `slot`; the last
// arriving warp of a block combines its rows.
__device__ __forceinline__ void dn_arrive_and_combine(const MoeDownArgs& a, uint32_t t, uint32_t r0, uint32_t r1) {
    const int lane = threadIdx.x & 31;
    const uint32_t H = (uint32_t)a.hidden;
    const uint32_t nblk = (H + kDNBlock - 1) / kDNBlock;
    for (uint32_t blk = r0 / kDNBlock; blk * kDNBlock < r1; blk++) {
        const uint32_t lo = blk * kDNBlock > r0 ? blk * kDNBlock : r0;
        const uint32_t hi = (blk + 1) * kDNBlock < r1 ? (blk + 1) * kDNBlock : r1;
        const uint32_t bend = (blk + 1) * kDNBlock < H ? (blk + 1) * kDNBlock : H;
        const uint32_t target = (uint32_t)(a.k + 1) * (bend - blk * kDNBlock);
        unsigned int* cnt = a.counters + (uint64_t)t * nblk + blk;
        unsigned old = 0;
        __syncwarp();  // the lanes' dot stores before lane 0's release
        if (lane == 0) old = atom_add_acq_rel_gpu(cnt, hi - lo);
        old = __shfl_sync(0xffffffffu, old, 0);
        __syncwarp();  // lane 0's acquire before the lanes' reads below
        if (old + (hi - lo) != target) continue;
        if (lane == 0) *cnt = 0u;  // ready for the next launch
        if (status_set(a.status)) continue;  // validation failed upstream: leave out unchanged
        const float* dt = a.dots + (uint64_t)t * (a.k + 1) * H;
        if (a.k <= (uint64_t)kCombineK && kDNBlock == 64) {
            // every dot of the block's two rows per lane in flight at once,
            // the coefficients read once per warp
            const float cl = (uint64_t)lane < a.k ? a.routed[(uint64_t)t * a.k + lane].coefficient : 0.0f;
            const uint32_t ra = blk * kDNBlock + lane, rb = ra + 32;
            float va[kCombineK], vb[kCombineK];
#pragma unroll
            for (int j = 0; j < kCombineK; j++) {
                va[j] = (uint64_t)j < a.k && ra < bend ? __ldcg(dt + (uint64_t)j * H + ra) : 0.0f;
                vb[j] = (uint64_t)j < a.k && rb < bend ? __ldcg(dt + (uint64_t)j * H + rb) : 0.0f;
            }
            const float sa = ra < bend ? __ldcg(dt + a.k * H + ra) : 0.0f;
            const float sb = rb < bend ? __ldcg(dt + a.k * H + rb) : 0.0f;
            float acc_a = 0.0f, acc_b = 0.0f;
#pragma unroll
            for (int j = 0; j < kCombineK; j++) {
                const float c = __shfl_sync(0xffffffffu, cl, j);
                if ((uint64_t)j < a.k) {
                    acc_a = __fadd_rn(acc_a, __fmul_rn(c, va[j]));
                    acc_b = __fadd_rn(acc_b, __fmul_rn(c, vb[j]));
                }
            }
            if (ra < bend) a.out[(uint64_t)t * H + ra] = __fadd_rn(acc_a, __fmul_rn(1.0f, sa));
            if (rb < bend) a.out[(uint64_t)t * H + rb] = __fadd_rn(acc_b, __fmul_rn(1.0f, sb));
            continue;
        }
        for (uint32_t r = blk * kDNBlock + lane; r < bend; r += 32) {
            float acc = 0.0f;
            for (uint64_t j = 0; j < a.k; j++) {
                const float c = a.routed[(uint64_t)t * a.k + j].coefficient;
                acc = __fadd_rn(acc, __fmul_rn(c, __ldcg(dt + j * H + r)));
            }
            acc = __fadd_rn(acc, __fmul_rn(1.0f, __ldcg(dt + a.k * H + r)));
            a.out[(uint64_t)t * H + r] = acc;
        }
    }
}

template <int T, bool kRouted>
__device__ __forceinline__ void dn_run(const MoeDownArgs& a, uint8_t* smem, uint32_t bar0, uint32_t role_warp,
                                       uint32_t role_warps, bool dep_wait, const uint8_t* const* s_ptr) {
    using RL = DNRole<T>;
    using HB = typename HBOf<T>::type;
    constexpr bool kIq = RL::kIq;
    constexpr int kTail = RL::kTail;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nb_f, tpr = a.tpr_f, R = 32 / tpr;
    const int sub = lane / tpr, hb = lane % tpr, b = hb >> 1, h = hb & 1;
    const bool lane_on = hb < 2 * nb;
    // lanes past the last whole row of a unit (ffn 1536: 24 of 32 busy) decode
    // a copy of row 0's first half block and store nothing: no branch per lane
    const bool lane_ok = lane_on && sub < R;
    const uint32_t rs = planar_row_bytes(RL::kBB, nb);
    const uint8_t* stage = smem + RL::kRingOff + warp * RL::kStage;
    const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage);
    float* prod = reinterpret_cast<float*>(smem + RL::kProdOff) + warp * RL::kProd;
    float* chains = reinterpret_cast<float*>(smem + RL::kChainOff) + warp * RL::kChain;
    float* res = reinterpret_cast<float*>(smem + RL::kResOff) + warp * RL::kRes;
    const uint32_t t0 = lane_addr(reinterpret_cast<const uint32_t*>(smem));
    const StageOff so = stage_off<T>(nb, lane_ok ? sub : 0, lane_ok ? b : 0, lane_ok ? h : 0);

    const uint32_t H = (uint32_t)a.hidden;
    const uint32_t slots = kRouted ? (uint32_t)a.k : 1u;
    RoleWork wk{(uint32_t)a.tokens, (uint32_t)(kRouted ? a.chunk_r : a.chunk_s), (uint32_t)(kRouted ? a.chunks_r : a.chunks_s)};
    if (kRouted && a.d_items != nullptr) wk = device_work(a.d_items, a.tokens, slots, role_warps, H, R);
    const uint32_t chunk = wk.chunk, chunks = wk.chunks;
    const uint32_t items = wk.tokens * slots * chunks;
    uint32_t phase = 0;  // bit s: parity of stage s's next phase
    bool live = true;
    for (uint32_t it = role_warp; it < items; it += role_warps) {
        const uint32_t t = it / (slots * chunks);
        const uint32_t rem = it - t * (slots * chunks);
        const uint32_t j = rem / chunks, c = rem - j * chunks;
        const uint32_t slot = kRouted ? j : (uint32_t)a.k;
        const uint32_t r0 = c * chunk, r1 = r0 + chunk < H ? r0 + chunk : H;
        if (r0 >= r1) continue;
        const uint32_t units = (r1 - r0 + R - 1) / R;
        ActHB act;
        uint32_t nact[32];
        // the negated words wait for the loads: formed after the first copies are issued
        auto load_act = [&]() {
            if (lane_on) load_act_global<!kIq>(act, a.hq + ((uint64_t)t * (a.k + 1) + slot) * nb * kQ8IBytes, b, h, !kIq);
        };
        auto negate_act = [&]() {
            if constexpr (T == LBK_TYPE_IQ3_S) {
                if (lane_on) {
#pragma unroll
                    for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
                }
            }
        };
        // the activations do not depend on the expert: in flight while it is resolved
        if (!dep_wait) load_act();
        const uint8_t* mat = a.sdown;
        if constexpr (kRouted) {
            // through L2: may be read before the grid wait (see route_flag)
            uint32_t e = __ldcg(reinterpret_cast<const unsigned int*>(a.routed + (uint64_t)t * a.k + j));
            if (e >= a.experts) {  // reported; compute on expert 0 so the arrival counts stay balanced
                if (lane == 0) report(a.status, LBK_INVALID_PARAMETER, e, 0);
                e = 0;
            }
            mat = s_ptr ? s_ptr[e] : a.down[e];
        }
        if (lane == 0 && live) {
            // single-token calls: the gate/up kernel has put these rows in L2
            if (a.route_flag == nullptr) prefetch_l2_stream(mat + (uint64_t)r0 * rs, (r1 - r0) * rs, policy_evict_first());
            for (uint32_t u = 0; u < 2 && u < units; u++) {
                const uint32_t ra = r0 + u * R;
                gut_issue(stage_s + u * RL::kUnit, bar0 + 8 * u, mat, rs, ra, r1 - ra < (uint32_t)R ? r1 - ra : R);
            }
        }
        if (dep_wait) {
            grid_dep_wait();
            dep_wait = false;
            load_act();
        }
        negate_act();
        float* drow = a.ret_addr != nullptr
                          ? reinterpret_cast<float*>(a.ret_peers[a.ret_addr[t].x] + a.ret_off) + (uint64_t)a.ret_addr[t].y * H
                          : a.dots + ((uint64_t)t * a.dots_slots + slot) * H;
        uint32_t rb = r0;
#pragma unroll 1
        for (uint32_t u = 0; u < units; u++) {
            const uint32_t s = u & 1;
            const uint32_t ra = r0 + u * R;
            const uint32_t nr = r1 - ra < (uint32_t)R ? r1 - ra : (uint32_t)R;
            if (live && !stage_wait(bar0 + 8 * s, (phase >> s) & 1u)) {
                live = false;
                report(a.status, LBK_TIMEOUT, it, 1);
            }
            phase ^= 1u << s;
            HB w;
            load_stage(w, stage + s * RL::kUnit, so);
            __syncwarp();
            if (lane == 0 && live && u + 2 < units) {
                fence_proxy_async_smem();
                const uint32_t rn = ra + 2 * R;
                gut_issue(stage_s + s * RL::kUnit, bar0 + 8 * s, mat, rs, rn, r1 - rn < (uint32_t)R ? r1 - rn : R);
            }
            const uint32_t row = ra + sub;
            IqPart ip{0, 0};
            KPart kp;
            HBDot<T>::run(w, act, nact, t0, h, ip, kp);
            write_products<T>(prod + (int)(row - rb) * nb * kTail, b, h, lane_ok && (uint32_t)sub < nr, ip, kp, act.d);
            const uint32_t rn = ra + R;
            if (rn - rb >= (uint32_t)RL::kBmax || rn >= r1) {
                const int nrows = (int)((rn < r1 ? rn : r1) - rb);
                __syncwarp();
                warp_tails<T>(prod, nrows, nb, chains, res);
                if (lane < nrows) drow[rb + lane] = res[lane];
                __syncwarp();
                rb = rn;
            }
        }
        if (a.combine) dn_arrive_and_combine(a, t, r0, r1);
    }
    // rows returned in place (peer stores): visible system-wide before this
    // grid is seen complete by the launch that releases the done flags
    if (a.ret_addr != nullptr) __threadfence_system();
}

template <int TD, int TSD>
__global__ void __launch_bounds__(kDNThreads, 1) moe_down_tma_kernel(MoeDownArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[kDNWarps * 2];
    __shared__ __align__(8) uint64_t s_tab;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&s_bar[2 * warp]);
    const uint32_t bar_t = (uint32_t)__cvta_generic_to_shared(&s_tab);
    const bool routed_role = blockIdx.x < a.routed_ctas;
    if (lane == 0) {
        mbar_init(bar, 1);
        mbar_init(bar + 8, 1);
        if (threadIdx.x == 0) mbar_init(bar_t, 1);
        mbar_init_fence();
    }
    // constant data (tables, the experts' down pointers) before the wait for
    // the gate/up kernel: this part overlaps that kernel's tail
    __shared__ __align__(16) const uint8_t* s_ptr[kPtrMax];
    const bool stage_ptr = a.experts <= kPtrMax && a.experts % 2 == 0;
    const uint32_t tab_tx = (uint32_t)DNRole<TD>::kTab + (stage_ptr ? 8u * (uint32_t)a.experts : 0);
    if (routed_role && threadIdx.x == 0) {
        using RL = DNRole<TD>;
        if (tab_tx != 0) mbar_expect_tx(bar_t, tab_tx);
        if constexpr (RL::kTab != 0) {
            const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
            bulk_g2s(base, TD == LBK_TYPE_IQ2_S ? (const void*)a.tables.iq2_codes : (const void*)a.tables.iq3_grid,
                     RL::kTab, bar_t);
        }
        if (stage_ptr) bulk_g2s((uint32_t)__cvta_generic_to_shared(s_ptr), a.down, 8u * (uint32_t)a.experts, bar_t);
    }
    __syncthreads();
    if (routed_role) {
        // Single token: the routing is final long before the gate/up grid
        // ends. Once its flag is seen (bounded poll), the first down rows are
        // requested before the wait for that grid; h is read after it. A poll
        // that runs out is reported (the output is then left unwritten) and
        // the CTA goes on after the grid wait: no copy is in flight yet.
        __shared__ int s_early;
        if (threadIdx.x == 0) {
            int ok = 0;
            if (a.route_flag != nullptr) {
                for (uint32_t i = 0; i < a.route_polls && !ok; i++) ok = ld_acquire_gpu(a.route_flag) != 0u;
                if (!ok) report(a.status, LBK_TIMEOUT, 4, 0);
            }
            s_early = ok;
        }
        __syncthreads();
        const bool early = s_early != 0;
        if (!early) grid_dep_wait();  // the routing and h images of the gate/up kernel
        // The flag is cleared by the last routed CTA to have read it, so the
        // next call's down kernel (which may start before that call's router
        // has run) never sees this call's flag. A CTA that did not see the
        // flag has waited for the gate/up grid, so the flag was set before it
        // arrives here. The next call's router starts only after this grid
        // ends, which orders the clear before that call's gate/up and down.
        if (a.route_flag != nullptr && threadIdx.x == 0) {
            if (atomicAdd(a.route_readers, 1u) + 1u == a.routed_ctas) {
                *a.route_readers = 0u;
                atomicExch(a.route_flag, 0u);
            }
        }
        if (tab_tx != 0) {
            if (!mbar_wait(bar_t, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 3, 0);
        }
        dn_run<TD, true>(a, smem, bar, blockIdx.x * kDNWarps + warp, a.routed_ctas * kDNWarps, early,
                         stage_ptr ? s_ptr : nullptr);
    } else {
        __shared__ __align__(8) uint64_t s_stab;
        load_role_tables<TSD, DNRole<TSD>::kTab>(a.tables, smem, &s_stab, a.status);
        // shared expert: its first rows are constant data, requested before
        // the wait for the gate/up kernel's output (inside dn_run)
        dn_run<TSD, false>(a, smem, bar, (blockIdx.x - a.routed_ctas) * kDNWarps + warp,
                           (gridDim.x - a.routed_ctas) * kDNWarps, true, nullptr);
    }
}

// ------------------------------------------------------ grouped (T tokens)
//
// Calls of several tokens (multi-sequence decode, short prefill, the items an
// expert-parallel rank received). The routed (token, slot) pairs are grouped
// by expert (moe_group_kernel); a warp item is (group, chunk of rows). A
// lane's half-block position is fixed for the whole item, so the activation
// half block of every pair of the group is loaded once into registers; each
// weight half block is then decoded once and dotted with all of them. The
// integer block sums, f32 block products and per-row tails are those of the
// single-token kernels, so every (token, slot) result is bit-identical to
// theirs. The shared expert is grouped the same way over consecutive tokens.

constexpr int kGrpDots = 64;  // dots per tail batch at most

// Pairs per group with W warps per CTA: each pair's activation half block is
// 33 registers (IQ) or 41 (K-quants), out of 255 a thread at 8 warps, 170 at
// 12 and 128 at 16.
template <int T, int W>
constexpr int grp_max() {
    return is_iq<T>() ? (W <= 8 ? 4 : (W <= 12 ? 3 : 2)) : (W <= 8 ? 2 : 1);
}

// Shared-memory plan of one grouped CTA role streaming type T with kMats
// matrices per unit (gate + up: one stage of both; down: two stages of one).
template <int T, int kMats, int W>
struct GrpRole {
    static constexpr bool kIq = is_iq<T>();
    static constexpr int kBB = TypeInfo<T>::kBlockBytes;
    static constexpr int kUnit = 16 * kBB + (kMats == 1 ? 256 : 0);  // down rows are each padded to 16 bytes
    static constexpr int kStage = 2 * kUnit;
    static constexpr int kTail = TypeInfo<T>::kTail;
    static constexpr int kProd = kIq ? (W <= 8 ? 512 : 256) : (W <= 8 ? 1152 : 576);  // floats per warp
    static constexpr int kChain = kIq ? 0 : kGrpDots * 9;
    static constexpr int kRes = kGrpDots;
    static constexpr int kTab = table_bytes<T>();
    static constexpr int kRingOff = kTab;
    static constexpr int kProdOff = kRingOff + W * kStage;
    static constexpr int kChainOff = kProdOff + W * kProd * 4;
    static constexpr int kResOff = kChainOff + W * kChain * 4;
    static constexpr int kBytes = kResOff + W * kRes * 4;
    // one unit of the largest group always fits a tail batch (R * nb <= 16)
    static_assert(16 * kMats * grp_max<T, W>() * kTail <= kProd, "grouped product buffer");
    // dots of one unit: R * kMats * pairs, R <= 2 for gate/up (nb_h 8 or 16), R <= 16 for down
    static_assert((kMats == 2 ? 2 : 16) * kMats * grp_max<T, W>() <= kGrpDots, "grouped dot buffer");
};

// The dots of one half block against the pairs p < n of a group: IQ types
// decode each 32-weight group once for all pairs (dot_hb_multi); a K-quant
// half block is dotted per pair straight from its packed words (its decode is
// two masks per word).
template <int T, int G>
__device__ __forceinline__ void grp_dots(const typename HBOf<T>::type& w, const ActHB* act, uint32_t n, uint32_t t0,
                                         int h, IqPart* ip, KPart* kp) {
    if constexpr (is_iq<T>()) {
        int32_t tot[G];
        dot_hb_multi<G, 128>(w, ActReg{act}, n, t0, tot);
#pragma unroll
        for (int p = 0; p < G; p++) ip[p] = IqPart{tot[p], w.d};
    } else {
#pragma unroll
        for (int p = 0; p < G; p++)
            if ((uint32_t)p < n) kp[p] = dot_hb(w, act[p], h);
    }
    (void)t0;
    (void)h;
}

template <int G>
__device__ __forceinline__ void grp_zero(IqPart* ip, KPart* kp) {
#pragma unroll
    for (int p = 0; p < G; p++) {
        ip[p] = IqPart{0, 0};
#pragma unroll
        for (int l = 0; l < 8; l++) kp[p].lane[l] = 0;
        kp[p].min_sum = 0;
        kp[p].dm = 0;
    }
}

// The pairs of group gi: routed groups from the grouping kernel's table
// (expert, first pair, count), shared groups as runs of consecutive tokens.
// Returns the pair count; tp / sp receive each pair's token and slot.
template <int G, bool kRouted>
__device__ __forceinline__ uint32_t grp_pairs(const uint4* grp, const uint32_t* pairs, uint32_t gi, uint32_t gsize,
                                              uint64_t tokens, uint64_t k, uint32_t* tp, uint32_t* sp, uint32_t& expert,
                                              DeviceStatus* st) {
    uint32_t n;
    if constexpr (kRouted) {
        const uint4 g = __ldcg(grp + gi);
        expert = g.x;
        n = g.z;
        if (n > (uint32_t)G) {  // the host sizes groups for the kernel; never more pairs than registers
            if ((threadIdx.x & 31) == 0) report(st, LBK_INVALID_PARAMETER, gi, n);
            n = 0;
        }
#pragma unroll
        for (int p = 0; p < G; p++) {
            const uint32_t i = (uint32_t)p < n ? __ldcg(pairs + g.y + p) : 0u;
            tp[p] = (uint32_t)(i / k);
            sp[p] = (uint32_t)(i % k);
        }
    } else {
        const uint64_t t0 = (uint64_t)gi * gsize;
        n = (uint32_t)(tokens - t0 < gsize ? tokens - t0 : gsize);
#pragma unroll
        for (int p = 0; p < G; p++) {
            tp[p] = (uint32_t)t0 + p;
            sp[p] = (uint32_t)k;
        }
        (void)grp;
        (void)pairs;
        (void)st;
    }
    return n;
}

// Row chunking of a grouped role: the groups' rows spread over the role's
// warps in whole steps of R rows.
__device__ __forceinline__ uint32_t grp_chunk(uint32_t rows, uint32_t groups, uint32_t role_warps, uint32_t R) {
    uint32_t per = groups ? role_warps / groups : 1u;
    per = per < 1u ? 1u : per;
    const uint32_t c = (rows + per - 1) / per;
    return (c + R - 1) / R * R;
}

// Units per tail batch: whole units within the product and dot buffers.
template <int kProd, int kTail>
__device__ __forceinline__ uint32_t grp_units(uint32_t dots_per_unit, int nb) {
    uint32_t ub = (uint32_t)kProd / (dots_per_unit * (uint32_t)nb * (uint32_t)kTail);
    const uint32_t ud = (uint32_t)kGrpDots / dots_per_unit;
    return ub < ud ? ub : ud;  // >= 1 by GrpRole's static checks
}

template <int T, bool kRouted, int W>
__device__ __forceinline__ void gup_run(const MoeGateUpArgs& a, uint8_t* smem, uint32_t bar0, uint32_t role_warp,
                                        uint32_t role_warps, const uint8_t* const* s_ptr) {
    using RL = GrpRole<T, 2, W>;
    using HB = typename HBOf<T>::type;
    constexpr bool kIq = RL::kIq;
    constexpr int kTail = RL::kTail;
    constexpr int G = grp_max<T, W>();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nb_h, tpr = a.tpr_h, R = 32 / tpr;
    const int sub = lane / tpr, hb = lane % tpr, b = hb >> 1, h = hb & 1;
    const bool lane_on = hb < 2 * nb;
    const uint32_t rs = planar_row_bytes(RL::kBB, nb);  // R * rs == 16 * kBB for nb in {8, 16}
    const uint8_t* stage = smem + RL::kRingOff + warp * RL::kStage;
    const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage);
    float* prod = reinterpret_cast<float*>(smem + RL::kProdOff) + warp * RL::kProd;
    float* chains = reinterpret_cast<float*>(smem + RL::kChainOff) + warp * RL::kChain;
    float* res = reinterpret_cast<float*>(smem + RL::kResOff) + warp * RL::kRes;
    const uint32_t t0 = lane_addr(reinterpret_cast<const uint32_t*>(smem));
    const StageOff so = stage_off<T>(nb, sub, b, h);

    const uint32_t ffn = (uint32_t)a.ffn;
    const uint32_t gsize = kRouted ? a.gsize_r : a.gsize_s;
    const uint32_t groups = kRouted ? __ldcg(a.grp_n) : (uint32_t)((a.tokens + gsize - 1) / gsize);
    const uint32_t chunk = grp_chunk(ffn, groups, role_warps, (uint32_t)R);
    const uint32_t chunks = (ffn + chunk - 1) / chunk;
    const uint32_t items = groups * chunks;
    uint32_t phase = 0;  // bit m: parity of matrix m's barrier
    bool live = true;    // false after a wait ran out: no further copies are issued
    for (uint32_t it = role_warp; it < items; it += role_warps) {
        const uint32_t gi = it / chunks, c = it - gi * chunks;
        uint32_t tp[G], sp[G], e = 0;
        const uint32_t n = grp_pairs<G, kRouted>(a.grp, a.grp_pairs, gi, gsize, a.tokens, a.k, tp, sp, e, a.status);
        const uint32_t r0 = c * chunk, r1 = r0 + chunk < ffn ? r0 + chunk : ffn;
        if (r0 >= r1 || n == 0) continue;
        const uint8_t* gmat = a.sgate;
        const uint8_t* umat = a.sup;
        if constexpr (kRouted) {
            if (e >= a.experts) {  // reported by the grouping kernel, which maps such IDs to expert 0
                e = 0;
            }
            gmat = s_ptr ? s_ptr[e] : a.gate[e];
            umat = s_ptr ? s_ptr[kPtrMax + e] : a.up[e];
        }
        const uint32_t steps = (r1 - r0 + R - 1) / R;
        if (lane == 0 && live) {
            prefetch_l2_stream(gmat + (uint64_t)r0 * rs, (r1 - r0) * rs, policy_evict_first());
            prefetch_l2_stream(umat + (uint64_t)r0 * rs, (r1 - r0) * rs, policy_evict_first());
            const uint32_t nr0 = r1 - r0 < (uint32_t)R ? r1 - r0 : R;
            gut_issue(stage_s, bar0, gmat, rs, r0, nr0);
            gut_issue(stage_s + RL::kUnit, bar0 + 8, umat, rs, r0, nr0);
        }
        ActHB act[G];
#pragma unroll
        for (int p = 0; p < G; p++)
            if ((uint32_t)p < n && lane_on)
                load_act_global<!kIq>(act[p], a.q8x + (uint64_t)tp[p] * nb * kQ8IBytes, b, h, !kIq);
        const uint32_t ub = grp_units<RL::kProd, kTail>((uint32_t)R * 2u * n, nb);
        uint32_t rb = r0;
#pragma unroll 1
        for (uint32_t q = 0; q < steps; q++) {
            const uint32_t ra = r0 + q * R;
            const uint32_t nr = r1 - ra < (uint32_t)R ? r1 - ra : (uint32_t)R;
            if (live && (!mbar_wait(bar0, phase & 1u) || !mbar_wait(bar0 + 8, (phase >> 1) & 1u))) {
                live = false;
                if (lane == 0) report(a.status, LBK_TIMEOUT, it, 4);
            }
            live = __all_sync(0xffffffffu, live);
            phase ^= 3u;
            const bool mine = lane_on && (uint32_t)sub < nr;
            HB wg, wu;
            if (mine) {
                load_stage(wg, stage, so);
                load_stage(wu, stage + RL::kUnit, so);
            }
            __syncwarp();
            const uint32_t rn = ra + R;
            if (lane == 0 && live && q + 1 < steps) {
                fence_proxy_async_smem();
                const uint32_t nn = r1 - rn < (uint32_t)R ? r1 - rn : R;
                gut_issue(stage_s, bar0, gmat, rs, rn, nn);
                gut_issue(stage_s + RL::kUnit, bar0 + 8, umat, rs, rn, nn);
            }
            const uint32_t row = ra + sub;
            // dots of a batch: [row - rb][matrix][pair]
            float* pr = prod + (size_t)(row - rb) * 2u * n * nb * kTail;
#pragma unroll
            for (int m = 0; m < 2; m++) {
                IqPart ip[G];
                KPart kp[G];
                grp_zero<G>(ip, kp);
                if (mine) grp_dots<T, G>(m == 0 ? wg : wu, act, n, t0, h, ip, kp);
#pragma unroll
                for (int p = 0; p < G; p++)
                    if ((uint32_t)p < n)
                        write_products<T>(pr + ((size_t)m * n + p) * nb * kTail, b, h, mine, ip[p], kp[p], act[p].d);
            }
            if ((rn - rb) / (uint32_t)R >= ub || rn >= r1) {
                const uint32_t nrows = (rn < r1 ? rn : r1) - rb;
                __syncwarp();
                warp_tails<T>(prod, (int)(nrows * 2u * n), nb, chains, res);
#pragma unroll
                for (int p = 0; p < G; p++) {
                    if ((uint32_t)p < n) {
                        const uint64_t sidx = (uint64_t)tp[p] * (a.k + 1) + sp[p];
                        float* hrow = a.h + sidx * a.ffn;
                        for (uint32_t rr = lane; rr < nrows; rr += 32) {
                            const float g = res[(rr * 2u) * n + p], u = res[(rr * 2u + 1u) * n + p];
                            const float v = swiglu_ref(g, u);
                            if (!isfinite(v))
                                report(a.status, LBK_NON_FINITE_VALUE, sidx * a.ffn + rb + rr, __float_as_uint(v));
                            hrow[rb + rr] = v;
                        }
                    }
                }
                __syncwarp();
                rb = rn;
            }
        }
#pragma unroll
        for (int p = 0; p < G; p++)
            if ((uint32_t)p < n) arrive_and_quantize(a, tp[p], sp[p], r0, r1);
    }
}

template <int T, bool kRouted, int W>
__device__ __forceinline__ void gdn_run(const MoeDownArgs& a, uint8_t* smem, uint32_t bar0, uint32_t role_warp,
                                        uint32_t role_warps, const uint8_t* const* s_ptr) {
    using RL = GrpRole<T, 1, W>;
    using HB = typename HBOf<T>::type;
    constexpr bool kIq = RL::kIq;
    constexpr int kTail = RL::kTail;
    constexpr int G = grp_max<T, W>();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nb_f, tpr = a.tpr_f, R = 32 / tpr;
    const int sub = lane / tpr, hb = lane % tpr, b = hb >> 1, h = hb & 1;
    const bool lane_on = hb < 2 * nb;
    const uint32_t rs = planar_row_bytes(RL::kBB, nb);
    const uint8_t* stage = smem + RL::kRingOff + warp * RL::kStage;
    const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage);
    float* prod = reinterpret_cast<float*>(smem + RL::kProdOff) + warp * RL::kProd;
    float* chains = reinterpret_cast<float*>(smem + RL::kChainOff) + warp * RL::kChain;
    float* res = reinterpret_cast<float*>(smem + RL::kResOff) + warp * RL::kRes;
    const uint32_t t0 = lane_addr(reinterpret_cast<const uint32_t*>(smem));
    const StageOff so = stage_off<T>(nb, sub, b, h);

    const uint32_t H = (uint32_t)a.hidden;
    const uint32_t gsize = kRouted ? a.gsize_r : a.gsize_s;
    const uint32_t groups = kRouted ? __ldcg(a.grp_n) : (uint32_t)((a.tokens + gsize - 1) / gsize);
    const uint32_t chunk = grp_chunk(H, groups, role_warps, (uint32_t)R);
    const uint32_t chunks = (H + chunk - 1) / chunk;
    const uint32_t items = groups * chunks;
    uint32_t phase = 0;  // bit s: parity of stage s's barrier
    bool live = true;
    for (uint32_t it = role_warp; it < items; it += role_warps) {
        const uint32_t gi = it / chunks, c = it - gi * chunks;
        uint32_t tp[G], sp[G], e = 0;
        const uint32_t n = grp_pairs<G, kRouted>(a.grp, a.grp_pairs, gi, gsize, a.tokens, a.k, tp, sp, e, a.status);
        const uint32_t r0 = c * chunk, r1 = r0 + chunk < H ? r0 + chunk : H;
        if (r0 >= r1 || n == 0) continue;
        const uint8_t* mat = a.sdown;
        if constexpr (kRouted) {
            if (e >= a.experts) e = 0;  // reported by the grouping kernel
            mat = s_ptr ? s_ptr[e] : a.down[e];
        }
        const uint32_t units = (r1 - r0 + R - 1) / R;
        if (lane == 0 && live) {
            prefetch_l2_stream(mat + (uint64_t)r0 * rs, (r1 - r0) * rs, policy_evict_first());
            for (uint32_t u = 0; u < 2 && u < units; u++) {
                const uint32_t ra = r0 + u * R;
                gut_issue(stage_s + u * RL::kUnit, bar0 + 8 * u, mat, rs, ra, r1 - ra < (uint32_t)R ? r1 - ra : R);
            }
        }
        ActHB act[G];
#pragma unroll
        for (int p = 0; p < G; p++)
            if ((uint32_t)p < n && lane_on)
                load_act_global<!kIq>(act[p], a.hq + ((uint64_t)tp[p] * (a.k + 1) + sp[p]) * nb * kQ8IBytes, b, h, !kIq);
        const uint32_t ub = grp_units<RL::kProd, kTail>((uint32_t)R * n, nb);
        uint32_t rb = r0;
#pragma unroll 1
        for (uint32_t u = 0; u < units; u++) {
            const uint32_t s = u & 1;
            const uint32_t ra = r0 + u * R;
            const uint32_t nr = r1 - ra < (uint32_t)R ? r1 - ra : (uint32_t)R;
            if (live && !mbar_wait(bar0 + 8 * s, (phase >> s) & 1u)) {
                live = false;
                if (lane == 0) report(a.status, LBK_TIMEOUT, it, 5);
            }
            live = __all_sync(0xffffffffu, live);
            phase ^= 1u << s;
            const bool mine = lane_on && (uint32_t)sub < nr;
            HB w;
            if (mine) load_stage(w, stage + s * RL::kUnit, so);
            __syncwarp();
            if (lane == 0 && live && u + 2 < units) {
                fence_proxy_async_smem();
                const uint32_t rn = ra + 2 * R;
                gut_issue(stage_s + s * RL::kUnit, bar0 + 8 * s, mat, rs, rn, r1 - rn < (uint32_t)R ? r1 - rn : R);
            }
            const uint32_t row = ra + sub;
            float* pr = prod + (size_t)(row - rb) * n * nb * kTail;  // dots [row - rb][pair]
            IqPart ip[G];
            KPart kp[G];
            grp_zero<G>(ip, kp);
            if (mine) grp_dots<T, G>(w, act, n, t0, h, ip, kp);
#pragma unroll
            for (int p = 0; p < G; p++)
                if ((uint32_t)p < n)
                    write_products<T>(pr + (size_t)p * nb * kTail, b, h, mine, ip[p], kp[p], act[p].d);
            const uint32_t rn = ra + R;
            if ((rn - rb) / (uint32_t)R >= ub || rn >= r1) {
                const uint32_t nrows = (rn < r1 ? rn : r1) - rb;
                __syncwarp();
                warp_tails<T>(prod, (int)(nrows * n), nb, chains, res);
#pragma unroll
                for (int p = 0; p < G; p++) {
                    if ((uint32_t)p < n) {
                        float* drow = a.ret_addr != nullptr
                                          ? reinterpret_cast<float*>(a.ret_peers[a.ret_addr[tp[p]].x] + a.ret_off) +
                                                (uint64_t)a.ret_addr[tp[p]].y * H
                                          : a.dots + ((uint64_t)tp[p] * a.dots_slots + sp[p]) * H;
                        for (uint32_t rr = lane; rr < nrows; rr += 32) drow[rb + rr] = res[rr * n + p];
                    }
                }
                __syncwarp();
                rb = rn;
            }
        }
        if (a.combine) {
#pragma unroll
            for (int p = 0; p < G; p++)
                if ((uint32_t)p < n) dn_arrive_and_combine(a, tp[p], r0, r1);
        }
    }
    if (a.ret_addr != nullptr) __threadfence_system();  // rows returned in place (see dn_run)
}

// Lookup tables of a role's type into the start of shared memory.
template <int T>
__device__ __forceinline__ void issue_tables(uint32_t base, const Tables& t, uint32_t bar) {
    if constexpr (table_bytes<T>() != 0) {
        bulk_g2s(base, T == LBK_TYPE_IQ2_S ? (const void*)t.iq2_codes : (const void*)t.iq3_grid, table_bytes<T>(), bar);
    }
    (void)base;
    (void)t;
    (void)bar;
}

template <int T>
constexpr uint32_t tables_tx() {
    return (uint32_t)table_bytes<T>();
}

// Grouped gate/up: CTAs [0, routed_ctas) take the routed groups, the others
// the shared expert's token groups. Constant data (tables, the experts'
// pointers) is requested before the wait for the grouping kernel.
template <int TG, int TS, int W>
__global__ void __launch_bounds__(W * 32, 1) moe_gate_up_grp_kernel(MoeGateUpArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[W * 2];
    __shared__ __align__(8) uint64_t s_tab;
    __shared__ __align__(16) const uint8_t* s_ptr[2 * kPtrMax];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&s_bar[2 * warp]);
    const uint32_t bar_t = (uint32_t)__cvta_generic_to_shared(&s_tab);
    const bool routed_role = blockIdx.x < a.routed_ctas;
    grid_dep_launch();
    if (lane == 0) {
        mbar_init(bar, 1);
        mbar_init(bar + 8, 1);
        if (threadIdx.x == 0) mbar_init(bar_t, 1);
        mbar_init_fence();
    }
    const bool stage_ptr = routed_role && a.experts <= kPtrMax && a.experts % 2 == 0;
    const uint32_t tab_tx = (routed_role ? tables_tx<TG>() : tables_tx<TS>()) + (stage_ptr ? 16u * (uint32_t)a.experts : 0u);
    if (threadIdx.x == 0 && tab_tx != 0) {
        mbar_expect_tx(bar_t, tab_tx);
        const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
        if (routed_role) issue_tables<TG>(base, a.tables, bar_t);
        else issue_tables<TS>(base, a.tables, bar_t);
        if (stage_ptr) {
            const uint32_t ps = (uint32_t)__cvta_generic_to_shared(s_ptr);
            bulk_g2s(ps, a.gate, 8u * (uint32_t)a.experts, bar_t);
            bulk_g2s(ps + 8 * kPtrMax, a.up, 8u * (uint32_t)a.experts, bar_t);
        }
    }
    __syncthreads();
    grid_dep_wait();  // the groups, the tokens' Q8_K images, the zeroed counters
    if (tab_tx != 0) {
        if (!mbar_wait(bar_t, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 6, 0);
    }
    if (routed_role)
        gup_run<TG, true, W>(a, smem, bar, blockIdx.x * W + warp, a.routed_ctas * W,
                          stage_ptr ? s_ptr : nullptr);
    else
        gup_run<TS, false, W>(a, smem, bar, (blockIdx.x - a.routed_ctas) * W + warp, (gridDim.x - a.routed_ctas) * W,
                              nullptr);
}

template <int TD, int TSD, int W>
__global__ void __launch_bounds__(W * 32, 1) moe_down_grp_kernel(MoeDownArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[W * 2];
    __shared__ __align__(8) uint64_t s_tab;
    __shared__ __align__(16) const uint8_t* s_ptr[kPtrMax];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar = (uint32_t)__cvta_generic_to_shared(&s_bar[2 * warp]);
    const uint32_t bar_t = (uint32_t)__cvta_generic_to_shared(&s_tab);
    const bool routed_role = blockIdx.x < a.routed_ctas;
    if (lane == 0) {
        mbar_init(bar, 1);
        mbar_init(bar + 8, 1);
        if (threadIdx.x == 0) mbar_init(bar_t, 1);
        mbar_init_fence();
    }
    const bool stage_ptr = routed_role && a.experts <= kPtrMax && a.experts % 2 == 0;
    const uint32_t tab_tx = (routed_role ? tables_tx<TD>() : tables_tx<TSD>()) + (stage_ptr ? 8u * (uint32_t)a.experts : 0u);
    if (threadIdx.x == 0 && tab_tx != 0) {
        mbar_expect_tx(bar_t, tab_tx);
        const uint32_t base = (uint32_t)__cvta_generic_to_shared(smem);
        if (routed_role) issue_tables<TD>(base, a.tables, bar_t);
        else issue_tables<TSD>(base, a.tables, bar_t);
        if (stage_ptr) bulk_g2s((uint32_t)__cvta_generic_to_shared(s_ptr), a.down, 8u * (uint32_t)a.experts, bar_t);
    }
    __syncthreads();
    grid_dep_wait();  // the h images of the gate/up kernel
    if (tab_tx != 0) {
        if (!mbar_wait(bar_t, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 7, 0);
    }
    if (routed_role)
        gdn_run<TD, true, W>(a, smem, bar, blockIdx.x * W + warp, a.routed_ctas * W,
                          stage_ptr ? s_ptr : nullptr);
    else
        gdn_run<TSD, false, W>(a, smem, bar, (blockIdx.x - a.routed_ctas) * W + warp, (gridDim.x - a.routed_ctas) * W,
                               nullptr);
}

// Groups the routed pairs of a call by expert (one CTA, one thread per
// expert): pairs[] lists, expert by expert in ascending ID, the routed
// indices t*k + j in ascending order; groups[] cuts each expert's list into
// runs of at most gsize pairs. An ID outside the layer is reported and
// counted as expert 0 (the single-token kernels compute such a slot on
// expert 0 as well), so every pair is computed once.
constexpr int kGroupThreads = 1024;
constexpr int kGroupStage = 8192;  // pairs of a call at most (their expert IDs staged in shared memory)

// Number of equal 16-bit halves of v and e2 (0, 1 or 2).
__device__ __forceinline__ uint32_t halves_equal(uint32_t v, uint32_t e2) {
    const uint32_t t = v ^ e2;
    return __popc(~(((t & 0x7fff7fffu) + 0x7fff7fffu) | t | 0x7fff7fffu));
}

__global__ void __launch_bounds__(kGroupThreads) moe_group_kernel(MoeGroupArgs a) {
    __shared__ uint32_t s_cnt[kGroupThreads], s_off[kGroupThreads];
    __shared__ __align__(16) uint16_t s_id[kGroupStage];
    __shared__ uint32_t s_wsum[2][32];
    grid_dep_launch();
    const uint32_t tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t E = (uint32_t)a.experts;  // <= kGroupThreads (host-checked)
    uint64_t n = a.tokens * a.k;
    if (a.d_items != nullptr) {  // the items a gather counted (launched after it, with a memset between)
        const uint64_t c = __ldcg(a.d_items);
        n = c < n ? c : n;
    }
    s_cnt[tid] = 0u;
    __syncthreads();
    for (uint64_t i = tid; i < n; i += kGroupThreads) {
        uint32_t e = a.routed[i].expert_id;
        if (e >= E) {
            report(a.status, LBK_INVALID_PARAMETER, e, 0);
            e = 0;
        }
        atomicAdd(&s_cnt[e], 1u);
    }
    __syncthreads();
    // exclusive scans of the pair counts and of the group counts
    const uint32_t c = tid < E ? s_cnt[tid] : 0u;
    const uint32_t g = (c + a.gsize - 1) / a.gsize;
    uint32_t ic = c, ig = g;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t x = __shfl_up_sync(0xffffffffu, ic, d), y = __shfl_up_sync(0xffffffffu, ig, d);
        if (lane >= (uint32_t)d) {
            ic += x;
            ig += y;
        }
    }
    if (lane == 31) {
        s_wsum[0][wid] = ic;
        s_wsum[1][wid] = ig;
    }
    __syncthreads();
    if (wid == 0) {
        uint32_t v0 = s_wsum[0][lane], v1 = s_wsum[1][lane], i0 = v0, i1 = v1;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, i0, d), y = __shfl_up_sync(0xffffffffu, i1, d);
            if (lane >= (uint32_t)d) {
                i0 += x;
                i1 += y;
            }
        }
        s_wsum[0][lane] = i0 - v0;
        s_wsum[1][lane] = i1 - v1;
    }
    __syncthreads();
    const uint32_t off = ic - c + s_wsum[0][wid], goff = ig - g + s_wsum[1][wid];
    s_off[tid] = off;
    // Stable placement: pair i goes to slot off[e] + (pairs j < i of its
    // expert), counted over the staged IDs eight at a time.
    const uint32_t m = (uint32_t)n;  // <= kGroupStage (host-checked)
    const uint32_t m8 = (m + 7) & ~7u;
    for (uint32_t i = tid; i < m8; i += kGroupThreads) {
        uint32_t e = 0xffffu;
        if (i < m) {
            e = a.routed[i].expert_id;
            e = e < E ? e : 0u;
        }
        s_id[i] = (uint16_t)e;
    }
    __syncthreads();
    const uint4* id8 = reinterpret_cast<const uint4*>(s_id);
    for (uint32_t i = tid; i < m; i += kGroupThreads) {
        const uint32_t e = s_id[i], e2 = e | (e << 16);
        uint32_t r = 0;
        for (uint32_t j8 = 0; j8 < i / 8; j8++) {
            const uint4 v = id8[j8];
            r += halves_equal(v.x, e2) + halves_equal(v.y, e2) + halves_equal(v.z, e2) + halves_equal(v.w, e2);
        }
        for (uint32_t j = i & ~7u; j < i; j++) r += s_id[j] == e;
        a.pairs[s_off[e] + r] = i;
    }
    if (tid < E) {
        for (uint32_t q = 0; q < g; q++) {
            const uint32_t left = c - q * a.gsize;
            a.groups[goff + q] = make_uint4(tid, off + q * a.gsize, left < a.gsize ? left : a.gsize, 0u);
        }
    }
    if (tid == E - 1) *a.n = goff + g;
}

// ---------------------------------------------------------------- launchers

// Launch allowed to begin before the preceding kernel of the stream has
// finished (programmatic stream serialization): the kernel calls
// grid_dep_wait() before it reads that kernel's output.
template <class Args>
cudaError_t launch_dependent(void (*kernel)(Args), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                             const Args& a) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int TG, int TS>
cudaError_t launch_gu(const MoeGateUpArgs& a, cudaStream_t stream) {
    using S = GUSmem<TG, TS>;
    size_t smem = S::kFixed + (size_t)kGUWarps * (a.prod_floats + a.chain_floats) * 4;
    if (smem > kMaxSmem) return cudaErrorInvalidValue;
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(moe_gate_up_kernel<TG, TS>));
    if (e != cudaSuccess) return e;
    uint64_t items = a.tokens * a.k * a.chunks_r + a.tokens * a.chunks_s;
    uint64_t ctas = (items + kGUWarps - 1) / kGUWarps;
    moe_gate_up_kernel<TG, TS><<<(unsigned)ctas, kGUThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

template <int TG, int TS>
cudaError_t launch_gut(const MoeGateUpArgs& a, unsigned ctas, cudaStream_t stream) {
    constexpr int kA = GUTRole<TG>::kBytes, kB = GUTRole<TS>::kBytes;
    constexpr size_t smem = kA > kB ? kA : kB;
    static_assert(smem + 32 * sizeof(lbk_routed) + kGUTWarps * 16 + 2 * kPtrMax * 8 + 256 <= (size_t)kMaxSmem,
                  "gate/up stage plan");
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(moe_gate_up_tma_kernel<TG, TS>));
    if (e != cudaSuccess) return e;
    // every role with work has CTAs: routed when k > 0, shared when present
    if ((a.k > 0) != (a.routed_ctas > 0) || (a.has_shared != 0) != (a.routed_ctas < ctas)) return cudaErrorInvalidValue;
    return launch_dependent(moe_gate_up_tma_kernel<TG, TS>, ctas, kGUTThreads, smem, stream, a);
}

template <int TD, int TSD>
cudaError_t launch_down(const MoeDownArgs& a, cudaStream_t stream) {
    using S = DownSmem<TD, TSD>;
    int warps = (int)((a.k + 1) * a.wps);
    size_t smem = S::kFixed + (size_t)(a.k + 1) * a.rows_per_cta * 4 + (size_t)warps * (a.prod_floats + a.chain_floats) * 4;
    if (smem > kMaxSmem) return cudaErrorInvalidValue;
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(moe_down_kernel<TD, TSD>));
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((a.hidden + a.rows_per_cta - 1) / a.rows_per_cta), (unsigned)a.tokens);
    moe_down_kernel<TD, TSD><<<grid, warps * 32, smem, stream>>>(a);
    return cudaGetLastError();
}

__global__ void swiglu_kernel(const float* gate, const float* up, float* h, uint64_t n, DeviceStatus* st) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        float v = swiglu_ref(gate[i], up[i]);
        if (!isfinite(v)) report(st, LBK_NON_FINITE_VALUE, i, __float_as_uint(v));
        h[i] = v;
    }
}

// Expert-parallel combine on the home GPU: out = 0; += c_j * dot_j over the
// token's routed slots in ascending ID (the routing's order); += 1.0 * shared
// (moe.rs:331-336), unless validation failed upstream. With a control block,
// warp 0 of every CTA first waits (bounded) until every rank's dots of this
// step are in.
__global__ void ep_combine_kernel(const lbk_routed* routed, const float* routed_dots, const float* shared_dots,
                                  float* out, uint64_t tokens, uint64_t k, uint64_t H, DeviceStatus* st,
                                  const EpControl* ctl, uint32_t world, uint32_t polls) {
    if (ctl != nullptr) {
        __shared__ int s_ok;
        if (threadIdx.x < 32) {
            const uint32_t step = __ldcg(&ctl->step);
            bool ok = true;
            for (uint32_t r = threadIdx.x; r < world; r += 32) {
                uint32_t i = 0;
                while ((int32_t)(ld_acquire_sys(&ctl->done[r]) - step) < 0 && ++i < polls) {
                    if ((i & 255u) == 0u && status_set(st)) i = polls;  // an error is recorded already
                    __nanosleep(64);
                }
                ok &= i < polls;
            }
            ok = __all_sync(0xffffffffu, ok);
            if (threadIdx.x == 0) {
                s_ok = ok;
                if (!ok) report(st, LBK_TIMEOUT, 9, step);
            }
        }
        __syncthreads();  // the flags' acquire before every thread's reads of the dots
        if (!s_ok) return;
    }
    if (status_set(st)) return;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tokens * H; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t t = i / H, r = i % H;
        float acc = 0.0f;
        for (uint64_t j = 0; j < k; j++)
            acc = __fadd_rn(acc, __fmul_rn(routed[t * k + j].coefficient, __ldcg(routed_dots + (t * k + j) * H + r)));
        out[i] = __fadd_rn(acc, __fmul_rn(1.0f, shared_dots[i]));
    }
}

}  // namespace

cudaError_t launch_ep_combine(const lbk_routed* routed, const float* routed_dots, const float* shared_dots, float* out,
                              uint64_t tokens, uint64_t k, uint64_t H, DeviceStatus* status, cudaStream_t stream) {
    uint64_t grid = (tokens * H + 255) / 256;
    if (grid > 4096) grid = 4096;
    if (grid < 1) grid = 1;
    ep_combine_kernel<<<(unsigned)grid, 256, 0, stream>>>(routed, routed_dots, shared_dots, out, tokens, k, H, status,
                                                          nullptr, 0, 0);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine_wait(const EpControl* ctl, uint32_t world, uint32_t polls, const lbk_routed* routed,
                                   const float* routed_dots, const float* shared_dots, float* out, uint64_t tokens,
                                   uint64_t k, uint64_t H, DeviceStatus* status, cudaStream_t stream) {
    uint64_t grid = (tokens * H + 255) / 256;
    if (grid > 1024) grid = 1024;
    if (grid < 1) grid = 1;  // a rank without tokens still waits: its buffer is then free for the next step
    ep_combine_kernel<<<(unsigned)grid, 256, 0, stream>>>(routed, routed_dots, shared_dots, out, tokens, k, H, status,
                                                          ctl, world, polls);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(const float* gate, const float* up, float* h, uint64_t n, DeviceStatus* status,
                          cudaStream_t stream) {
    uint64_t grid = (n + 255) / 256;
    if (grid > 4096) grid = 4096;
    if (grid < 1) grid = 1;
    swiglu_kernel<<<(unsigned)grid, 256, 0, stream>>>(gate, up, h, n, status);
    return cudaGetLastError();
}

bool moe_fused_supported(int gate_type, int shared_gate_type, int down_type, int shared_down_type) {
    bool gu = (gate_type == LBK_TYPE_IQ2_S || gate_type == LBK_TYPE_Q4_K) && shared_gate_type == LBK_TYPE_Q4_K;
    bool dn = (down_type == LBK_TYPE_IQ3_S || down_type == LBK_TYPE_IQ2_S || down_type == LBK_TYPE_Q4_K) &&
              shared_down_type == LBK_TYPE_Q4_K;
    return gu && dn;
}

size_t moe_gate_up_fixed_smem(int gate_type, int shared_gate_type) {
    if (gate_type == LBK_TYPE_IQ2_S && shared_gate_type == LBK_TYPE_Q4_K) return GUSmem<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>::kFixed;
    return GUSmem<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>::kFixed;
}

size_t moe_down_fixed_smem(int down_type, int shared_down_type) {
    (void)shared_down_type;
    if (down_type == LBK_TYPE_IQ3_S) return DownSmem<LBK_TYPE_IQ3_S, LBK_TYPE_Q4_K>::kFixed;
    if (down_type == LBK_TYPE_IQ2_S) return DownSmem<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>::kFixed;
    return DownSmem<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>::kFixed;
}

cudaError_t launch_moe_gate_up(int gate_type, int shared_gate_type, const MoeGateUpArgs& a, cudaStream_t stream) {
    (void)shared_gate_type;
    if (gate_type == LBK_TYPE_IQ2_S) return launch_gu<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>(a, stream);
    return launch_gu<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>(a, stream);
}

bool moe_gate_up_tma_supported(int gate_type, int shared_gate_type, int nb_h) {
    // the config-3 combinations and the checkpoint's (routed and shared IQ2_S)
    const bool types = ((gate_type == LBK_TYPE_IQ2_S || gate_type == LBK_TYPE_Q4_K) && shared_gate_type == LBK_TYPE_Q4_K) ||
                       (gate_type == LBK_TYPE_IQ2_S && shared_gate_type == LBK_TYPE_IQ2_S);
    return types && (nb_h == 8 || nb_h == 16);
}

bool moe_gate_up_tma_defer_fits(int gate_type, uint64_t experts, uint64_t chunks) {
    const uint64_t floats = gate_type == LBK_TYPE_IQ2_S ? (uint64_t)kGUTWarps * GUTRole<LBK_TYPE_IQ2_S>::kProd
                                                        : (uint64_t)kGUTWarps * GUTRole<LBK_TYPE_Q4_K>::kProd;
    return ((experts * chunks + 3) & ~(uint64_t)3) + 4 * experts <= floats;  // partials, 64-bit keys, p, bias
}

cudaError_t launch_moe_gate_up_tma(int gate_type, int shared_gate_type, const MoeGateUpArgs& a, unsigned ctas,
                                   cudaStream_t stream) {
    (void)shared_gate_type;
    if (gate_type == LBK_TYPE_IQ2_S && shared_gate_type == LBK_TYPE_IQ2_S)
        return launch_gut<LBK_TYPE_IQ2_S, LBK_TYPE_IQ2_S>(a, ctas, stream);
    if (gate_type == LBK_TYPE_IQ2_S) return launch_gut<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>(a, ctas, stream);
    return launch_gut<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>(a, ctas, stream);
}

template <int TD, int TSD>
cudaError_t launch_dnt(const MoeDownArgs& a, unsigned ctas, cudaStream_t stream) {
    constexpr int kA = DNRole<TD>::kBytes, kB = DNRole<TSD>::kBytes;
    constexpr size_t smem = kA > kB ? kA : kB;
    static_assert(smem + kDNWarps * 16 + 8 <= (size_t)kMaxSmem, "down stage plan");
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(moe_down_tma_kernel<TD, TSD>));
    if (e != cudaSuccess) return e;
    if ((a.k > 0) != (a.routed_ctas > 0) || (a.has_shared != 0) != (a.routed_ctas < ctas)) return cudaErrorInvalidValue;
    if (a.combine && !a.has_shared) return cudaErrorInvalidValue;
    return launch_dependent(moe_down_tma_kernel<TD, TSD>, ctas, kDNThreads, smem, stream, a);
}

bool moe_down_tma_supported(int down_type, int shared_down_type, int nb_f) {
    // the config-3 combinations (shared Q4_K) and the checkpoint's: routed
    // IQ3_S with shared IQ3_S or IQ2_S, routed IQ2_S with shared IQ2_S
    const bool q4 = (down_type == LBK_TYPE_IQ3_S || down_type == LBK_TYPE_IQ2_S || down_type == LBK_TYPE_Q4_K) &&
                    shared_down_type == LBK_TYPE_Q4_K;
    const bool iq = (down_type == LBK_TYPE_IQ3_S && (shared_down_type == LBK_TYPE_IQ3_S || shared_down_type == LBK_TYPE_IQ2_S)) ||
                    (down_type == LBK_TYPE_IQ2_S && shared_down_type == LBK_TYPE_IQ2_S);
    return (q4 || iq) && nb_f >= 1 && nb_f <= 16;
}

cudaError_t launch_moe_down_tma(int down_type, int shared_down_type, const MoeDownArgs& a, unsigned ctas,
                                cudaStream_t stream) {
    if (down_type == LBK_TYPE_IQ3_S && shared_down_type == LBK_TYPE_IQ3_S)
        return launch_dnt<LBK_TYPE_IQ3_S, LBK_TYPE_IQ3_S>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ3_S && shared_down_type == LBK_TYPE_IQ2_S)
        return launch_dnt<LBK_TYPE_IQ3_S, LBK_TYPE_IQ2_S>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ2_S && shared_down_type == LBK_TYPE_IQ2_S)
        return launch_dnt<LBK_TYPE_IQ2_S, LBK_TYPE_IQ2_S>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ3_S) return launch_dnt<LBK_TYPE_IQ3_S, LBK_TYPE_Q4_K>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ2_S) return launch_dnt<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>(a, ctas, stream);
    return launch_dnt<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>(a, ctas, stream);
}

cudaError_t launch_moe_down(int down_type, int shared_down_type, const MoeDownArgs& a, cudaStream_t stream) {
    (void)shared_down_type;
    if (down_type == LBK_TYPE_IQ3_S) return launch_down<LBK_TYPE_IQ3_S, LBK_TYPE_Q4_K>(a, stream);
    if (down_type == LBK_TYPE_IQ2_S) return launch_down<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>(a, stream);
    return launch_down<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>(a, stream);
}

namespace {

// Warps per CTA of a grouped kernel: the most of LBK_GRP_WARPS, 12 and 8
// whose shared-memory plan fits (both roles' plans plus the static arrays).
#ifndef LBK_GRP_WARPS
#define LBK_GRP_WARPS 16
#endif

template <int TA, int TB, int kMats, int W>
constexpr size_t grp_smem() {
    return (size_t)(GrpRole<TA, kMats, W>::kBytes > GrpRole<TB, kMats, W>::kBytes ? GrpRole<TA, kMats, W>::kBytes
                                                                                  : GrpRole<TB, kMats, W>::kBytes);
}
template <int TA, int TB, int kMats, int W>
constexpr bool grp_fits() {
    return grp_smem<TA, TB, kMats, W>() + (size_t)W * 16 + 16 + (size_t)kMats * kPtrMax * 8 <= (size_t)kMaxSmem;
}
template <int TA, int TB, int kMats>
constexpr int grp_warps() {
    return grp_fits<TA, TB, kMats, LBK_GRP_WARPS>() ? LBK_GRP_WARPS : (grp_fits<TA, TB, kMats, 12>() ? 12 : 8);
}

template <int TG, int TS>
cudaError_t launch_gup(const MoeGateUpArgs& a, unsigned ctas, cudaStream_t stream) {
    constexpr int W = grp_warps<TG, TS, 2>();
    static_assert(grp_fits<TG, TS, 2, W>(), "grouped gate/up stage plan");
    constexpr size_t smem = grp_smem<TG, TS, 2, W>();
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(moe_gate_up_grp_kernel<TG, TS, W>));
    if (e != cudaSuccess) return e;
    if ((a.k > 0) != (a.routed_ctas > 0) || (a.has_shared != 0) != (a.routed_ctas < ctas)) return cudaErrorInvalidValue;
    if (a.k > 0 && (a.gsize_r < 1 || a.gsize_r > (uint32_t)grp_max<TG, W>())) return cudaErrorInvalidValue;
    if (a.has_shared && (a.gsize_s < 1 || a.gsize_s > (uint32_t)grp_max<TS, W>())) return cudaErrorInvalidValue;
    return launch_dependent(moe_gate_up_grp_kernel<TG, TS, W>, ctas, W * 32, smem, stream, a);
}

template <int TD, int TSD>
cudaError_t launch_gdn(const MoeDownArgs& a, unsigned ctas, cudaStream_t stream) {
    constexpr int W = grp_warps<TD, TSD, 1>();
    static_assert(grp_fits<TD, TSD, 1, W>(), "grouped down stage plan");
    constexpr size_t smem = grp_smem<TD, TSD, 1, W>();
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(moe_down_grp_kernel<TD, TSD, W>));
    if (e != cudaSuccess) return e;
    if ((a.k > 0) != (a.routed_ctas > 0) || (a.has_shared != 0) != (a.routed_ctas < ctas)) return cudaErrorInvalidValue;
    if (a.combine && !a.has_shared) return cudaErrorInvalidValue;
    if (a.k > 0 && (a.gsize_r < 1 || a.gsize_r > (uint32_t)grp_max<TD, W>())) return cudaErrorInvalidValue;
    if (a.has_shared && (a.gsize_s < 1 || a.gsize_s > (uint32_t)grp_max<TSD, W>())) return cudaErrorInvalidValue;
    return launch_dependent(moe_down_grp_kernel<TD, TSD, W>, ctas, W * 32, smem, stream, a);
}

// Group sizes and warps of one kernel's type pair: {routed pairs, shared pairs, warps}.
template <int TA, int TB, int kMats>
GrpShape grp_shape() {
    constexpr int W = grp_warps<TA, TB, kMats>();
    return GrpShape{(uint32_t)grp_max<TA, W>(), (uint32_t)grp_max<TB, W>(), (uint32_t)W};
}

}  // namespace

GrpShape moe_gate_up_grp_shape(int gate_type, int shared_gate_type) {
    if (gate_type == LBK_TYPE_IQ2_S && shared_gate_type == LBK_TYPE_IQ2_S)
        return grp_shape<LBK_TYPE_IQ2_S, LBK_TYPE_IQ2_S, 2>();
    if (gate_type == LBK_TYPE_IQ2_S) return grp_shape<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K, 2>();
    return grp_shape<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K, 2>();
}

GrpShape moe_down_grp_shape(int down_type, int shared_down_type) {
    if (down_type == LBK_TYPE_IQ3_S && shared_down_type == LBK_TYPE_IQ3_S)
        return grp_shape<LBK_TYPE_IQ3_S, LBK_TYPE_IQ3_S, 1>();
    if (down_type == LBK_TYPE_IQ3_S && shared_down_type == LBK_TYPE_IQ2_S)
        return grp_shape<LBK_TYPE_IQ3_S, LBK_TYPE_IQ2_S, 1>();
    if (down_type == LBK_TYPE_IQ2_S && shared_down_type == LBK_TYPE_IQ2_S)
        return grp_shape<LBK_TYPE_IQ2_S, LBK_TYPE_IQ2_S, 1>();
    if (down_type == LBK_TYPE_IQ3_S) return grp_shape<LBK_TYPE_IQ3_S, LBK_TYPE_Q4_K, 1>();
    if (down_type == LBK_TYPE_IQ2_S) return grp_shape<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K, 1>();
    return grp_shape<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K, 1>();
}

bool moe_grouped_supported(int gate_type, int shared_gate_type, int down_type, int shared_down_type, int nb_h, int nb_f) {
    return moe_gate_up_tma_supported(gate_type, shared_gate_type, nb_h) &&
           moe_down_tma_supported(down_type, shared_down_type, nb_f);
}

cudaError_t launch_moe_group(const MoeGroupArgs& a, cudaStream_t stream) {
    if (a.experts < 1 || a.experts > (uint64_t)kGroupThreads || a.gsize < 1 || a.tokens * a.k > (uint64_t)kGroupStage)
        return cudaErrorInvalidValue;
    moe_group_kernel<<<1, kGroupThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_moe_gate_up_grp(int gate_type, int shared_gate_type, const MoeGateUpArgs& a, unsigned ctas,
                                   cudaStream_t stream) {
    if (gate_type == LBK_TYPE_IQ2_S && shared_gate_type == LBK_TYPE_IQ2_S)
        return launch_gup<LBK_TYPE_IQ2_S, LBK_TYPE_IQ2_S>(a, ctas, stream);
    if (gate_type == LBK_TYPE_IQ2_S) return launch_gup<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>(a, ctas, stream);
    return launch_gup<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>(a, ctas, stream);
}

cudaError_t launch_moe_down_grp(int down_type, int shared_down_type, const MoeDownArgs& a, unsigned ctas,
                                cudaStream_t stream) {
    if (down_type == LBK_TYPE_IQ3_S && shared_down_type == LBK_TYPE_IQ3_S)
        return launch_gdn<LBK_TYPE_IQ3_S, LBK_TYPE_IQ3_S>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ3_S && shared_down_type == LBK_TYPE_IQ2_S)
        return launch_gdn<LBK_TYPE_IQ3_S, LBK_TYPE_IQ2_S>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ2_S && shared_down_type == LBK_TYPE_IQ2_S)
        return launch_gdn<LBK_TYPE_IQ2_S, LBK_TYPE_IQ2_S>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ3_S) return launch_gdn<LBK_TYPE_IQ3_S, LBK_TYPE_Q4_K>(a, ctas, stream);
    if (down_type == LBK_TYPE_IQ2_S) return launch_gdn<LBK_TYPE_IQ2_S, LBK_TYPE_Q4_K>(a, ctas, stream);
    return launch_gdn<LBK_TYPE_Q4_K, LBK_TYPE_Q4_K>(a, ctas, stream);
}


}  // namespace lbk
