// gemv.cu -- packed-row GEMV / dot kernels (IQ2_S, IQ3_S, Q4_K, Q5_K) x Q8_K.
//
// Replaces gemv_into / gemv_cpu_parallel_q8k_into / gemv_accumulate_scaled_into
// (bridge-kernels-reference/src/gemv.rs:56-70, :88-115, :117-174) and
// vec_dot_q8_k (bridge-quant-layout/src/q8_k.rs:80-119), bit-identical.
//
// One kernel per call: every CTA quantizes x to Q8_K itself (x is small and
// L2-resident), so a non-finite x is seen by every CTA and no output is
// written -- the reference's validate-before-write atomicity without a
// second launch. Each thread owns one half block (128 lanes) of the input
// and streams that half block of its rows; the per-block f32 products go to a
// per-warp shared buffer and one lane per row replays the sequential tail.

#include "lbk_kernels.h"

namespace lbk {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

template <int T>
struct GemvCfg {
    static constexpr bool kIq = (T == LBK_TYPE_IQ2_S || T == LBK_TYPE_IQ3_S);
    static constexpr int kTail = TypeInfo<T>::kTail;
    static constexpr int kTableBytes =
        T == LBK_TYPE_IQ2_S ? kIq2CodeBytes : (T == LBK_TYPE_IQ3_S ? kIq3GridBytes : 0);
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

// Shared memory: [tables][act qs K][act d nb][bsums nb*16][tail kWarps*slots*nb*kTail][flag]
template <int T>
__host__ __device__ inline size_t gemv_smem_bytes(int nb, int slots) {
    size_t s = (size_t)GemvCfg<T>::kTableBytes;
    s += (size_t)nb * kQK;                 // qs
    s += (size_t)nb * 4;                   // d
    s += (size_t)nb * 16 * 2;              // bsums
    s = (s + 15) & ~(size_t)15;
    s += (size_t)kWarps * slots * nb * GemvCfg<T>::kTail * 4;
    s += 16;
    return s;
}

// Quantizes x (or parses a given Q8_K row) into the CTA's activation image.
// Returns false if the input failed validation (reported to the status word).
__device__ bool stage_activations(const GemvArgs& a, int nb, int8_t* qs, float* dsm, int16_t* bs, int* flag) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) *flag = 0;
    __syncthreads();
    for (int b = warp; b < nb; b += kWarps) {
        if (a.q8_in != nullptr) {
            const uint8_t* src = a.q8_in + (size_t)b * kQ8Bytes;
            // qs at +4: 4-byte aligned words
            const uint32_t* qw = reinterpret_cast<const uint32_t*>(src + 4);
            uint32_t* dst = reinterpret_cast<uint32_t*>(qs + b * kQK);
            dst[lane * 2] = __ldg(qw + lane * 2);
            dst[lane * 2 + 1] = __ldg(qw + lane * 2 + 1);
            if (lane < 16) bs[b * 16 + lane] = (int16_t)ldg_u16(src + 260 + 2 * lane);
            if (lane == 0) {
                float d = __uint_as_float(__ldg(reinterpret_cast<const unsigned int*>(src)));
                dsm[b] = d;
                if (!isfinite(d)) {
                    report(a.status, LBK_NON_FINITE_Q8_SCALE, (uint64_t)b, __float_as_uint(d));
                    atomicExch(flag, 1);
                }
            }
            continue;
        }
        float v[8];
        const float4* xp = reinterpret_cast<const float4*>(a.x + (size_t)b * kQK + lane * 8);
        float4 p0 = __ldg(xp), p1 = __ldg(xp + 1);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
        v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
        bool bad = false;
        int bad_i = 0;
#pragma unroll
        for (int i = 7; i >= 0; i--)
            if (!isfinite(v[i])) {
                bad = true;
                bad_i = i;
            }
        unsigned badmask = __ballot_sync(0xffffffffu, bad);
        if (badmask) {
            int first_lane = __ffs(badmask) - 1;
            if (lane == first_lane)
                report(a.status, LBK_NON_FINITE_ACTIVATION, (uint64_t)b * kQK + lane * 8 + bad_i,
                       __float_as_uint(v[bad_i]));
            if (lane == 0) atomicExch(flag, 1);
            continue;
        }
        Q8Block q = quantize_q8k_warp(v, lane);
        uint32_t* dst = reinterpret_cast<uint32_t*>(qs + b * kQK);
        dst[lane * 2] = q.q[0];
        dst[lane * 2 + 1] = q.q[1];
        int32_t pair = q.pair_sum + __shfl_xor_sync(0xffffffffu, q.pair_sum, 1);
        if ((lane & 1) == 0) bs[b * 16 + (lane >> 1)] = (int16_t)pair;
        if (lane == 0) dsm[b] = q.d;
        if (a.q8_out != nullptr && blockIdx.x == 0) {
            uint8_t* o = a.q8_out + (size_t)b * kQ8Bytes;
            uint32_t* ow = reinterpret_cast<uint32_t*>(o + 4);
            ow[lane * 2] = q.q[0];
            ow[lane * 2 + 1] = q.q[1];
            if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(o + 260 + lane) = (int16_t)pair;
            if (lane == 0) *reinterpret_cast<float*>(o) = q.d;
        }
    }
    __syncthreads();
    bool ok = (*flag == 0);
    // The accumulate form also requires a finite destination (gemv.rs:126-127).
    if (ok && a.mode == kGemvAccumulate) {
        for (uint64_t i = threadIdx.x; i < a.w.rows; i += kThreads) {
            float yv = a.y[i];
            if (!isfinite(yv)) {
                report(a.status, LBK_NON_FINITE_VALUE, i, __float_as_uint(yv));
                atomicExch(flag, 1);
            }
        }
        __syncthreads();
        ok = (*flag == 0);
    }
    return ok;
}

template <int T, int L>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(GemvArgs a) {
    if (a.mat_table != nullptr) {  // routed expert selected on the device
        uint32_t e = a.sel->expert_id;
        if (e >= a.mat_count) {  // bad routing: report and skip (no out-of-table read)
            if (blockIdx.x == 0 && threadIdx.x == 0) report(a.status, LBK_INVALID_PARAMETER, e, 0);
            return;
        }
        a.w.data = a.mat_table[e];
        a.scale = a.sel->coefficient;
    }
    using Cfg = GemvCfg<T>;
    using HB = typename HBOf<T>::type;
    extern __shared__ __align__(16) uint8_t smem[];
    const int nb = a.w.nb;
    uint32_t* tab0 = reinterpret_cast<uint32_t*>(smem);
    int8_t* qs = reinterpret_cast<int8_t*>(smem + Cfg::kTableBytes);
    float* dsm = reinterpret_cast<float*>(qs + (size_t)nb * kQK);
    int16_t* bs = reinterpret_cast<int16_t*>(dsm + nb);
    size_t tail_off = ((size_t)Cfg::kTableBytes + (size_t)nb * kQK + nb * 4 + nb * 32 + 15) & ~(size_t)15;
    float* tail_all = reinterpret_cast<float*>(smem + tail_off);
    int* flag = reinterpret_cast<int*>(tail_all + (size_t)kWarps * a.tail_slots * nb * Cfg::kTail);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* tail = tail_all + (size_t)warp * a.tail_slots * nb * Cfg::kTail;

    // lane -> (row within step, half block)
    const int tpr = a.tpr;  // threads per row (power of two, >= 2*nb when nb <= 16, else 32)
    const int rps = 32 / tpr;
    const int sub = lane / tpr;
    const int hb0 = lane % tpr;
    const int nhb = 2 * nb;
    const uint64_t rows = a.w.rows;
    const uint64_t steps = (rows + rps - 1) / rps;
    const uint64_t gwarp = (uint64_t)blockIdx.x * kWarps + warp;
    const uint64_t nwarp = (uint64_t)gridDim.x * kWarps;

    // Issue the first step's weight loads before the prologue so their latency
    // overlaps the table fill and the quantization.
    HB cur;
    uint64_t step = gwarp;
    auto row_of = [&](uint64_t s) -> uint64_t { return s * rps + sub; };
    const bool single = (nhb <= tpr);  // each thread owns at most one half block
    if (single && step < steps && row_of(step) < rows && hb0 < nhb) load_hb<L>(cur, a.w, row_of(step), hb0 >> 1, hb0 & 1);

    if (T == LBK_TYPE_IQ2_S) fill_iq2_codes(tab0, a.tables);
    else if (T == LBK_TYPE_IQ3_S) fill_iq3_grid(tab0, a.tables);
    if (!stage_activations(a, nb, qs, dsm, bs, flag)) return;

    ActSmem as{qs, dsm, bs};
    constexpr bool kTr = !Cfg::kIq;
    ActHB act;
    uint32_t nact[32];
    if (single && hb0 < nhb) {
        load_act_hb<kTr>(act, as, hb0 >> 1, hb0 & 1, !Cfg::kIq);
        if (T == LBK_TYPE_IQ3_S) {
#pragma unroll
            for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
        }
    }
    const uint32_t t0 = (uint32_t)__cvta_generic_to_shared(tab0 + lane);

    const int slots = a.tail_slots;  // >= rps, multiple of rps
    auto flush = [&](int nslots, uint64_t first_step) {
        __syncwarp();
        if (lane < nslots) {
            int s_in = lane / rps, sb = lane % rps;
            uint64_t row = (first_step + (uint64_t)s_in * nwarp) * rps + sb;
            if (row < rows) {
                const float* prod = tail + (size_t)lane * nb * Cfg::kTail;
                float v = Cfg::kIq ? iq_tail(prod, nb, 1, T == LBK_TYPE_IQ2_S) : k_tail(prod, nb, 9);
                if (a.mode == kGemvAccumulate)
                    a.y[row] = __fadd_rn(a.y[row], __fmul_rn(a.scale, v));
                else
                    a.y[row] = v;
            }
        }
        __syncwarp();
    };

    uint64_t batch_first = step;
    const int steps_per_batch = slots / rps;
    const int iters = single ? 1 : (nhb + 31) / 32;  // uniform across the warp
    int in_batch = 0;
    for (; step < steps; step += nwarp) {
        const uint64_t row = row_of(step);
        const bool active = row < rows;
        const int slot = in_batch * rps + sub;
        for (int it = 0; it < iters; ++it) {
            const int hb = hb0 + it * tpr;
            const int b = hb >> 1, h = hb & 1;
            const bool mine = active && hb < nhb;
            HB w;
            if (single) {
                w = cur;
                // prefetch the next step's half block while this one computes
                uint64_t ns = step + nwarp;
                if (ns < steps && row_of(ns) < rows && hb0 < nhb) load_hb<L>(cur, a.w, row_of(ns), b, h);
            } else if (mine) {
                load_hb<L>(w, a.w, row, b, h);
                load_act_hb<kTr>(act, as, b, h, !Cfg::kIq);
                if (T == LBK_TYPE_IQ3_S) {
#pragma unroll
                    for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
                }
            }
            if constexpr (Cfg::kIq) {
                IqPart p{0, 0};
                if (mine) {
                    if constexpr (T == LBK_TYPE_IQ2_S)
                        p = dot_hb(w, act, t0);
                    else
                        p = dot_hb(w, act, nact, t0);
                }
                int other = __shfl_xor_sync(0xffffffffu, p.sum, 1);
                if (mine && h == 0) {
                    p.sum += other;
                    if (a.block_sums) a.block_sums[row * nb + b] = p.sum;
                    tail[(size_t)slot * nb + b] = iq_block_product(p, dsm[b]);
                    if (!h_finite(p.d)) report(a.status, LBK_NON_FINITE_SCALE, row * nb + b, p.d);
                }
            } else {
                KPart p;
#pragma unroll
                for (int l = 0; l < 8; l++) p.lane[l] = 0;
                p.min_sum = 0;
                p.dm = 0;
                if (mine) p = dot_hb(w, act, h);
#pragma unroll
                for (int l = 0; l < 8; l++) p.lane[l] += __shfl_xor_sync(0xffffffffu, p.lane[l], 1);
                p.min_sum += __shfl_xor_sync(0xffffffffu, p.min_sum, 1);
                if (mine && h == 0) {
                    if (a.block_sums) {
#pragma unroll
                        for (int l = 0; l < 8; l++) a.block_sums[(row * nb + b) * 9 + l] = p.lane[l];
                        a.block_sums[(row * nb + b) * 9 + 8] = p.min_sum;
                    }
                    float pr[9];
                    k_block_products(p, dsm[b], pr);
                    float* dst = tail + ((size_t)slot * nb + b) * 9;
#pragma unroll
                    for (int i = 0; i < 9; i++) dst[i] = pr[i];
                    if (!h_finite(p.dm & 0xffffu)) report(a.status, LBK_NON_FINITE_SCALE, row * nb + b, p.dm & 0xffffu);
                    if (!h_finite(p.dm >> 16)) report(a.status, LBK_NON_FINITE_SCALE, row * nb + b, p.dm >> 16);
                }
            }
        }
        if (++in_batch == steps_per_batch) {
            flush(steps_per_batch * rps, batch_first);
            in_batch = 0;
            batch_first = step + nwarp;
        }
    }
    if (in_batch > 0) flush(in_batch * rps, batch_first);
}

// ---------------------------------------------------------------------------
// Planar rows by bulk copy. Each warp streams its rows through a ring of
// `stages` shared-memory stages (one step -- 32 / tpr consecutive rows, one
// half block per lane -- per stage, one mbarrier each): the copies of the next
// stages are in flight while a step is decoded, so a warp keeps several KB of
// its rows in flight instead of one register-held step. The IQ lookup table
// arrives by one bulk copy of its prebuilt image. Results, validation and
// reporting are the register kernel's (same products, same tails, same
// order).
//
// The kernel is a programmatic dependent launch: it starts while the stream's
// previous kernel is still running, lets the next one launch at once, and
// before its grid_dep_wait() only asks L2 for its first rows and copies the
// context's lookup table (written once at context creation). The prefetch
// reads the matrix and nothing else, so it is safe whatever the previous
// kernel wrote: L2 is the point of coherence and the later copies read the
// current bytes. The shared-memory copies of the rows, x (or its Q8_K image)
// and every write of y or the status word come after the wait. Back-to-back
// calls thus overlap one call's launch, prologue and first DRAM round trip
// with the previous call's tail.
//
// Shared memory: [table][stages: kWarps * stages * stage][act qs K][d nb]
//                [bsums nb*16][tails kWarps*slots*nb*kTail][flag]

// Bytes of the activation image's qs: rows of more than 16 blocks keep a full
// 32-block image (the two-pass kernel rearranges it lane-major in place).
__host__ __device__ inline uint32_t bulk_qs_bytes(int nb) { return (uint32_t)(nb > 16 ? 32 : nb) * kQK; }

template <int T>
struct BulkLayout {
    uint32_t stage, ring, act, tail, flag, total;
};

template <int T>
__host__ __device__ inline BulkLayout<T> bulk_layout(int nb, int tpr, int slots, int stages) {
    BulkLayout<T> o{};
    const uint32_t rs = planar_row_bytes(TypeInfo<T>::kBlockBytes, nb);
    o.stage = (uint32_t)(32 / tpr) * rs;
    o.ring = (uint32_t)GemvCfg<T>::kTableBytes;
    o.act = o.ring + (uint32_t)(kWarps * stages) * o.stage;
    uint32_t t = o.act + bulk_qs_bytes(nb) + (uint32_t)nb * 4 + (uint32_t)nb * 32;
    o.tail = (t + 15u) & ~15u;
    o.flag = o.tail + (uint32_t)(kWarps * slots * nb * GemvCfg<T>::kTail) * 4u;
    o.total = o.flag + 16u;
    return o;
}

constexpr int kBulkMaxStages = 8;

// P = 1: rows of at most 16 blocks, one half block per lane, its activations
// held in registers for the whole launch. P = 2: rows of 17-32 blocks (a
// block's 8192-wide attention output projection), one row per step; lane l
// decodes half blocks l and l + 32 of the row, each pass with its activations
// loaded from the shared Q8_K image (two sets would not fit in registers).
template <int T, int P>
__global__ void __launch_bounds__(kThreads, 1) gemv_bulk_kernel(GemvArgs a, int stages) {
    using Cfg = GemvCfg<T>;
    using HB = typename HBOf<T>::type;
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[kWarps * kBulkMaxStages + 1];
    const int nb = a.w.nb;
    const BulkLayout<T> lay = bulk_layout<T>(nb, a.tpr, a.tail_slots, stages);
    uint32_t* tab0 = reinterpret_cast<uint32_t*>(smem);
    int8_t* qs = reinterpret_cast<int8_t*>(smem + lay.act);
    float* dsm = reinterpret_cast<float*>(qs + bulk_qs_bytes(nb));
    int16_t* bs = reinterpret_cast<int16_t*>(dsm + nb);
    float* tail_all = reinterpret_cast<float*>(smem + lay.tail);
    int* flag = reinterpret_cast<int*>(smem + lay.flag);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* tail = tail_all + (size_t)warp * a.tail_slots * nb * Cfg::kTail;
    const int tpr = a.tpr;  // threads per row, >= 2 * nb (one half block per lane)
    const int rps = 32 / tpr;
    const int sub = lane / tpr, hb0 = lane % tpr;
    const int b0 = hb0 >> 1, h0 = hb0 & 1;
    const bool lane_on = hb0 < 2 * nb;
    const uint64_t rows = a.w.rows;
    const uint64_t steps = (rows + rps - 1) / rps;
    const uint64_t gwarp = (uint64_t)blockIdx.x * kWarps + warp;
    const uint64_t nwarp = (uint64_t)gridDim.x * kWarps;
    const uint32_t rs = planar_row_bytes(TypeInfo<T>::kBlockBytes, nb);
    const uint8_t* ring = smem + lay.ring + (size_t)warp * stages * lay.stage;
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&s_bar[warp * kBulkMaxStages]);
    const uint32_t bar_t = (uint32_t)__cvta_generic_to_shared(&s_bar[kWarps * kBulkMaxStages]);
    const uint64_t pol = policy_evict_first();

    grid_dep_launch();
    if (lane == 0)
        for (int s = 0; s < stages; s++) {
            const uint64_t st = gwarp + (uint64_t)s * nwarp;
            if (st >= steps) break;
            const uint64_t r0 = st * rps;
            const uint64_t nr = rows - r0 < (uint64_t)rps ? rows - r0 : (uint64_t)rps;
            prefetch_l2(a.w.data + r0 * rs, (uint32_t)(nr * rs));
        }

    // step i of this warp (global step gwarp + i * nwarp) into stage i % stages
    auto issue = [&](uint64_t i) {
        const uint64_t st = gwarp + i * nwarp;
        if (st >= steps) return;
        const uint64_t r0 = st * rps;
        const uint32_t nr = (uint32_t)(rows - r0 < (uint64_t)rps ? rows - r0 : (uint64_t)rps);
        const uint32_t s = (uint32_t)(i % stages);
        mbar_expect_tx(bar0 + 8 * s, nr * rs);
        bulk_g2s_stream(ring_s + s * lay.stage, a.w.data + r0 * rs, nr * rs, bar0 + 8 * s, pol);
    };
    if (lane == 0) {
        for (int s = 0; s < stages; s++) mbar_init(bar0 + 8 * s, 1);
        if (warp == 0 && Cfg::kTableBytes != 0) mbar_init(bar_t, 1);
        mbar_init_fence();
    }
    __syncthreads();
    if constexpr (Cfg::kTableBytes != 0) {
        if (threadIdx.x == 0) {
            mbar_expect_tx(bar_t, (uint32_t)Cfg::kTableBytes);
            bulk_g2s((uint32_t)__cvta_generic_to_shared(tab0),
                     T == LBK_TYPE_IQ2_S ? (const void*)a.tables.iq2_codes : (const void*)a.tables.iq3_grid,
                     (uint32_t)Cfg::kTableBytes, bar_t);
        }
    }
    grid_dep_wait();  // the previous kernel's writes (x, y, the matrix) are visible from here
    // the first stages' rows are in flight during the activation prologue
    if (lane == 0)
        for (int s = 0; s < stages; s++) issue((uint64_t)s);
    const bool ok = stage_activations(a, nb, qs, dsm, bs, flag);
    if constexpr (Cfg::kTableBytes != 0) {
        if (!mbar_wait(bar_t, 0) && threadIdx.x == 0) report(a.status, LBK_TIMEOUT, 10, 0);
    }
    if (!ok) {
        // nothing is written; the copies in flight complete before the CTA exits
        for (int s = 0; s < stages; s++)
            if (gwarp + (uint64_t)s * nwarp < steps) mbar_wait(bar0 + 8 * s, 0);
        return;
    }

    if constexpr (P == 2) {
        // The lane-major image: lane l's 16-byte chunk i of pass p (half block
        // l + 32 p) moves to word (8 p + i) * 32 + l, so that each pass loads
        // its activations without bank conflicts (in natural order the lanes'
        // half blocks lie 128 bytes apart, all in the same banks). One chunk
        // per thread; chunks of half blocks past the row's end are not
        // moved, and their lanes decode but never store.
        static_assert(kThreads == 2 * 8 * 32, "one 16-byte chunk per thread");
        const int t = threadIdx.x, pp = t >> 8, ci = (t >> 5) & 7, l = t & 31;
        const int hb = pp * 32 + l;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (hb < 2 * nb) v = reinterpret_cast<const uint4*>(qs)[hb * 8 + ci];
        __syncthreads();
        if (hb < 2 * nb) reinterpret_cast<uint4*>(qs)[(pp * 8 + ci) * 32 + l] = v;
        __syncthreads();
    }
    ActSmem as{qs, dsm, bs};
    constexpr bool kTr = !Cfg::kIq;
    ActHB act;
    uint32_t nact[32];
    auto load_act = [&](int b) {
        if constexpr (P == 1) {
            load_act_hb<kTr>(act, as, b, h0, !Cfg::kIq);
        } else {
            const uint4* img = reinterpret_cast<const uint4*>(qs) + (b >= 16 ? 8 * 32 : 0) + lane;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint4 v = img[i * 32];
                act.w[4 * i + 0] = v.x;
                act.w[4 * i + 1] = v.y;
                act.w[4 * i + 2] = v.z;
                act.w[4 * i + 3] = v.w;
            }
            finish_act_hb<kTr>(act, as, b, h0, !Cfg::kIq);
        }
        if constexpr (T == LBK_TYPE_IQ3_S) {
#pragma unroll
            for (int i = 0; i < 32; i++) nact[i] = (uint32_t)__vneg4((int)act.w[i]);
        }
    };
    if constexpr (P == 1) {
        if (lane_on) load_act(b0);
    }
    const uint32_t t0 = (uint32_t)__cvta_generic_to_shared(tab0 + lane);
    const StageOff so = stage_off<T>(nb, lane_on ? sub : 0, lane_on ? b0 : 0, lane_on ? h0 : 0);
    // P = 2: the second pass's half block (lane + 32), block 0's offsets on
    // lanes past the row's end (decoded, never stored)
    const bool on1 = P == 2 && lane + 32 < 2 * nb;
    const int b1 = on1 ? b0 + 16 : 0;
    const StageOff so1 = stage_off<T>(nb, 0, b1, on1 ? h0 : 0);

    const int slots = a.tail_slots;  // >= rps, multiple of rps
    auto flush = [&](int nslots, uint64_t first_step) {
        __syncwarp();
        if (lane < nslots) {
            int s_in = lane / rps, sb = lane % rps;
            uint64_t row = (first_step + (uint64_t)s_in * nwarp) * rps + sb;
            if (row < rows) {
                const float* prod = tail + (size_t)lane * nb * Cfg::kTail;
                float v = Cfg::kIq ? iq_tail(prod, nb, 1, T == LBK_TYPE_IQ2_S) : k_tail(prod, nb, 9);
                if (a.mode == kGemvAccumulate)
                    a.y[row] = __fadd_rn(a.y[row], __fmul_rn(a.scale, v));
                else
                    a.y[row] = v;
            }
        }
        __syncwarp();
    };

    const int steps_per_batch = slots / rps;
    int in_batch = 0;
    uint64_t batch_first = gwarp;
    bool live = true;
    uint64_t i = 0;
    for (uint64_t step = gwarp; step < steps; step += nwarp, i++) {
        const uint32_t s = (uint32_t)(i % stages);
        if (live && !(mbar_try_wait(bar0 + 8 * s, (uint32_t)((i / stages) & 1)) ||
                      mbar_wait(bar0 + 8 * s, (uint32_t)((i / stages) & 1)))) {
            live = false;
            if (lane == 0) report(a.status, LBK_TIMEOUT, 11, step);
        }
        HB w, w1;
        load_stage(w, ring + s * lay.stage, so);
        if constexpr (P == 2) load_stage(w1, ring + s * lay.stage, so1);
        __syncwarp();
        if (lane == 0 && live) {
            fence_proxy_async_smem();  // the warp's reads of this stage before its refill
            issue(i + stages);
        }
        const uint64_t row = step * rps + sub;
        const int slot = in_batch * rps + sub;
        // half block hv of block b: its block product into the row's tail slot
        auto consume = [&](const HB& hv, int b, bool mine) {
            if constexpr (Cfg::kIq) {
                IqPart p{0, 0};
                if constexpr (T == LBK_TYPE_IQ2_S)
                    p = dot_hb(hv, act, t0);
                else
                    p = dot_hb(hv, act, nact, t0);
                int other = __shfl_xor_sync(0xffffffffu, p.sum, 1);
                if (mine && h0 == 0) {
                    p.sum += other;
                    tail[(size_t)slot * nb + b] = iq_block_product(p, dsm[b]);
                    if (!h_finite(p.d)) report(a.status, LBK_NON_FINITE_SCALE, row * nb + b, p.d);
                }
            } else {
                KPart p = dot_hb(hv, act, h0);
#pragma unroll
                for (int l = 0; l < 8; l++) p.lane[l] += __shfl_xor_sync(0xffffffffu, p.lane[l], 1);
                p.min_sum += __shfl_xor_sync(0xffffffffu, p.min_sum, 1);
                if (mine && h0 == 0) {
                    float pr[9];
                    k_block_products(p, dsm[b], pr);
                    float* dst = tail + ((size_t)slot * nb + b) * 9;
#pragma unroll
                    for (int q = 0; q < 9; q++) dst[q] = pr[q];
                    if (!h_finite(p.dm & 0xffffu)) report(a.status, LBK_NON_FINITE_SCALE, row * nb + b, p.dm & 0xffffu);
                    if (!h_finite(p.dm >> 16)) report(a.status, LBK_NON_FINITE_SCALE, row * nb + b, p.dm >> 16);
                }
            }
        };
        if constexpr (P == 1) {
            consume(w, b0, live && lane_on && row < rows);
        } else {
            load_act(b0);
            consume(w, b0, live && row < rows);
            load_act(b1);
            consume(w1, b1, live && on1 && row < rows);
        }
        if (++in_batch == steps_per_batch) {
            flush(steps_per_batch * rps, batch_first);
            in_batch = 0;
            batch_first = step + nwarp;
        }
    }
    if (in_batch > 0) flush(in_batch * rps, batch_first);
}

// Stages per warp and tail slots the bulk kernel runs with (stages 0: the
// register kernel instead): as many stages as shared memory holds next to the
// tails, at most kBulkMaxStages, at least two; fewer tail slots (rows per
// tail batch) when that buys stages.
constexpr uint32_t kBulkStaticSmem = (kWarps * kBulkMaxStages + 1) * 8;
template <int T>
int bulk_stages(const GemvArgs& a, int* slots) {
    if (a.mat_table != nullptr || a.block_sums != nullptr || a.w.nb > 32) return 0;
    if (a.tpr < 2 * a.w.nb && a.tpr != 32) return 0;  // 17-32 blocks: one row per step, two passes
    const int rps = 32 / a.tpr;
    int best = 0;
    const bool wide = a.w.nb > 16;  // tail batches down to one row only there (the 16-block plans stay)
    for (int sl : {a.tail_slots, 16, 8, wide ? 4 : 0, wide ? 2 : 0, wide ? 1 : 0}) {
        if (sl == 0) continue;
        if (sl < rps || sl % rps != 0 || sl > a.tail_slots) continue;
        for (int s = kBulkMaxStages; s > best && s >= 2; s--)
            if (bulk_layout<T>(a.w.nb, a.tpr, sl, s).total + kBulkStaticSmem <= kMaxSmem) {
                best = s;
                *slots = sl;
                break;
            }
    }
    return best;
}

template <int T>
cudaError_t launch_gemv_bulk(const GemvArgs& a, int stages, int sm_count, cudaStream_t stream) {
    const size_t smem = bulk_layout<T>(a.w.nb, a.tpr, a.tail_slots, stages).total;
    void (*kernel)(GemvArgs, int) = a.w.nb > 16 ? gemv_bulk_kernel<T, 2> : gemv_bulk_kernel<T, 1>;
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(kernel));
    if (e != cudaSuccess) return e;
    const uint64_t rps = 32 / a.tpr;
    const uint64_t steps = (a.w.rows + rps - 1) / rps;
    uint64_t ctas = (steps + kWarps - 1) / kWarps;
    if (ctas > (uint64_t)sm_count) ctas = sm_count;
    if (ctas < 1) ctas = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see the kernel's grid_dep_wait()
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a, stages);
}

template <int T, int L>
cudaError_t launch_gemv_t(const GemvArgs& a, int sm_count, cudaStream_t stream) {
    if constexpr (L == LBK_LAYOUT_PLANAR) {
        int slots = a.tail_slots;
        const int stages = bulk_stages<T>(a, &slots);
        if (stages > 0 && ((uintptr_t)a.w.data & 15u) == 0) {
            GemvArgs b = a;
            b.tail_slots = slots;
            return launch_gemv_bulk<T>(b, stages, sm_count, stream);
        }
    }
    size_t smem = gemv_smem_bytes<T>(a.w.nb, a.tail_slots);
    if (smem > kMaxSmem) return cudaErrorInvalidValue;
    cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(gemv_kernel<T, L>));
    if (e != cudaSuccess) return e;
    uint64_t rps = 32 / a.tpr;
    uint64_t steps = (a.w.rows + rps - 1) / rps;
    uint64_t ctas = (steps + kWarps - 1) / kWarps;
    if (ctas > (uint64_t)sm_count) ctas = sm_count;
    if (ctas < 1) ctas = 1;
    gemv_kernel<T, L><<<(unsigned)ctas, kThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

size_t gemv_smem_required(int type, int nb, int slots) {
    switch (type) {
        case LBK_TYPE_IQ2_S: return gemv_smem_bytes<LBK_TYPE_IQ2_S>(nb, slots);
        case LBK_TYPE_IQ3_S: return gemv_smem_bytes<LBK_TYPE_IQ3_S>(nb, slots);
        case LBK_TYPE_Q4_K: return gemv_smem_bytes<LBK_TYPE_Q4_K>(nb, slots);
        default: return gemv_smem_bytes<LBK_TYPE_Q5_K>(nb, slots);
    }
}

void gemv_plan(int type, int nb, int* tpr, int* slots) {
    int t = 32;
    if (nb <= 16) {
        t = 2;
        while (t < 2 * nb) t <<= 1;
    }
    int rps = 32 / t;
    bool iq = type == LBK_TYPE_IQ2_S || type == LBK_TYPE_IQ3_S;
    int s = iq ? 32 : 8;
    if (s < rps) s = rps;
    // keep the tail buffer within shared memory for wide rows
    while (s > rps && gemv_smem_required(type, nb, s) > kMaxSmem) s -= rps;
    *tpr = t;
    *slots = s;
}

cudaError_t launch_gemv(int type, int layout, const GemvArgs& a, int sm_count, cudaStream_t stream) {
    const bool planar = layout == LBK_LAYOUT_PLANAR;
    switch (type) {
        case LBK_TYPE_IQ2_S:
            return planar ? launch_gemv_t<LBK_TYPE_IQ2_S, LBK_LAYOUT_PLANAR>(a, sm_count, stream)
                          : launch_gemv_t<LBK_TYPE_IQ2_S, LBK_LAYOUT_GGUF>(a, sm_count, stream);
        case LBK_TYPE_IQ3_S:
            return planar ? launch_gemv_t<LBK_TYPE_IQ3_S, LBK_LAYOUT_PLANAR>(a, sm_count, stream)
                          : launch_gemv_t<LBK_TYPE_IQ3_S, LBK_LAYOUT_GGUF>(a, sm_count, stream);
        case LBK_TYPE_Q4_K:
            return planar ? launch_gemv_t<LBK_TYPE_Q4_K, LBK_LAYOUT_PLANAR>(a, sm_count, stream)
                          : launch_gemv_t<LBK_TYPE_Q4_K, LBK_LAYOUT_GGUF>(a, sm_count, stream);
        default:
            return planar ? launch_gemv_t<LBK_TYPE_Q5_K, LBK_LAYOUT_PLANAR>(a, sm_count, stream)
                          : launch_gemv_t<LBK_TYPE_Q5_K, LBK_LAYOUT_GGUF>(a, sm_count, stream);
    }
}

}  // namespace lbk
