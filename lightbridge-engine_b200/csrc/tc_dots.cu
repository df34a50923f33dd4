// tc_dots.cu -- grouped row dots of IQ2_S and IQ3_S matrices on the
// 5th-generation tensor cores (tcgen05.mma kind::i8), bit-identical to the
// dp4a kernels. The expert-parallel items path runs its gate/up (IQ2_S) and
// down (IQ3_S) here when an expert has enough pairs. IQ3_S differs from the
// IQ2_S scheme below only in its groups: one multiplier per 32 weights, so
// one MMA and one accumulator per 32-byte chunk, with the signs applied to
// the weight bytes.
//
// A job is one 128-row tile of one matrix and up to 32 tokens (the pairs
// routed to one expert). The reference's dot of an IQ2_S block with a Q8_K
// block (dot_iq2_s, bridge-quant-layout/src/q8_k.rs:339-364) is an integer
// sum over sixteen 16-weight groups, each multiplied by its own scale
// 1 + 2s (s a 4-bit field), then one f32 product per block, chained over the
// blocks. Scaled weights reach 43 * 31 = 1333, beyond int8, so the scales
// cannot be folded into the operands: instead every 16-weight group gets its
// own int32 accumulator. One MMA (K = 32 int8) covers two groups; it runs
// twice, once against the activations with the second 16 bytes of each
// 32-byte chunk zeroed and once with the first 16 zeroed -- two shared-memory
// descriptors over one activation copy laid out [lo | zeros | hi], so the
// masking costs no extra bytes. Per half block (128 weights: 8 groups):
//   decode  128 threads, one row each, write the half block's int8 weights
//           into the canonical K-major, no-swizzle layout (4 chunks of
//           128 rows x 32 bytes);
//   MMA     one thread issues 8 MMAs (M = 128, N = 16 or 32, K = 32) into 8
//           TMEM accumulators of this unit's buffer (two buffers: the decode
//           of the next unit overlaps these MMAs);
//   epilogue every thread reads its row's 8 x N accumulators (tcgen05.ld),
//           forms the exact integer sum sum_g (1 + 2 s_g) acc_g per token,
//           and at the end of a block the reference's f32 block product and
//           chain (iq_block_product, then 0.125 * the sum over blocks).
// Waits on MMA completion are bounded (LBK_TIMEOUT).

#include "lbk_kernels.h"
#include "lbk_tc.h"

namespace lbk {

namespace {

constexpr int kTcThreads = 128;  // one thread per tile row (TMEM lane)
constexpr int kTcRows = 128;
constexpr int kTcMaxTok = 32;
// TMEM per CTA: two buffers of kAcc accumulators x 32 columns (IQ2_S: 512,
// the whole of an SM's; IQ3_S: 256, so two CTAs share an SM)
constexpr int kTabCopies = 8;        // copies of the 1024-entry code table (bank spread)

// shared memory: [table 1024 * 8 words][W: 2 x 4 chunks x 4 KB][A: 2 x 4 chunks x 3 x 32 x 16 B][dx: 2 x 32]
constexpr int kTabBytes = 1024 * kTabCopies * 4;
constexpr int kWChunk = kTcRows * 32;        // 4 KB: 128 rows x 32 bytes
constexpr int kWUnit = 4 * kWChunk;          // one half block
constexpr int kAChunkMax = 3 * kTcMaxTok * 16;
constexpr int kAUnit = 4 * kAChunkMax;
constexpr int kOffW = kTabBytes;
constexpr int kOffA = kOffW + 2 * kWUnit;
constexpr int kOffDx = kOffA + 2 * kAUnit;
constexpr int kOffChain = kOffDx + 2 * kTcMaxTok * 4;  // [token][thread] f32 chains
constexpr int kTcSmem = kOffChain + kTcMaxTok * kTcThreads * 4;
// IQ2_S launches take more than half of an SM's shared memory: one CTA per
// SM, so no CTA waits in tcgen05.alloc for another's 512 columns. IQ3_S
// launches take less: two CTAs per SM, 256 columns each.
constexpr int kTcSmemLaunch = 116 * 1024;
static_assert(kTcSmem <= kTcSmemLaunch, "shared memory");
static_assert(2 * kTcSmem + 2 * 2048 <= 228 * 1024, "two IQ3_S CTAs per SM");

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    // K-major, no swizzle: start, leading (K-half) and stride (8-row group)
    // byte offsets in 16-byte units; bits 46-47 = 1 (the sm_100 descriptor)
    return (uint64_t)((addr & 0x3ffffu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46);
}

// kind::i8: D s32 (bits 4-5 = 2), A and B signed (bits 7-9, 10-12 = 1),
// both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Signed grid bytes of one IQ2_S half block (the decode of dot_hb without the
// dot): words 8g + 2l, 8g + 2l + 1 hold weights 8l .. 8l + 7 of group g.
__device__ __forceinline__ void decode_iq2_hb(const Iq2HB& w, const uint32_t* tab, uint32_t copy, uint32_t (&out)[32]) {
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const uint32_t qsw = w32(w.qs, gi);
        const uint32_t sgw = w32(w.sg, gi);
        const uint32_t Q = (w.qh >> (2 * gi)) & 0x03030303u;
        const uint32_t sp[4] = {signs_at2<0>(sgw), signs_at2<1>(sgw), signs_at2<2>(sgw), signs_at2<3>(sgw)};
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t idx = prmt(qsw, Q, sel_idx(l, l));
            const uint32_t code = tab[idx * kTabCopies + copy];
            const uint32_t sel = code | (sp[l] & 0x44444444u);
            out[gi * 8 + 2 * l] = prmt(kIq2PoolPos, kIq2PoolNeg, sel);
            out[gi * 8 + 2 * l + 1] = prmt(kIq2PoolPos, kIq2PoolNeg, sel >> 16);
        }
    }
}

// Epilogue of the unit in TMEM buffer BUF (a half block; BUF is its half):
// the exact integer group sums per token, and after the second half the
// block's f32 product, chained in block order.
// Signed weight bytes of one IQ3_S half block (the decode of dot_hb for
// IQ3_S, the signs applied to the weights instead of the activations): words
// 8g + 2l, 8g + 2l + 1 hold weights 8l .. 8l + 7 of group g.
__device__ __forceinline__ void decode_iq3_hb(const Iq3HB& w, const uint32_t* tab, uint32_t copy, uint32_t (&out)[32]) {
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const uint32_t qa = gi < 2 ? w32(w.qs0, gi * 2) : w32(w.qs1, (gi - 2) * 2);
        const uint32_t qb = gi < 2 ? w32(w.qs0, gi * 2 + 1) : w32(w.qs1, (gi - 2) * 2 + 1);
        const uint32_t sgw = w32(w.sg, gi);
        const uint32_t Q = (w.qh >> (2 * gi)) & 0x03030303u;
        const uint32_t Q1 = Q & 0x01010101u;
        const uint32_t Q2 = (Q >> 1) & 0x01010101u;
        const uint32_t sp[4] = {signs_at2<0>(sgw), signs_at2<1>(sgw), signs_at2<2>(sgw), signs_at2<3>(sgw)};
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t q2 = l < 2 ? qa : qb;
            const uint32_t i1 = prmt(q2, Q1, sel_idx(2 * (l & 1), l));
            const uint32_t i2 = prmt(q2, Q2, sel_idx(2 * (l & 1) + 1, l));
            const uint32_t g1 = tab[i1 * kTabCopies + copy];
            const uint32_t g2 = tab[i2 * kTabCopies + copy];
            const uint32_t slo = (sp[l] & 0x4444u) | 0x3210u;
            const uint32_t shi = ((sp[l] >> 16) & 0x4444u) | 0x3210u;
            out[gi * 8 + 2 * l] = prmt(g1, (uint32_t)__vneg4((int)g1), slo);
            out[gi * 8 + 2 * l + 1] = prmt(g2, (uint32_t)__vneg4((int)g2), shi);
        }
    }
}

template <int T>
struct TcType {
    static constexpr bool kIq2 = T == LBK_TYPE_IQ2_S;
    static constexpr int kAcc = kIq2 ? 8 : 4;  // accumulators per half block: 16-weight groups / 32-weight groups
    static constexpr int kEntries = kIq2 ? kIq2CodeEntries : kIq3GridEntries;
    static constexpr uint32_t kBufCols = (uint32_t)kAcc * 32;  // one buffer: kAcc accumulators of up to 32 tokens
    // TMEM buffers: IQ3_S double-buffers (its MMAs overlap the previous
    // unit's epilogue) in 256 columns; IQ2_S (8 accumulators) single-buffers
    // in 256 columns too, so that two CTAs share an SM and one CTA's MMA
    // waits overlap the other's decode
    static constexpr uint32_t kTmemBufs = kIq2 ? 1 : 2;
    static constexpr uint32_t kTmemCols = kTmemBufs * kBufCols;
    static constexpr int kSmemLaunch = kTcSmem;
    using HB = typename std::conditional<kIq2, Iq2HB, Iq3HB>::type;
};

template <int T, int BUF>
__device__ __forceinline__ void tc_epilogue(const TcDotsArgs& a, uint32_t bar0, uint32_t tmem, int warp, int npad,
                                            uint32_t n, int b, const float* s_dx, const uint32_t (&ls)[2][8],
                                            const uint32_t (&dw)[2], uint32_t (&phase)[2], bool& live,
                                            int32_t (&bsum)[kTcMaxTok], float* chain) {
    if (live && !(mbar_try_wait(bar0 + 8 * BUF, phase[BUF]) || mbar_wait(bar0 + 8 * BUF, phase[BUF]))) {
        live = false;
        report(a.status, LBK_TIMEOUT, 12, (uint32_t)blockIdx.x);
    }
    phase[BUF] ^= 1u;
    tc_fence_after();
    const uint32_t tbase =
        tmem + ((uint32_t)(warp * 32) << 16) + (TcType<T>::kTmemBufs == 2 ? (uint32_t)BUF * TcType<T>::kBufCols : 0u);
    // two groups' accumulators per wait (up to four loads in flight)
#pragma unroll
    for (int g = 0; g < TcType<T>::kAcc; g += 2) {
        uint32_t r[2][kTcMaxTok];
#pragma unroll
        for (int gg = 0; gg < 2; gg++) {
            tc_ld16(tbase + (uint32_t)((g + gg) * npad), *reinterpret_cast<uint32_t(*)[16]>(&r[gg][0]));
            if (npad > 16) tc_ld16(tbase + (uint32_t)((g + gg) * npad + 16), *reinterpret_cast<uint32_t(*)[16]>(&r[gg][16]));
        }
        tc_wait_ld();
#pragma unroll
        for (int gg = 0; gg < 2; gg++) {
            const int32_t m = (int32_t)ls[BUF][g + gg];
#pragma unroll
            for (int i = 0; i < kTcMaxTok; i++)
                if (i < npad) bsum[i] += m * (int32_t)r[gg][i];
        }
    }
    tc_fence_before();
    if constexpr (BUF == 1) {
#pragma unroll
        for (int t = 0; t < kTcMaxTok; t++) {
            if (t < (int)n) {
                const IqPart p{bsum[t], dw[1]};
                float* c = chain + t * kTcThreads;
                *c = __fadd_rn(*c, iq_block_product(p, s_dx[(b & 1) * kTcMaxTok + t]));
            }
            bsum[t] = 0;
        }
    }
}

template <int T>
__global__ void __launch_bounds__(kTcThreads, 1) tc_dots_kernel(TcDotsArgs a) {
    using TT = TcType<T>;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[2];
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5;
    uint4 job;  // {matrix, first row, first pair, tokens}
    TcMatrix mat;
    if (a.jobs != nullptr) {
        job = a.jobs[blockIdx.x];
        if (job.x >= a.nmat || job.w == 0 || job.w > (uint32_t)kTcMaxTok || job.y >= a.mats[job.x].rows ||
            ((uintptr_t)a.mats[job.x].data & 15u) != 0) {
            if (tid == 0) report(a.status, LBK_INVALID_PARAMETER, blockIdx.x, job.x);
            return;  // before any TMEM allocation
        }
        mat = a.mats[job.x];
    } else {
        const uint32_t tiles = (a.rows + kTcRows - 1) / kTcRows, mpg = a.mats_per_group;
        const uint32_t g = blockIdx.x / (mpg * tiles), m = (blockIdx.x / tiles) % mpg, tile = blockIdx.x % tiles;
        if (g >= __ldcg(a.ngroups)) return;  // fewer groups than the grid's bound
        const uint4 gr = __ldcg(a.groups + g);
        if (gr.x >= a.experts || gr.z == 0 || gr.z > (uint32_t)kTcMaxTok) {
            if (tid == 0) report(a.status, LBK_INVALID_PARAMETER, g, gr.z);
            return;
        }
        mat = TcMatrix{m == 0 ? a.gate[gr.x] : a.up[gr.x], a.rows, a.nb, (uint64_t)m * a.rows};
        if (((uintptr_t)mat.data & 15u) != 0) {
            if (tid == 0) report(a.status, LBK_INVALID_PARAMETER, g, gr.x);
            return;
        }
        job = make_uint4(0, tile * kTcRows, gr.y, gr.z);
    }
    const uint32_t row0 = job.y, p0 = job.z, n = job.w;
    const int npad = n <= 16 ? 16 : 32;
    const uint32_t idesc = idesc_i8(kTcRows, npad);
    const int nb = (int)mat.nb;
    const uint32_t rs = planar_row_bytes(TypeInfo<T>::kBlockBytes, nb);
    const uint32_t row = row0 + (uint32_t)tid;
    const bool row_ok = row < mat.rows;

    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
    const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&s_bar[0]);
    float* s_dx = reinterpret_cast<float*>(smem + kOffDx);
    const int achunk = 3 * npad * 16;  // [lo | zeros | hi] of one 32-byte chunk, npad tokens

    // the code table / grid, compact, kTabCopies interleaved copies (entry e's copy j at e * kTabCopies + j)
    const uint32_t* img = reinterpret_cast<const uint32_t*>(TT::kIq2 ? (const void*)a.tables.iq2_codes
                                                                      : (const void*)a.tables.iq3_grid);
    for (int i = tid; i < TT::kEntries * kTabCopies; i += kTcThreads) tab[i] = img[(i / kTabCopies) * 32];
    // zero rows of the activation buffers (the masks, and padded tokens)
    for (int i = tid; i < 2 * kAUnit / 16; i += kTcThreads)
        reinterpret_cast<uint4*>(smem + kOffA)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        mbar_init(bar0, 1);
        mbar_init(bar0 + 8, 1);
        mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(&s_tmem)),
                     "r"(TT::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    float* chain = reinterpret_cast<float*>(smem + kOffChain) + tid;  // this thread's chains, kTcThreads apart
    int32_t bsum[kTcMaxTok];
#pragma unroll
    for (int t = 0; t < kTcMaxTok; t++) {
        chain[t * kTcThreads] = 0.0f;
        bsum[t] = 0;
    }
    uint32_t ls[2][8];  // the units' group multipliers (this thread's row): IQ2_S 8 x (1 + 2s), IQ3_S 4
    uint32_t dw[2];     // their block scales (binary16 bits)
    uint32_t phase[2] = {0, 0};
    bool live = true;

    typename TT::HB w{};
    const uint8_t* rowp = mat.data + (uint64_t)(row_ok ? row : row0) * rs;
    uint4 av[2];  // this thread's activation words of the next unit (pairs * 8 <= 2 * kTcThreads)
    auto load_w = [&](int bb, int hh) {
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int i = tid + j * kTcThreads;
            if (i < (int)n * 8) {
                const int t = i >> 3, gi = (i >> 1) & 3, half = i & 1;
                const uint8_t* img =
                    a.q8 + (uint64_t)a.pair_tokens[p0 + t] * a.q8_row_bytes + (uint64_t)bb * kQ8IBytes;
                av[j] = __ldg(reinterpret_cast<const uint4*>(img + hh * 128 + gi * 32 + half * 16));
            }
        }
        if (row_ok) {
            if constexpr (TT::kIq2) {  // planar IQ2_S: qs | signs | qh | scales | d
                w.qs = __ldg(reinterpret_cast<const uint4*>(rowp + bb * 32 + 16 * hh));
                w.sg = __ldg(reinterpret_cast<const uint4*>(rowp + nb * 32 + bb * 32 + 16 * hh));
                w.qh = __ldg(reinterpret_cast<const uint32_t*>(rowp + nb * 64 + bb * 8 + 4 * hh));
                w.sc = __ldg(reinterpret_cast<const uint32_t*>(rowp + nb * 72 + bb * 8 + 4 * hh));
                w.d = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(rowp + nb * 80 + bb * 2));
            } else {  // planar IQ3_S: qs | signs | qh | scales | d
                w.qs0 = __ldg(reinterpret_cast<const uint4*>(rowp + bb * 64 + 32 * hh));
                w.qs1 = __ldg(reinterpret_cast<const uint4*>(rowp + bb * 64 + 32 * hh + 16));
                w.sg = __ldg(reinterpret_cast<const uint4*>(rowp + nb * 64 + bb * 32 + 16 * hh));
                w.qh = __ldg(reinterpret_cast<const uint32_t*>(rowp + nb * 96 + bb * 8 + 4 * hh));
                w.sc = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(rowp + nb * 104 + bb * 4 + 2 * hh));
                w.d = (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(rowp + nb * 108 + bb * 2));
            }
        }
    };
    load_w(0, 0);
#pragma unroll 1
    for (int b = 0; b < nb; b++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int buf = h;
            uint8_t* wu = smem + kOffW + buf * kWUnit;
            uint8_t* au = smem + kOffA + buf * kAUnit;
            // decode this thread's row, half block (b, h) (loaded one unit ahead)
            uint32_t q[32];
            if constexpr (TT::kIq2)
                decode_iq2_hb(w, tab, (uint32_t)(tid & (kTabCopies - 1)), q);
            else
                decode_iq3_hb(w, tab, (uint32_t)(tid & (kTabCopies - 1)), q);
            if (!row_ok) {
#pragma unroll
                for (int i = 0; i < 32; i++) q[i] = 0u;
            }
            if constexpr (TT::kIq2) {
                const uint32_t s1w = (w.sc & 0x0f0f0f0fu) * 2u + 0x01010101u;
                const uint32_t s2w = ((w.sc >> 4) & 0x0f0f0f0fu) * 2u + 0x01010101u;
#pragma unroll
                for (int gi = 0; gi < 4; gi++) {
                    ls[buf][2 * gi] = prmt(s1w, 0, 0x4440u | gi);
                    ls[buf][2 * gi + 1] = prmt(s2w, 0, 0x4440u | gi);
                }
            } else {  // one multiplier 1 + 2 * nibble per 32-weight group (dot_hb for IQ3_S)
                const uint32_t st = (w.sc & 0x0f0fu) | ((w.sc & 0xf0f0u) << 12);
                const uint32_t sw = st * 2u + 0x01010101u;
#pragma unroll
                for (int gi = 0; gi < 4; gi++) ls[buf][gi] = prmt(sw, 0, 0x4440u | (uint32_t)((gi & 1) * 2 + (gi >> 1)));
            }
            dw[buf] = w.d;
            // chunk gi: [K-half 0: 16 row groups x 128 B][K-half 1: 16 x 128 B]
#pragma unroll
            for (int gi = 0; gi < 4; gi++) {
                uint8_t* ch = wu + gi * kWChunk + (tid >> 3) * 128 + (tid & 7) * 16;
                *reinterpret_cast<uint4*>(ch) = make_uint4(q[gi * 8 + 0], q[gi * 8 + 1], q[gi * 8 + 2], q[gi * 8 + 3]);
                *reinterpret_cast<uint4*>(ch + 2048) =
                    make_uint4(q[gi * 8 + 4], q[gi * 8 + 5], q[gi * 8 + 6], q[gi * 8 + 7]);
            }
            // the tokens' activations for this unit (loaded one unit ahead):
            // chunk gi, token t -> lo at (t / 8) * 128 + (t % 8) * 16, hi at
            // 2 * npad * 16 + the same
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int i = tid + j * kTcThreads;
                if (i < (int)n * 8) {
                    const int t = i >> 3, gi = (i >> 1) & 3, half = i & 1;
                    *reinterpret_cast<uint4*>(au + gi * achunk + half * 2 * npad * 16 + (t >> 3) * 128 + (t & 7) * 16) =
                        av[j];
                }
            }
            if (h == 0 && tid < (int)n)
                s_dx[(b & 1) * kTcMaxTok + tid] =
                    __uint_as_float(__ldg(reinterpret_cast<const uint32_t*>(
                        a.q8 + (uint64_t)a.pair_tokens[p0 + tid] * a.q8_row_bytes + (uint64_t)b * kQ8IBytes + 288)));
            // the next unit's weights and activations, in flight during this
            // unit's MMAs and epilogue (w and av are consumed above)
            if (h == 0) load_w(b, 1);
            else if (b + 1 < nb) load_w(b + 1, 0);
            fence_proxy_async_smem();  // the decoded tiles before the tensor core reads them
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0 && live) {
                const uint32_t wb = sbase + (uint32_t)(kOffW + buf * kWUnit);
                const uint32_t ab = sbase + (uint32_t)(kOffA + buf * kAUnit);
#pragma unroll
                for (int gi = 0; gi < 4; gi++) {
                    const uint64_t da = smem_desc(wb + gi * kWChunk, 2048, 128);
                    const uint32_t ac = ab + (uint32_t)(gi * achunk);
                    if constexpr (TT::kIq2) {  // two 16-weight groups: one MMA each, the other half zeroed
                        const uint64_t dlo = smem_desc(ac, (uint32_t)(npad * 16), 128);  // K-half 1 -> the zeros
                        const uint64_t dhi = smem_desc(ac + (uint32_t)(npad * 16), (uint32_t)(npad * 16), 128);
                        const uint32_t d0 = tmem + (TT::kTmemBufs == 2 ? (uint32_t)buf * TT::kBufCols : 0u) +
                                            (uint32_t)((2 * gi) * npad);
                        tc_mma_i8(d0, da, dlo, idesc);
                        tc_mma_i8(d0 + (uint32_t)npad, da, dhi, idesc);
                    } else {  // one 32-weight group: K-half 1 is the hi part, past the zeros
                        const uint64_t dfull = smem_desc(ac, (uint32_t)(2 * npad * 16), 128);
                        tc_mma_i8(tmem + (TT::kTmemBufs == 2 ? (uint32_t)buf * TT::kBufCols : 0u) + (uint32_t)(gi * npad),
                                  da, dfull, idesc);
                    }
                }
                tc_commit(bar0 + 8 * buf);
            }
            if constexpr (TT::kTmemBufs == 2) {
                // the previous unit's epilogue while these MMAs run
                if (h == 1)
                    tc_epilogue<T, 0>(a, bar0, tmem, warp, npad, n, b, s_dx, ls, dw, phase, live, bsum, chain);
                else if (b > 0)
                    tc_epilogue<T, 1>(a, bar0, tmem, warp, npad, n, b - 1, s_dx, ls, dw, phase, live, bsum, chain);
            } else {
                // one TMEM buffer: this unit's epilogue before the next unit's MMAs
                if (h == 0)
                    tc_epilogue<T, 0>(a, bar0, tmem, warp, npad, n, b, s_dx, ls, dw, phase, live, bsum, chain);
                else
                    tc_epilogue<T, 1>(a, bar0, tmem, warp, npad, n, b, s_dx, ls, dw, phase, live, bsum, chain);
            }
            // the next decode overwrites the other buffer: its MMAs completed
            // (waited above) and its accumulators are read
            __syncthreads();
        }
    }
    if constexpr (TT::kTmemBufs == 2)
        tc_epilogue<T, 1>(a, bar0, tmem, warp, npad, n, nb - 1, s_dx, ls, dw, phase, live, bsum, chain);

    if (row_ok && live) {
#pragma unroll
        for (int t = 0; t < kTcMaxTok; t++) {
            if (t < (int)n) {
                // the pair's row: its grouped position, or its token (item) when scattering
                const uint64_t r = a.out_by_token ? (uint64_t)a.pair_tokens[p0 + t] : (uint64_t)(p0 + t);
                const float c = chain[t * kTcThreads];
                float* dst = a.ret_addr != nullptr
                                 ? reinterpret_cast<float*>(a.ret_peers[a.ret_addr[r].x] + a.ret_off) +
                                       (uint64_t)a.ret_addr[r].y * a.dots_stride
                                 : a.dots + r * a.dots_stride;
                dst[mat.out_offset + row] = TT::kIq2 ? __fmul_rn(0.125f, c) : c;
            }
        }
    }
    if (a.ret_addr != nullptr) __threadfence_system();  // rows returned in place: visible before the done flags
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TT::kTmemCols) : "memory");
}

// One warp per (grouped pair, 256-row block of h): SwiGLU of the block's
// gate / up dots, then the warp's Q8_K of the block into the pair's image.
__global__ void __launch_bounds__(256) tc_swiglu_quant_kernel(TcSwigluArgs a) {
    const int lane = threadIdx.x & 31;
    const uint32_t n = min(__ldcg(a.count), a.cap);
    const uint64_t units = (uint64_t)n * a.nb_f;
    for (uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < units;
         w += ((uint64_t)gridDim.x * blockDim.x) >> 5) {
        const uint32_t p = (uint32_t)(w / a.nb_f), blk = (uint32_t)(w % a.nb_f);
        const uint32_t item = __ldcg(a.pairs + p);
        const float* g = a.dots + (uint64_t)p * 2 * a.ffn + blk * kQK + lane * 8;
        const float* u = g + a.ffn;
        float v[8];
        bool bad = false;
        int bad_i = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            v[i] = swiglu_ref(__ldcg(g + i), __ldcg(u + i));
            if (!isfinite(v[i]) && !bad) {
                bad = true;
                bad_i = i;
            }
        }
        const uint64_t sidx = (uint64_t)item * a.slots;  // slot 0 of the item
        if (bad) report(a.status, LBK_NON_FINITE_VALUE, sidx * a.ffn + blk * kQK + lane * 8 + bad_i, __float_as_uint(v[bad_i]));
        if (__ballot_sync(0xffffffffu, bad)) continue;
        Q8Block q = quantize_q8k_warp(v, lane);
        int32_t pair = q.pair_sum + __shfl_xor_sync(0xffffffffu, q.pair_sum, 1);
        store_q8i(a.hq + (sidx * a.nb_f + blk) * kQ8IBytes, q, pair, lane);
    }
}

}  // namespace

int tc_dots_smem_bytes() { return kTcSmemLaunch; }

cudaError_t launch_tc_swiglu_quant(const TcSwigluArgs& a, int sm_count, cudaStream_t stream) {
    uint64_t warps = (uint64_t)a.cap * a.nb_f;
    uint64_t grid = (warps + 7) / 8;
    if (grid > (uint64_t)sm_count * 8) grid = (uint64_t)sm_count * 8;
    if (grid < 1) grid = 1;
    tc_swiglu_quant_kernel<<<(unsigned)grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

template <int T>
cudaError_t launch_tc_dots_t(const TcDotsArgs& a, uint32_t jobs, cudaStream_t stream) {
    if (jobs == 0) return cudaSuccess;
    cudaError_t e =
        cudaFuncSetAttribute(tc_dots_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcType<T>::kSmemLaunch);
    if (e != cudaSuccess) return e;
    tc_dots_kernel<T><<<jobs, kTcThreads, TcType<T>::kSmemLaunch, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_tc_dots(int type, const TcDotsArgs& a, uint32_t jobs, cudaStream_t stream) {
    if (type == LBK_TYPE_IQ2_S) return launch_tc_dots_t<LBK_TYPE_IQ2_S>(a, jobs, stream);
    if (type == LBK_TYPE_IQ3_S) return launch_tc_dots_t<LBK_TYPE_IQ3_S>(a, jobs, stream);
    return cudaErrorInvalidValue;
}

}  // namespace lbk
