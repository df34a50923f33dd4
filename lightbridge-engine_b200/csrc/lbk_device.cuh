// lbk_device.cuh -- device building blocks of the quantized expert kernels.
//
// Work unit: a "half block" (HB) = 128 consecutive lanes of one 256-lane
// super-block of one packed row. A thread owns one HB position of the input
// vector for the whole kernel and keeps that HB's Q8_K activation bytes in
// registers; it then streams the matching HB of many weight rows. Integer sums
// are exact, so any split of a block's lanes gives the reference's per-block
// int32 sums; the f32 tail (product per block, then a sequential sum over
// blocks in block order) is replayed separately, one row per lane.
//
// Reference arithmetic restated here: bridge-quant-layout/src/q8_k.rs
// (quantize :16-76, nearest_int :224-228, dot_q4_or_q5_k :247-327,
// dot_iq2_s :329-370, dot_iq3_s :372-434), k_quants.rs (scale_min :231-240).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/lightbridge_kernels.h"

namespace lbk {

constexpr int kQK = 256;
constexpr int kQ8Bytes = 292;

// ------------------------------------------------------------ device status

// First device-detected failure; written once (CAS on `status`).
struct DeviceStatus {
    int32_t status;
    uint32_t bits;
    uint64_t index;
};

__device__ __forceinline__ void report(DeviceStatus* st, int32_t code, uint64_t index, uint32_t bits) {
    if (st == nullptr) return;
    if (atomicCAS(&st->status, 0, -1) == 0) {
        st->index = index;
        st->bits = bits;
        __threadfence();
        atomicExch(&st->status, code);
    }
}

__device__ __forceinline__ bool status_set(const DeviceStatus* st) {
    return st != nullptr && *((volatile const int32_t*)&st->status) != 0;
}

// ----------------------------------------------------------------- types

template <int T>
struct TypeInfo;
template <>
struct TypeInfo<LBK_TYPE_IQ2_S> {
    static constexpr int kBlockBytes = 82;
    static constexpr int kTail = 1;  // f32 products per block in the tail
};
template <>
struct TypeInfo<LBK_TYPE_IQ3_S> {
    static constexpr int kBlockBytes = 110;
    static constexpr int kTail = 1;
};
template <>
struct TypeInfo<LBK_TYPE_Q4_K> {
    static constexpr int kBlockBytes = 144;
    static constexpr int kTail = 9;  // 8 lane products + min product
};
template <>
struct TypeInfo<LBK_TYPE_Q5_K> {
    static constexpr int kBlockBytes = 176;
    static constexpr int kTail = 9;
};

// ------------------------------------------------------------ small helpers

__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) {
    return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p));
}
__device__ __forceinline__ uint32_t ldg_u32(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
__device__ __forceinline__ uint4 ldg_u128(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// Streaming loads for packed weights: read once, do not keep in L1.
__device__ __forceinline__ uint4 ldw_u128(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldw_u32(const uint8_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldw_u16(const uint8_t* p) {
    unsigned short v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
// Two-byte-aligned 4-byte load (GGUF IQ blocks are only 2-byte aligned).
__device__ __forceinline__ uint32_t ldw_u32_a2(const uint8_t* p) { return ldw_u16(p) | (ldw_u16(p + 2) << 16); }
__device__ __forceinline__ uint4 ldw_u128_a2(const uint8_t* p) {
    return make_uint4(ldw_u32_a2(p), ldw_u32_a2(p + 4), ldw_u32_a2(p + 8), ldw_u32_a2(p + 12));
}

// Planar rows staged in shared memory (a copy of consecutive planar rows is
// itself a planar matrix): the HB loaders read it with ordinary shared loads.
constexpr int kLayoutStage = 2;

template <int LAYOUT>
__device__ __forceinline__ uint4 wld128(const uint8_t* p) {
    if constexpr (LAYOUT == kLayoutStage) return *reinterpret_cast<const uint4*>(p);
    else return ldw_u128(p);
}
template <int LAYOUT>
__device__ __forceinline__ uint32_t wld32(const uint8_t* p) {
    if constexpr (LAYOUT == kLayoutStage) return *reinterpret_cast<const uint32_t*>(p);
    else return ldw_u32(p);
}
template <int LAYOUT>
__device__ __forceinline__ uint32_t wld16(const uint8_t* p) {
    if constexpr (LAYOUT == kLayoutStage) return *reinterpret_cast<const uint16_t*>(p);
    else return ldw_u16(p);
}

// ------------------------------------------------ bulk copies and mbarriers
//
// Global -> shared bulk copies (cp.async.bulk into the issuing CTA only)
// completing on an mbarrier in that CTA. Source and destination 16-byte aligned, size a
// multiple of 16.

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity: false after ~2^22 polls
// (each poll may itself suspend briefly), so a lost copy ends in an error
// status instead of a hang.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); i++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// L2 eviction priority for bytes read once (the streamed weight rows): they
// are evicted before anything else, so the lines that are read again -- the
// kernels' code, the table images, the activations, and the down rows the
// gate/up kernel prefetches for the down kernel -- stay in L2.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s_stream(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void prefetch_l2_stream(const void* p, uint32_t bytes, uint64_t pol) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p), "r"(bytes), "l"(pol) : "memory");
}
// Orders this thread's earlier generic-proxy shared accesses before later
// async-proxy (bulk copy) writes to the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Programmatic dependent launch: wait until the grid this one depends on has
// completed and its writes are visible (a no-op for an ordinary launch), and
// let the grid that depends on this one start launching.
// Flag published with release semantics at GPU scope, read with acquire.
__device__ __forceinline__ void st_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// System scope (another GPU's flags, over NVLink).
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Arrival on a counter with release (this warp's earlier writes, ordered by a
// __syncwarp before it, become visible with the arrival) and acquire (the
// other arrivers' writes are visible to the last one) at GPU scope: one
// operation instead of a fence, the atomic and a second fence.
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Hint that [p, p+bytes) will be read soon: bring it into L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }
__device__ __forceinline__ bool h_finite(uint32_t bits16) { return ((bits16 >> 10) & 0x1f) != 0x1f; }
__device__ __forceinline__ uint32_t w32(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// PTX byte permute with the full 4-bit selector (bit 3 = replicate the
// selected byte's sign bit; __byte_perm only honours 3 bits).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 32-bit shared-memory load at a shared-window address.
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// Transpose of a 4x4 matrix of 2-bit cells (cell (r, c) at bit 8r + 2c).
// The planar layout stores a thread's IQ2_S / IQ3_S qh word transposed, so
// byte l holds the high index bits of subgroup l of all four groups. It is its
// own inverse.
__host__ __device__ __forceinline__ uint32_t qh_transpose(uint32_t w) {
    uint32_t t = ((w >> 12) ^ w) & 0x0000f0f0u;
    w ^= t ^ (t << 12);
    t = ((w >> 6) ^ w) & 0x00cc00ccu;
    w ^= t ^ (t << 6);
    return w;
}

// Sign words of the planar IQ2_S / IQ3_S layout. A GGUF sign word holds the
// sign bytes of a group's four 8-lane subgroups (bit 8l + i: subgroup l, lane
// i); the planar layout stores it transposed (bit 4i + l), so that the signs
// of subgroup l sit one nibble apart: a shift and a mask put them where the
// decoders need them, with no lookup. Four delta swaps rotate the five
// bit-index bits (p4 p3 p2 p1 p0 -> p2 p1 p0 p4 p3); sign_untranspose applies
// them in reverse order.
__host__ __device__ __forceinline__ uint32_t delta_swap(uint32_t w, uint32_t mask, int d) {
    const uint32_t t = ((w >> d) ^ w) & mask;
    return w ^ t ^ (t << d);
}
__host__ __device__ __forceinline__ uint32_t sign_transpose(uint32_t w) {
    w = delta_swap(w, 0x22222222u, 1);
    w = delta_swap(w, 0x0c0c0c0cu, 2);
    w = delta_swap(w, 0x00aa00aau, 7);
    return delta_swap(w, 0x0000ccccu, 14);
}
__host__ __device__ __forceinline__ uint32_t sign_untranspose(uint32_t w) {
    w = delta_swap(w, 0x0000ccccu, 14);
    w = delta_swap(w, 0x00aa00aau, 7);
    w = delta_swap(w, 0x0c0c0c0cu, 2);
    return delta_swap(w, 0x22222222u, 1);
}
// The signs of subgroup L of a transposed sign word at bit 4i + 2 (lane i),
// other bits unspecified: a shift by 2 - L.
template <int L>
__device__ __forceinline__ uint32_t signs_at2(uint32_t sgt) {
    if constexpr (L <= 2) return sgt << (2 - L);
    else return sgt >> (L - 2);
}

// 4x4 byte transpose: out[k] byte i = in[i] byte k.
__device__ __forceinline__ void transpose4(uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t& o0,
                                           uint32_t& o1, uint32_t& o2, uint32_t& o3) {
    uint32_t t0 = __byte_perm(a, b, 0x5140);
    uint32_t t1 = __byte_perm(a, b, 0x7362);
    uint32_t t2 = __byte_perm(c, d, 0x5140);
    uint32_t t3 = __byte_perm(c, d, 0x7362);
    o0 = __byte_perm(t0, t2, 0x5410);
    o1 = __byte_perm(t0, t2, 0x7632);
    o2 = __byte_perm(t1, t3, 0x5410);
    o3 = __byte_perm(t1, t3, 0x7632);
}

// ------------------------------------------------------- shared-memory tables
//
// Lookup tables are replicated 32 times, copy c living entirely in bank c
// (word address = entry * 32 + c). Lane l reads copy l, so a warp-wide lookup
// with arbitrary indices is one shared-memory wavefront.

constexpr int kIq2CodeEntries = 1024;  // IQ2_S grid as 8 code nibbles (0,1,2 = 8,25,43)
constexpr int kIq3GridEntries = 512;   // IQ3_S grid magnitudes, 4 bytes

constexpr int kIq2CodeBytes = kIq2CodeEntries * 32 * 4;  // 128 KiB
constexpr int kIq3GridBytes = kIq3GridEntries * 32 * 4;  // 64 KiB

// Replicated table images in global memory, built once per context from the
// codebooks of lbk_iq_tables.h (build_table_images). A kernel copies the
// images it needs into shared memory. (The signs need no table: see
// sign_transpose.)
struct Tables {
    const uint4* iq2_codes;  // kIq2CodeBytes
    const uint4* iq3_grid;   // kIq3GridBytes
};

__device__ __forceinline__ void copy_table(uint32_t* dst, const uint4* src, int bytes) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = __ldg(src + i);
}

__device__ __forceinline__ uint32_t iq2_code_of(uint64_t g) {
    uint32_t v = 0;
#pragma unroll
    for (int l = 0; l < 8; l++) {
        uint32_t m = (uint32_t)(g >> (8 * l)) & 0xff;
        uint32_t c = m == 8 ? 0u : (m == 25 ? 1u : 2u);
        v |= c << (4 * l);
    }
    return v;
}

// Copies the replicated images into shared memory; all threads participate.
__device__ __forceinline__ void fill_iq2_codes(uint32_t* tab, const Tables& t) { copy_table(tab, t.iq2_codes, kIq2CodeBytes); }
__device__ __forceinline__ void fill_iq3_grid(uint32_t* tab, const Tables& t) { copy_table(tab, t.iq3_grid, kIq3GridBytes); }

// Pools for IQ2_S signed-grid expansion through byte permutes: selector
// nibble c in {0,1,2} picks +8/+25/+43, c+4 picks the negated value.
constexpr uint32_t kIq2PoolPos = 0x002b1908u;
constexpr uint32_t kIq2PoolNeg = 0x00d5e7f8u;

// ------------------------------------------------------------------- exp
// exp for the sigmoid / SwiGLU stages: CUDA's double-precision exp rounded to
// f32, i.e. the correctly rounded f32 result except in vanishingly rare
// cases. The reference uses the platform libm expf (glibc's is also correctly
// rounded in all but rare cases); these stages are held to 1e-5 relative.
__device__ __forceinline__ float exp_f32(float v) { return (float)exp((double)v); }

// sigmoid, bridge-model-hy3/src/routing.rs:109-111
__device__ __forceinline__ float sigmoid_ref(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-v))); }

// SwiGLU of one lane, apply_swiglu (activation.rs:170-178)
__device__ __forceinline__ float swiglu_ref(float g, float u) {
    float act = __fdiv_rn(g, __fadd_rn(1.0f, exp_f32(-g)));
    return __fmul_rn(act, u);
}

// ------------------------------------------------------------ Q8_K quantizer

// Activations of one Q8_K block held by a warp: lane l owns lanes 8l..8l+7.
// Returns false (and writes nothing) when a value is non-finite.
// Restates quantize_row_q8_k_into (q8_k.rs:35-73) for one block:
//   first index of the largest |x| keeps its sign as `max`;
//   iscale = -127/max; q = min(nearest_int(iscale*x), 127);
//   16 group sums of 16 lanes; d = 1/iscale.
struct Q8Block {
    uint32_t q[2];      // this lane's 8 quants
    int32_t pair_sum;   // sum of this lane's 8 quants
    float d;            // block scale (all lanes)
};

__device__ __forceinline__ Q8Block quantize_q8k_warp(const float v[8], int lane) {
    // max-abs with ties to the first index: key = (|x| bits, ~index)
    unsigned long long key = 0ull;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint32_t ab = __float_as_uint(fabsf(v[i]));
        uint32_t idx = (uint32_t)(lane * 8 + i);
        unsigned long long k = ((unsigned long long)ab << 32) | (unsigned long long)(0xffffffffu - idx);
        key = k > key ? k : key;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    uint32_t amax_bits = (uint32_t)(key >> 32);
    uint32_t idx = 0xffffffffu - (uint32_t)(key & 0xffffffffull);
    Q8Block out;
    if (amax_bits == 0u) {
        out.q[0] = out.q[1] = 0u;
        out.pair_sum = 0;
        out.d = 0.0f;
        return out;
    }
    float mine = v[0];
#pragma unroll
    for (int i = 1; i < 8; i++)
        if ((int)(idx & 7) == i) mine = v[i];
    float maxv = __shfl_sync(0xffffffffu, mine, (int)(idx >> 3));
    float iscale = __fdiv_rn(-127.0f, maxv);
    int32_t s = 0;
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        int q = __float2int_rn(__fmul_rn(iscale, v[i]));
        q = q > 127 ? 127 : q;
        s += q;
        w[i >> 2] |= ((uint32_t)q & 0xffu) << (8 * (i & 3));
    }
    out.q[0] = w[0];
    out.q[1] = w[1];
    out.pair_sum = s;
    out.d = __fdiv_rn(1.0f, iscale);
    return out;
}

// Internal Q8_K block image used inside workspaces (never exposed): the same
// values as the 292-byte Q8_K block, with 16-byte aligned fields so a thread's
// half block is eight 16-byte loads:
//   qs int8[256] @0 | bsums int16[16] @256 | d f32 @288 | pad to 304
constexpr int kQ8IBytes = 304;

// Stores a warp's quantized block (see quantize_q8k_warp); `pair` is the
// lane-pair group sum (valid on even lanes).
__device__ __forceinline__ void store_q8i(uint8_t* blk, const Q8Block& q, int32_t pair, int lane) {
    uint2* qs = reinterpret_cast<uint2*>(blk);
    qs[lane] = make_uint2(q.q[0], q.q[1]);
    if ((lane & 1) == 0) reinterpret_cast<int16_t*>(blk + 256)[lane >> 1] = (int16_t)pair;
    if (lane == 0) *reinterpret_cast<float*>(blk + 288) = q.d;
}

// ------------------------------------------------------ activation registers

// A thread's HB of Q8_K activations: 128 int8 lanes as 32 words, in natural
// lane order for the IQ types and transposed per 32-lane sub-block for the
// K-quants (word 8j+l holds lanes l, l+8, l+16, l+24 of sub-block j).
struct ActHB {
    uint32_t w[32];
    float d;
    int32_t bsum[8];  // the HB's 8 Q8_K 16-lane group sums (K-quants only)
};

// Smem image of a Q8_K row: qs[K] int8 (16 B aligned), d[nb], bsums[nb*16].
struct ActSmem {
    const int8_t* qs;
    const float* d;
    const int16_t* bsums;
};

// The rest of load_act_hb once a.w holds the half block's 128 activation
// bytes in natural order: the K-quant transposition, d and the group sums.
template <bool kTransposed>
__device__ __forceinline__ void finish_act_hb(ActHB& a, const ActSmem& s, int block, int half, bool with_bsums) {
    if (kTransposed) {
        // sub-block j (32 lanes = words 8j..8j+7 in natural order):
        // out word l (l<4)  = byte l of words 8j+0, +2, +4, +6
        // out word l (l>=4) = byte l-4 of words 8j+1, +3, +5, +7
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t n[8];
#pragma unroll
            for (int i = 0; i < 8; i++) n[i] = a.w[8 * j + i];
            transpose4(n[0], n[2], n[4], n[6], a.w[8 * j + 0], a.w[8 * j + 1], a.w[8 * j + 2], a.w[8 * j + 3]);
            transpose4(n[1], n[3], n[5], n[7], a.w[8 * j + 4], a.w[8 * j + 5], a.w[8 * j + 6], a.w[8 * j + 7]);
        }
    }
    a.d = s.d[block];
    if (with_bsums) {
#pragma unroll
        for (int i = 0; i < 8; i++) a.bsum[i] = s.bsums[block * 16 + half * 8 + i];
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) a.bsum[i] = 0;
    }
}

template <bool kTransposed>
__device__ __forceinline__ void load_act_hb(ActHB& a, const ActSmem& s, int block, int half, bool with_bsums) {
    const uint4* src = reinterpret_cast<const uint4*>(s.qs + block * kQK + half * 128);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint4 v = src[i];
        a.w[4 * i + 0] = v.x;
        a.w[4 * i + 1] = v.y;
        a.w[4 * i + 2] = v.z;
        a.w[4 * i + 3] = v.w;
    }
    finish_act_hb<kTransposed>(a, s, block, half, with_bsums);
}

// ------------------------------------------------------------ HB weight data

// Field planes of the planar layout (bytes per block, in plane order).
//   IQ2_S: qs 32 | signs 32 | qh 8 | scales 8 | d 2
//   IQ3_S: qs 64 | signs 32 | qh 8 | scales 4 | d 2
//   Q4_K : qs 128 (lane-major) | scales 12 | dm 4
//   Q5_K : qs 128 (lane-major) | qh 32 (lane-major) | scales 12 | dm 4
// "lane-major" permutes the 32 bytes of each qs group g as
// new[4k+i] = old[k+8i] (k < 8, i < 4), so after nibble extraction a word
// holds four lanes of one lane class (index mod 8) of one sub-block.
struct MatrixRef {
    const uint8_t* data;
    uint64_t rows;
    int nb;  // blocks per row
};

__device__ __forceinline__ uint64_t blk_index(const MatrixRef& m, uint64_t row, int b) {
    return row * (uint64_t)m.nb + (uint64_t)b;
}

// Row stride of the planar layout: the GGUF row bytes rounded up to 16.
__host__ __device__ __forceinline__ constexpr uint32_t planar_row_bytes(int block_bytes, int nb) {
    return ((uint32_t)(nb * block_bytes) + 15u) & ~15u;
}
template <int T>
__device__ __forceinline__ const uint8_t* planar_row(const MatrixRef& m, uint64_t row) {
    return m.data + row * planar_row_bytes(TypeInfo<T>::kBlockBytes, m.nb);
}

struct Iq2HB {
    uint4 qs, sg;
    uint32_t qh, sc, d;
};
struct Iq3HB {
    uint4 qs0, qs1, sg;
    uint32_t qh, sc, d;
};
struct Q4HB {
    uint4 qs[4];
    uint32_t sc[3];
    uint32_t dm;
};
struct Q5HB {
    uint4 qs[4];
    uint4 qh[2];
    uint32_t sc[3];
    uint32_t dm;
};

template <int LAYOUT>
__device__ __forceinline__ void load_hb(Iq2HB& o, const MatrixRef& m, uint64_t row, int b, int h) {
    const uint64_t bi = blk_index(m, row, b);  // GGUF
    if (LAYOUT != LBK_LAYOUT_GGUF) {
        const uint8_t* base = planar_row<LBK_TYPE_IQ2_S>(m, row);
        const int nb = m.nb;
        o.qs = wld128<LAYOUT>(base + b * 32 + 16 * h);
        o.sg = wld128<LAYOUT>(base + nb * 32 + b * 32 + 16 * h);
        o.qh = wld32<LAYOUT>(base + nb * 64 + b * 8 + 4 * h);
        o.sc = wld32<LAYOUT>(base + nb * 72 + b * 8 + 4 * h);
        o.d = wld16<LAYOUT>(base + nb * 80 + b * 2);
    } else {
        const uint8_t* p = m.data + bi * 82;
        o.d = ldw_u16(p);
        o.qs = ldw_u128_a2(p + 2 + 16 * h);
        o.sg = ldw_u128_a2(p + 34 + 16 * h);
        o.sg = make_uint4(sign_transpose(o.sg.x), sign_transpose(o.sg.y), sign_transpose(o.sg.z), sign_transpose(o.sg.w));
        o.qh = qh_transpose(ldw_u32_a2(p + 66 + 4 * h));
        o.sc = ldw_u32_a2(p + 74 + 4 * h);
    }
}

template <int LAYOUT>
__device__ __forceinline__ void load_hb(Iq3HB& o, const MatrixRef& m, uint64_t row, int b, int h) {
    uint64_t bi = blk_index(m, row, b);
    if (LAYOUT != LBK_LAYOUT_GGUF) {
        const uint8_t* base = planar_row<LBK_TYPE_IQ3_S>(m, row);
        const int nb = m.nb;
        o.qs0 = wld128<LAYOUT>(base + b * 64 + 32 * h);
        o.qs1 = wld128<LAYOUT>(base + b * 64 + 32 * h + 16);
        o.sg = wld128<LAYOUT>(base + nb * 64 + b * 32 + 16 * h);
        o.qh = wld32<LAYOUT>(base + nb * 96 + b * 8 + 4 * h);
        o.sc = wld16<LAYOUT>(base + nb * 104 + b * 4 + 2 * h);
        o.d = wld16<LAYOUT>(base + nb * 108 + b * 2);
    } else {
        const uint8_t* p = m.data + bi * 110;
        o.d = ldw_u16(p);
        o.qs0 = ldw_u128_a2(p + 2 + 32 * h);
        o.qs1 = ldw_u128_a2(p + 2 + 32 * h + 16);
        o.qh = qh_transpose(ldw_u32_a2(p + 66 + 4 * h));
        o.sg = ldw_u128_a2(p + 74 + 16 * h);
        o.sg = make_uint4(sign_transpose(o.sg.x), sign_transpose(o.sg.y), sign_transpose(o.sg.z), sign_transpose(o.sg.w));
        o.sc = ldw_u16(p + 106 + 2 * h);
    }
}

// Half-block loads from a stage of planar rows in shared memory (same row
// stride as in global memory): the lane's byte offsets are fixed for a
// kernel, so they are computed once (stage_off) and every step is a handful
// of shared loads at constant offsets.
struct StageOff {
    uint32_t f0, f1, f2, f3, f4;
};

template <int T>
__device__ __forceinline__ StageOff stage_off(int nb, int sub, int b, int h) {
    const uint32_t r = (uint32_t)sub * planar_row_bytes(TypeInfo<T>::kBlockBytes, nb), n = (uint32_t)nb;
    StageOff o{};
    if constexpr (T == LBK_TYPE_IQ2_S) {
        o.f0 = r + b * 32 + 16 * h;            // qs
        o.f1 = r + n * 32 + b * 32 + 16 * h;   // signs
        o.f2 = r + n * 64 + b * 8 + 4 * h;     // qh
        o.f3 = r + n * 72 + b * 8 + 4 * h;     // scales
        o.f4 = r + n * 80 + b * 2;             // d
    } else if constexpr (T == LBK_TYPE_IQ3_S) {
        o.f0 = r + b * 64 + 32 * h;            // qs (two 16-byte words)
        o.f1 = r + n * 64 + b * 32 + 16 * h;   // signs
        o.f2 = r + n * 96 + b * 8 + 4 * h;     // qh
        o.f3 = r + n * 104 + b * 4 + 2 * h;    // scales
        o.f4 = r + n * 108 + b * 2;            // d
    } else if constexpr (T == LBK_TYPE_Q4_K) {
        o.f0 = r + b * 128 + 64 * h;           // qs (four 16-byte words)
        o.f1 = r + n * 128 + b * 12;           // scales
        o.f2 = r + n * 140 + b * 4;            // d, dmin
    } else {
        o.f0 = r + b * 128 + 64 * h;           // qs
        o.f1 = r + n * 128 + b * 32;           // qh
        o.f2 = r + n * 160 + b * 12;           // scales
        o.f3 = r + n * 172 + b * 4;            // d, dmin
    }
    return o;
}

__device__ __forceinline__ uint4 sld128(const uint8_t* s, uint32_t off) { return *reinterpret_cast<const uint4*>(s + off); }
__device__ __forceinline__ uint32_t sld32(const uint8_t* s, uint32_t off) { return *reinterpret_cast<const uint32_t*>(s + off); }
__device__ __forceinline__ uint32_t sld16(const uint8_t* s, uint32_t off) { return *reinterpret_cast<const uint16_t*>(s + off); }

__device__ __forceinline__ void load_stage(Iq2HB& o, const uint8_t* s, const StageOff& f) {
    o.qs = sld128(s, f.f0);
    o.sg = sld128(s, f.f1);
    o.qh = sld32(s, f.f2);
    o.sc = sld32(s, f.f3);
    o.d = sld16(s, f.f4);
}
__device__ __forceinline__ void load_stage(Iq3HB& o, const uint8_t* s, const StageOff& f) {
    o.qs0 = sld128(s, f.f0);
    o.qs1 = sld128(s, f.f0 + 16);
    o.sg = sld128(s, f.f1);
    o.qh = sld32(s, f.f2);
    o.sc = sld16(s, f.f3);
    o.d = sld16(s, f.f4);
}
__device__ __forceinline__ void load_stage(Q4HB& o, const uint8_t* s, const StageOff& f) {
#pragma unroll
    for (int i = 0; i < 4; i++) o.qs[i] = sld128(s, f.f0 + 16 * i);
    o.sc[0] = sld32(s, f.f1);
    o.sc[1] = sld32(s, f.f1 + 4);
    o.sc[2] = sld32(s, f.f1 + 8);
    o.dm = sld32(s, f.f2);
}
__device__ __forceinline__ void load_stage(Q5HB& o, const uint8_t* s, const StageOff& f) {
#pragma unroll
    for (int i = 0; i < 4; i++) o.qs[i] = sld128(s, f.f0 + 16 * i);
    o.qh[0] = sld128(s, f.f1);
    o.qh[1] = sld128(s, f.f1 + 16);
    o.sc[0] = sld32(s, f.f2);
    o.sc[1] = sld32(s, f.f2 + 4);
    o.sc[2] = sld32(s, f.f2 + 8);
    o.dm = sld32(s, f.f3);
}

// GGUF qs group (8 words, natural order) -> lane-major order.
__device__ __forceinline__ void lane_major8(uint32_t* w) {
    uint32_t n[8];
#pragma unroll
    for (int i = 0; i < 8; i++) n[i] = w[i];
    transpose4(n[0], n[2], n[4], n[6], w[0], w[1], w[2], w[3]);
    transpose4(n[1], n[3], n[5], n[7], w[4], w[5], w[6], w[7]);
}

template <int LAYOUT>
__device__ __forceinline__ void load_hb(Q4HB& o, const MatrixRef& m, uint64_t row, int b, int h) {
    uint64_t bi = blk_index(m, row, b);
    if (LAYOUT != LBK_LAYOUT_GGUF) {
        const uint8_t* base = planar_row<LBK_TYPE_Q4_K>(m, row);
        const int nb = m.nb;
#pragma unroll
        for (int i = 0; i < 4; i++) o.qs[i] = wld128<LAYOUT>(base + b * 128 + 64 * h + 16 * i);
        const uint8_t* s = base + nb * 128 + b * 12;
        o.sc[0] = wld32<LAYOUT>(s);
        o.sc[1] = wld32<LAYOUT>(s + 4);
        o.sc[2] = wld32<LAYOUT>(s + 8);
        o.dm = wld32<LAYOUT>(base + nb * 140 + b * 4);
    } else {
        const uint8_t* p = m.data + bi * 144;
        o.dm = ldw_u32(p);
        o.sc[0] = ldw_u32(p + 4);
        o.sc[1] = ldw_u32(p + 8);
        o.sc[2] = ldw_u32(p + 12);
#pragma unroll
        for (int g = 0; g < 2; g++) {
            uint4 a = ldw_u128(p + 16 + 64 * h + 32 * g);
            uint4 c = ldw_u128(p + 16 + 64 * h + 32 * g + 16);
            uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
            lane_major8(w);
            o.qs[2 * g] = make_uint4(w[0], w[1], w[2], w[3]);
            o.qs[2 * g + 1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
    }
}

template <int LAYOUT>
__device__ __forceinline__ void load_hb(Q5HB& o, const MatrixRef& m, uint64_t row, int b, int h) {
    uint64_t bi = blk_index(m, row, b);
    if (LAYOUT != LBK_LAYOUT_GGUF) {
        const uint8_t* base = planar_row<LBK_TYPE_Q5_K>(m, row);
        const int nb = m.nb;
#pragma unroll
        for (int i = 0; i < 4; i++) o.qs[i] = wld128<LAYOUT>(base + b * 128 + 64 * h + 16 * i);
        o.qh[0] = wld128<LAYOUT>(base + nb * 128 + b * 32);
        o.qh[1] = wld128<LAYOUT>(base + nb * 128 + b * 32 + 16);
        const uint8_t* s = base + nb * 160 + b * 12;
        o.sc[0] = wld32<LAYOUT>(s);
        o.sc[1] = wld32<LAYOUT>(s + 4);
        o.sc[2] = wld32<LAYOUT>(s + 8);
        o.dm = wld32<LAYOUT>(base + nb * 172 + b * 4);
    } else {
        const uint8_t* p = m.data + bi * 176;
        o.dm = ldw_u32(p);
        o.sc[0] = ldw_u32(p + 4);
        o.sc[1] = ldw_u32(p + 8);
        o.sc[2] = ldw_u32(p + 12);
        {
            uint4 a = ldw_u128(p + 16);
            uint4 c = ldw_u128(p + 32);
            uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
            lane_major8(w);
            o.qh[0] = make_uint4(w[0], w[1], w[2], w[3]);
            o.qh[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
#pragma unroll
        for (int g = 0; g < 2; g++) {
            uint4 a = ldw_u128(p + 48 + 64 * h + 32 * g);
            uint4 c = ldw_u128(p + 48 + 64 * h + 32 * g + 16);
            uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
            lane_major8(w);
            o.qs[2 * g] = make_uint4(w[0], w[1], w[2], w[3]);
            o.qs[2 * g + 1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
    }
}

// ------------------------------------------------------------ HB int dots

// Result of one HB: integer partial sums of its block plus the block scales.
struct IqPart {
    int32_t sum;
    uint32_t d;  // binary16 bits
};
struct KPart {
    int32_t lane[8];
    int32_t min_sum;
    uint32_t dm;  // d | dmin << 16 (binary16 bits)
};

// Selector of prmt() giving [byte `lo` of a, byte `hi` of b, 0, 0]: the two
// upper selector nibbles replicate the sign of b's byte `hi` (bit 3 set),
// which is zero because b's bytes hold 2-bit values.
__host__ __device__ constexpr uint32_t sel_idx(int lo, int hi) {
    return (uint32_t)(lo | ((4 + hi) << 4) | ((0xC + hi) << 8) | ((0xC + hi) << 12));
}

// dot_iq2_s (q8_k.rs:339-364) over groups 4h..4h+3 of one block.
// code_base is the shared-window address of this lane's copy of the
// replicated code table (entry e at base + 128 e). The qh word is the
// bit-transposed one (qh_transpose): byte l, bits 2g..2g+1 = high index bits
// of subgroup l of group g; the sign words are transposed too
// (sign_transpose). Per subgroup of 8 lanes: one permute builds the 10-bit
// index, one multiply-add its table address; the code nibbles plus the sign
// bits (shifted to bit 2 of each nibble) select signed grid bytes from a byte
// pool.
__device__ __forceinline__ IqPart dot_hb(const Iq2HB& w, const ActHB& a, uint32_t code_base) {
    int32_t total = 0;
    const uint32_t s1w = (w.sc & 0x0f0f0f0fu) * 2u + 0x01010101u;          // 1 + 2*(scale & 15), four groups
    const uint32_t s2w = ((w.sc >> 4) & 0x0f0f0f0fu) * 2u + 0x01010101u;   // 1 + 2*(scale >> 4)
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const uint32_t qsw = w32(w.qs, gi);
        const uint32_t sgw = w32(w.sg, gi);
        const uint32_t Q = (w.qh >> (2 * gi)) & 0x03030303u;  // byte l: high index bits of subgroup l
        const uint32_t sp[4] = {signs_at2<0>(sgw), signs_at2<1>(sgw), signs_at2<2>(sgw), signs_at2<3>(sgw)};
        int32_t part0 = 0, part1 = 0;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t idx = prmt(qsw, Q, sel_idx(l, l));
            const uint32_t code = lds32(idx * 128u + code_base);
            const uint32_t sel = code | (sp[l] & 0x44444444u);
            const uint32_t g0 = prmt(kIq2PoolPos, kIq2PoolNeg, sel);
            const uint32_t g1 = prmt(kIq2PoolPos, kIq2PoolNeg, sel >> 16);
            if (l < 2) {
                part0 = dp4a(g0, a.w[gi * 8 + 2 * l], part0);
                part0 = dp4a(g1, a.w[gi * 8 + 2 * l + 1], part0);
            } else {
                part1 = dp4a(g0, a.w[gi * 8 + 2 * l], part1);
                part1 = dp4a(g1, a.w[gi * 8 + 2 * l + 1], part1);
            }
        }
        const int32_t s1 = (int32_t)prmt(s1w, 0, 0x4440u | gi);
        const int32_t s2 = (int32_t)prmt(s2w, 0, 0x4440u | gi);
        total += s1 * part0 + s2 * part1;
    }
    IqPart r;
    r.sum = total;
    r.d = w.d;
    return r;
}

// dot_iq3_s (q8_k.rs:380-428) over groups 4h..4h+3 of one block. The signs
// are applied to the activations: na holds the negated activation words and
// a byte permute picks a or -a per lane, its selector (3210 plus bit 2 of
// each nibble from the transposed sign word) built by a shift and a mask.
// qh is bit-transposed as for IQ2_S: bit 0 of byte l holds the high bit of
// the first index of subgroup l, bit 1 of the second.
__device__ __forceinline__ IqPart dot_hb(const Iq3HB& w, const ActHB& a, const uint32_t* na, uint32_t grid_base) {
    int32_t total = 0;
    // pair scales: bytes [lo0, lo1, hi0, hi1] -> 1 + 2*nibble; group gi uses byte {0,2,1,3}[gi]
    const uint32_t st = (w.sc & 0x0f0fu) | ((w.sc & 0xf0f0u) << 12);
    const uint32_t sw = st * 2u + 0x01010101u;
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const uint32_t qa = gi < 2 ? w32(w.qs0, gi * 2) : w32(w.qs1, (gi - 2) * 2);
        const uint32_t qb = gi < 2 ? w32(w.qs0, gi * 2 + 1) : w32(w.qs1, (gi - 2) * 2 + 1);
        const uint32_t sgw = w32(w.sg, gi);
        const uint32_t Q = (w.qh >> (2 * gi)) & 0x03030303u;
        const uint32_t Q1 = Q & 0x01010101u;          // high bit of the first index
        const uint32_t Q2 = (Q >> 1) & 0x01010101u;   // high bit of the second index
        const uint32_t sp[4] = {signs_at2<0>(sgw), signs_at2<1>(sgw), signs_at2<2>(sgw), signs_at2<3>(sgw)};
        int32_t gsum = 0;
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t q2 = l < 2 ? qa : qb;
            const uint32_t i1 = prmt(q2, Q1, sel_idx(2 * (l & 1), l));
            const uint32_t i2 = prmt(q2, Q2, sel_idx(2 * (l & 1) + 1, l));
            const uint32_t g1 = lds32(i1 * 128u + grid_base);
            const uint32_t g2 = lds32(i2 * 128u + grid_base);
            const uint32_t slo = (sp[l] & 0x4444u) | 0x3210u;            // lanes 0-3: sign bits 0-3
            const uint32_t shi = ((sp[l] >> 16) & 0x4444u) | 0x3210u;    // lanes 4-7: sign bits 4-7
            const int wi = gi * 8 + 2 * l;
            const uint32_t a1 = prmt(a.w[wi], na[wi], slo);
            const uint32_t a2 = prmt(a.w[wi + 1], na[wi + 1], shi);
            gsum = dp4a(g1, a1, gsum);
            gsum = dp4a(g2, a2, gsum);
        }
        const int32_t scale = (int32_t)prmt(sw, 0, 0x4440u | (uint32_t)((gi & 1) * 2 + (gi >> 1)));
        total += gsum * scale;
    }
    IqPart r;
    r.sum = total;
    r.d = w.d;
    return r;
}

// scale_min (k_quants.rs:231-240) from three little-endian words of scales[12].
__device__ __forceinline__ void scale_min_dev(const uint32_t sc[3], int j, int32_t& s, int32_t& m) {
    auto byte = [&](int i) -> uint32_t { return (sc[i >> 2] >> (8 * (i & 3))) & 0xffu; };
    if (j < 4) {
        s = (int32_t)(byte(j) & 0x3f);
        m = (int32_t)(byte(j + 4) & 0x3f);
    } else {
        s = (int32_t)((byte(j + 4) & 0x0f) | ((byte(j - 4) >> 6) << 4));
        m = (int32_t)((byte(j + 4) >> 4) | ((byte(j) >> 6) << 4));
    }
}

// dot_q4_or_q5_k (q8_k.rs:257-312) over sub-blocks 4h..4h+3 of one block.
template <bool kQ5>
__device__ __forceinline__ KPart dot_hb_k(const uint4* qs, const uint4* qh, const uint32_t sc[3], uint32_t dm,
                                          const ActHB& a, int h) {
    KPart r;
#pragma unroll
    for (int l = 0; l < 8; l++) r.lane[l] = 0;
    int32_t ms = 0;
#pragma unroll
    for (int gg = 0; gg < 2; gg++) {  // qs group g = 2h + gg covers sub-blocks 2g (lo) and 2g+1 (hi)
        int g = 2 * h + gg;
        int32_t s_lo, m_lo, s_hi, m_hi;
        scale_min_dev(sc, 2 * g, s_lo, m_lo);
        scale_min_dev(sc, 2 * g + 1, s_hi, m_hi);
        // Q8_K group sums of the 16-lane groups of these two sub-blocks
        ms += (a.bsum[4 * gg + 0] + a.bsum[4 * gg + 1]) * m_lo;
        ms += (a.bsum[4 * gg + 2] + a.bsum[4 * gg + 3]) * m_hi;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            uint32_t q = w32(qs[2 * gg + (k >> 2)], k & 3);
            uint32_t lo = q & 0x0f0f0f0fu;
            uint32_t hi = (q >> 4) & 0x0f0f0f0fu;
            if (kQ5) {
                uint32_t hb = w32(qh[k >> 2], k & 3);
                lo |= ((hb >> (2 * g)) & 0x01010101u) << 4;
                hi |= ((hb >> (2 * g + 1)) & 0x01010101u) << 4;
            }
            // act word for sub-block (4h + 2gg [+1]) lane k: index 8*(2gg [+1]) + k
            int32_t plo = dp4a(lo, a.w[8 * (2 * gg) + k], 0);
            int32_t phi = dp4a(hi, a.w[8 * (2 * gg + 1) + k], 0);
            r.lane[k] += s_lo * plo + s_hi * phi;
        }
    }
    r.min_sum = ms;
    r.dm = dm;
    return r;
}

__device__ __forceinline__ KPart dot_hb(const Q4HB& w, const ActHB& a, int h) {
    return dot_hb_k<false>(w.qs, nullptr, w.sc, w.dm, a, h);
}
__device__ __forceinline__ KPart dot_hb(const Q5HB& w, const ActHB& a, int h) {
    return dot_hb_k<true>(w.qs, w.qh, w.sc, w.dm, a, h);
}

// ------------------------------------------------ decode once, dot many
// For several tokens on the same weights (a grouped expert): each 32-weight
// group of a half block is decoded once into signed int8 words, in the
// activation word order, and dotted at once with the activations of every
// pair of the group (only one group's 8 decoded words are live). The integer
// sums are those of dot_hb -- the same products, summed in another order --
// so every block sum is identical.

// Byte-wise negation of four grid magnitudes in [1, 127]: ~g + 1 per byte
// never carries into the next byte.
__device__ __forceinline__ uint32_t neg4_nonzero(uint32_t g) { return ~g + 0x01010101u; }

// Activations of the pairs of a group, as words gi*8 .. gi*8+7 (lo: the
// first four) of pair p's half block held in registers.
struct ActReg {
    const ActHB* a;
    __device__ __forceinline__ void operator()(int p, int gi, uint4& lo, uint4& hi) const {
        lo = make_uint4(a[p].w[gi * 8 + 0], a[p].w[gi * 8 + 1], a[p].w[gi * 8 + 2], a[p].w[gi * 8 + 3]);
        hi = make_uint4(a[p].w[gi * 8 + 4], a[p].w[gi * 8 + 5], a[p].w[gi * 8 + 6], a[p].w[gi * 8 + 7]);
    }
};

// IQ2_S (dot_iq2_s, q8_k.rs:339-364) over groups 4h..4h+3 for pairs p < n:
// tot[p] = the half block's integer sum against pair p's activations.
// kStride: bytes between table entries (the lane's copy at base).
template <int G, int kStride, class Act>
__device__ __forceinline__ void dot_hb_multi(const Iq2HB& w, const Act& act, uint32_t n, uint32_t code_base,
                                             int32_t* tot) {
    const uint32_t s1w = (w.sc & 0x0f0f0f0fu) * 2u + 0x01010101u;
    const uint32_t s2w = ((w.sc >> 4) & 0x0f0f0f0fu) * 2u + 0x01010101u;
#pragma unroll
    for (int p = 0; p < G; p++) tot[p] = 0;
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const uint32_t qsw = w32(w.qs, gi);
        const uint32_t sgw = w32(w.sg, gi);
        const uint32_t Q = (w.qh >> (2 * gi)) & 0x03030303u;
        const uint32_t sp[4] = {signs_at2<0>(sgw), signs_at2<1>(sgw), signs_at2<2>(sgw), signs_at2<3>(sgw)};
        uint32_t wd[8];
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t code = lds32(prmt(qsw, Q, sel_idx(l, l)) * (uint32_t)kStride + code_base);
            const uint32_t sel = code | (sp[l] & 0x44444444u);
            wd[2 * l] = prmt(kIq2PoolPos, kIq2PoolNeg, sel);
            wd[2 * l + 1] = prmt(kIq2PoolPos, kIq2PoolNeg, sel >> 16);
        }
        const int32_t s1 = (int32_t)prmt(s1w, 0, 0x4440u | gi);
        const int32_t s2 = (int32_t)prmt(s2w, 0, 0x4440u | gi);
#pragma unroll
        for (int p = 0; p < G; p++) {
            if ((uint32_t)p < n) {
                uint4 lo, hi;
                act(p, gi, lo, hi);
                int32_t p0 = dp4a(wd[0], lo.x, 0), p1 = dp4a(wd[4], hi.x, 0);
                p0 = dp4a(wd[1], lo.y, p0);
                p1 = dp4a(wd[5], hi.y, p1);
                p0 = dp4a(wd[2], lo.z, p0);
                p1 = dp4a(wd[6], hi.z, p1);
                p0 = dp4a(wd[3], lo.w, p0);
                p1 = dp4a(wd[7], hi.w, p1);
                tot[p] += s1 * p0 + s2 * p1;
            }
        }
    }
}

// IQ3_S (dot_iq3_s, q8_k.rs:380-428): the grid bytes with the sign bits
// applied to the weights (byte-wise g or -g selection with dot_hb's
// selectors, which apply them to the activations: the same products).
template <int G, int kStride, class Act>
__device__ __forceinline__ void dot_hb_multi(const Iq3HB& w, const Act& act, uint32_t n, uint32_t grid_base,
                                             int32_t* tot) {
    const uint32_t st = (w.sc & 0x0f0fu) | ((w.sc & 0xf0f0u) << 12);
    const uint32_t sw = st * 2u + 0x01010101u;
#pragma unroll
    for (int p = 0; p < G; p++) tot[p] = 0;
#pragma unroll
    for (int gi = 0; gi < 4; gi++) {
        const uint32_t qa = gi < 2 ? w32(w.qs0, gi * 2) : w32(w.qs1, (gi - 2) * 2);
        const uint32_t qb = gi < 2 ? w32(w.qs0, gi * 2 + 1) : w32(w.qs1, (gi - 2) * 2 + 1);
        const uint32_t sgw = w32(w.sg, gi);
        const uint32_t Q = (w.qh >> (2 * gi)) & 0x03030303u;
        const uint32_t Q1 = Q & 0x01010101u;
        const uint32_t Q2 = (Q >> 1) & 0x01010101u;
        const uint32_t sp[4] = {signs_at2<0>(sgw), signs_at2<1>(sgw), signs_at2<2>(sgw), signs_at2<3>(sgw)};
        uint32_t wd[8];
#pragma unroll
        for (int l = 0; l < 4; l++) {
            const uint32_t q2 = l < 2 ? qa : qb;
            const uint32_t g1 = lds32(prmt(q2, Q1, sel_idx(2 * (l & 1), l)) * (uint32_t)kStride + grid_base);
            const uint32_t g2 = lds32(prmt(q2, Q2, sel_idx(2 * (l & 1) + 1, l)) * (uint32_t)kStride + grid_base);
            const uint32_t slo = (sp[l] & 0x4444u) | 0x3210u;
            const uint32_t shi = ((sp[l] >> 16) & 0x4444u) | 0x3210u;
            wd[2 * l] = prmt(g1, neg4_nonzero(g1), slo);
            wd[2 * l + 1] = prmt(g2, neg4_nonzero(g2), shi);
        }
        const int32_t scale = (int32_t)prmt(sw, 0, 0x4440u | (uint32_t)((gi & 1) * 2 + (gi >> 1)));
#pragma unroll
        for (int p = 0; p < G; p++) {
            if ((uint32_t)p < n) {
                uint4 lo, hi;
                act(p, gi, lo, hi);
                int32_t g = dp4a(wd[0], lo.x, 0);
                g = dp4a(wd[1], lo.y, g);
                g = dp4a(wd[2], lo.z, g);
                g = dp4a(wd[3], lo.w, g);
                g = dp4a(wd[4], hi.x, g);
                g = dp4a(wd[5], hi.y, g);
                g = dp4a(wd[6], hi.z, g);
                g = dp4a(wd[7], hi.w, g);
                tot[p] += g * scale;
            }
        }
    }
}

// ------------------------------------------------------------ block products
// The per-block f32 products of the reference tails, computed by the thread
// that holds half 0 after adding half 1's integers (shfl_xor 1).

__device__ __forceinline__ float iq_block_product(const IqPart& p, float dx) {
    float scale = __fmul_rn(h2f(p.d), dx);
    return __fmul_rn(scale, __int2float_rn(p.sum));
}

// The nine products of dot_q4_or_q5_k's per-block tail (q8_k.rs:314-320).
__device__ __forceinline__ void k_block_products(const KPart& p, float dx, float out[9]) {
    float scale = __fmul_rn(h2f(p.dm & 0xffffu), dx);
#pragma unroll
    for (int l = 0; l < 8; l++) out[l] = __fmul_rn(scale, __int2float_rn(p.lane[l]));
    float mscale = __fmul_rn(h2f(p.dm >> 16), dx);
    out[8] = __fmul_rn(mscale, __int2float_rn(p.min_sum));
}

// Sequential per-row tails: products for blocks 0..nb-1 at stride `stride`.
__device__ __forceinline__ float iq_tail(const float* prod, int nb, int stride, bool iq2) {
    float sum = 0.0f;
    for (int b = 0; b < nb; b++) sum = __fadd_rn(sum, prod[b * stride]);
    return iq2 ? __fmul_rn(0.125f, sum) : sum;
}

__device__ __forceinline__ float k_tail(const float* prod, int nb, int stride) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sum = 0.0f;
    for (int b = 0; b < nb; b++) {
#pragma unroll
        for (int l = 0; l < 8; l++) sums[l] = __fadd_rn(sums[l], prod[b * stride + l]);
        sum = __fsub_rn(sum, prod[b * stride + 8]);
    }
#pragma unroll
    for (int l = 0; l < 8; l++) sum = __fadd_rn(sum, sums[l]);
    return sum;
}

}  // namespace lbk
