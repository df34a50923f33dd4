// ep.cu -- expert-parallel exchange over peer memory (NVLink), no host round trip.
//
// Every rank owns one exchange buffer, mapped into every other rank of the
// node (CUDA IPC, plain peer loads and stores; no multicast):
//   [routing: cap * k lbk_routed][control block: EpControl, 512 bytes]
//   [Q8_K images: cap * q8b][routed dots: cap * k * H f32]
// A layer step, with no collective and no host involvement:
//   publish  the home rank routes its tokens into its own buffer, then raises
//            its step number and releases `published` = step;
//   gather   each rank waits until every buffer is published for this step,
//            then copies the (token, slot) pairs routed to its experts -- their
//            images over NVLink into a local item list, the count kept on the
//            device (zero at the start of a step: the scatter resets it);
//   (items)  the item kernels read the count on the device;
//   scatter  each item's row dots go straight into the home rank's buffer at
//            routed_dots[t * k + j]; the scatter's last CTA then releases
//            done[rank] = step in every buffer;
//   combine  the home rank waits until done[r] = step for every rank r and
//            adds the dots in ascending expert ID (the one-GPU order).
// Only the bytes the pairs need cross NVLink. A buffer is not overwritten
// while a peer still reads it: a rank publishes step s + 1 only after its
// combine of step s saw every rank's scatter of step s, which follows that
// rank's gather of step s. Every wait is bounded (LBK_TIMEOUT through the
// status word; the kernels still finish).

#include "lbk_kernels.h"
#include "lbk_moe.h"

namespace lbk {

namespace {

constexpr int kGatherWarps = 8;

__device__ __forceinline__ const EpControl* ctl_of(const uint8_t* buf, uint64_t off) {
    return reinterpret_cast<const EpControl*>(buf + off);
}

// Wait until `flag` reaches `step` (wrapping compare), at most `polls` polls;
// none once an error is recorded (a rank that stopped would otherwise cost
// every later wait its full limit).
__device__ __forceinline__ bool wait_step(const uint32_t* flag, uint32_t step, uint32_t polls, const DeviceStatus* st) {
    for (uint32_t i = 0; i < polls; i++) {
        if ((int32_t)(ld_acquire_sys(flag) - step) >= 0) return true;
        if ((i & 255u) == 0u && status_set(st)) return false;
        __nanosleep(64);
    }
    return false;
}

// A Q8_K image in 16-byte words per lane: at most kImgWords per lane (hidden
// 4096: 292 words over 32 lanes), all loads in flight before any store.
constexpr int kImgWords = 10;

// One warp per (rank, token): the token's k routing entries; each entry whose
// expert is local becomes an item (slot from an atomic counter). The warp
// loads the token's image once (all its words in flight) and stores it to
// every item of the token. Warp 0 of every CTA first waits for every rank's
// publication of this step.
__global__ void __launch_bounds__(kGatherWarps * 32) ep_gather_kernel(EpGatherArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ int s_ok;
    if (warp == 0) {
        const uint32_t step = __ldcg(&ctl_of(a.peers[a.rank], a.off_ctl)->step);
        bool ok = true;
        for (uint32_t r = lane; r < a.world; r += 32)
            ok &= wait_step(&ctl_of(a.peers[r], a.off_ctl)->published, step, a.polls, a.status);
        ok = __all_sync(0xffffffffu, ok);
        if (lane == 0) {
            s_ok = ok;
            if (!ok) report(a.status, LBK_TIMEOUT, 8, step);
        }
    }
    __syncthreads();  // the flags' acquire before every warp's reads of the buffers
    if (!s_ok) return;
    const uint32_t words = a.q8b / 16;  // <= 32 * kImgWords (host-checked)
    const uint64_t pairs_total = (uint64_t)a.world * a.cap;
    for (uint64_t w = (uint64_t)blockIdx.x * kGatherWarps + warp; w < pairs_total;
         w += (uint64_t)gridDim.x * kGatherWarps) {
        const uint32_t s = (uint32_t)(w / a.cap), t = (uint32_t)(w % a.cap);
        const uint8_t* buf = a.peers[s];
        const uint32_t ntok = __ldcg(&ctl_of(buf, a.off_ctl)->tokens);
        if (t >= ntok) continue;
        const lbk_routed* routing = reinterpret_cast<const lbk_routed*>(buf) + (uint64_t)t * a.k;
        uint32_t eid = 0;
        bool mine = false;  // slot `lane`'s expert is local
        if ((uint32_t)lane < a.k) {
            eid = __ldcg(reinterpret_cast<const uint32_t*>(routing + lane));
            mine = eid >= a.first && eid < a.first + a.count;
        }
        const uint32_t mask = __ballot_sync(0xffffffffu, mine);
        if (mask == 0u) continue;
        const uint4* src = reinterpret_cast<const uint4*>(buf + a.off_q8 + (uint64_t)t * a.q8b);
        uint4 v[kImgWords];
#pragma unroll
        for (int q = 0; q < kImgWords; q++)
            if ((uint32_t)(lane + 32 * q) < words) v[q] = __ldcg(src + lane + 32 * q);
        // the token's items take consecutive slots; slot order within the token follows j
        uint32_t base = 0;
        if (lane == 0) base = atomicAdd(a.d_count, (uint32_t)__popc(mask));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (mine) {
            const uint32_t slot = base + (uint32_t)__popc(mask & ((1u << lane) - 1u));
            if (slot < a.cap_items) {  // cannot fail: cap_items = world * cap * k
                a.items[slot] = lbk_routed{eid - a.first, 0.0f};
                a.returns[slot] = make_uint2(s, t * a.k + (uint32_t)lane);
            }
        }
        for (uint32_t m = mask; m; m &= m - 1) {
            const uint32_t slot = base + (uint32_t)__popc(mask & ((1u << (__ffs(m) - 1)) - 1u));
            if (slot >= a.cap_items) continue;
            uint4* dst = reinterpret_cast<uint4*>(a.q8_items + (uint64_t)slot * a.q8b);
#pragma unroll
            for (int q = 0; q < kImgWords; q++)
                if ((uint32_t)(lane + 32 * q) < words) dst[lane + 32 * q] = v[q];
        }
    }
}

// One CTA per item (grid-stride): its H row dots into the home buffer, each
// thread's words loaded before any is stored. The last CTA to finish resets
// the item count for the next step and releases done[rank] = step in every
// rank's buffer.
constexpr int kScatterThreads = 256;
constexpr int kScatterWords = 4;  // hidden 4096: 1024 float4 over 256 threads
__global__ void __launch_bounds__(kScatterThreads) ep_scatter_kernel(EpScatterArgs a) {
    EpControl* me = reinterpret_cast<EpControl*>(a.peers[a.rank] + a.off_ctl);
    const uint32_t step = __ldcg(&me->step);
    const uint32_t n = __ldcg(a.d_count);
    const uint32_t words = a.hidden / 4;  // <= kScatterThreads * kScatterWords (host-checked)
    for (uint32_t i = blockIdx.x; i < n && i < a.cap_items; i += gridDim.x) {
        const uint2 r = a.returns[i];
        const float4* __restrict__ src = reinterpret_cast<const float4*>(a.dots + (uint64_t)i * a.hidden);
        float4* dst = reinterpret_cast<float4*>(a.peers[r.x] + a.off_dots) + (uint64_t)r.y * words;
        float4 v[kScatterWords];
#pragma unroll
        for (int q = 0; q < kScatterWords; q++)
            if (threadIdx.x + kScatterThreads * q < words) v[q] = __ldcg(src + threadIdx.x + kScatterThreads * q);
#pragma unroll
        for (int q = 0; q < kScatterWords; q++)
            if (threadIdx.x + kScatterThreads * q < words) dst[threadIdx.x + kScatterThreads * q] = v[q];
    }
    __threadfence_system();  // this thread's peer stores before the CTA's arrival
    __syncthreads();
    __shared__ bool s_last;
    if (threadIdx.x == 0) s_last = atomicAdd(&me->scatter_ctas, 1u) + 1u == gridDim.x;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();  // the other CTAs' stores (seen through their arrivals) before the flags
    if (threadIdx.x == 0) {
        me->scatter_ctas = 0u;  // ready for the next step
        *a.d_count = 0u;        // every CTA has read it
    }
    for (uint32_t r = threadIdx.x; r < a.world; r += blockDim.x) {
        EpControl* c = reinterpret_cast<EpControl*>(a.peers[r] + a.off_ctl);
        st_release_sys(&c->done[a.rank], step);
    }
}

// Items returned in place by the down kernels (their rows already fenced):
// reset the item count and release done[rank] = step in every buffer.
__global__ void ep_signal_kernel(EpScatterArgs a) {
    EpControl* me = reinterpret_cast<EpControl*>(a.peers[a.rank] + a.off_ctl);
    const uint32_t step = __ldcg(&me->step);
    if (threadIdx.x == 0) *a.d_count = 0u;
    __threadfence_system();
    for (uint32_t r = threadIdx.x; r < a.world; r += blockDim.x) {
        EpControl* c = reinterpret_cast<EpControl*>(a.peers[r] + a.off_ctl);
        st_release_sys(&c->done[a.rank], step);
    }
}

// Raise this rank's step number; store the token count; publish.
__global__ void ep_publish_kernel(EpControl* ctl, uint32_t tokens) {
    const uint32_t step = ctl->step + 1u;
    ctl->step = step;
    ctl->tokens = tokens;
    st_release_sys(&ctl->published, step);
}

}  // namespace

cudaError_t launch_ep_gather(const EpGatherArgs& a, int sm_count, cudaStream_t stream) {
    if (a.q8b % 16 != 0 || a.q8b / 16 > 32u * kImgWords) return cudaErrorInvalidValue;
    const uint64_t warps = (uint64_t)a.world * a.cap;
    uint64_t grid = (warps + kGatherWarps - 1) / kGatherWarps;
    if (grid > (uint64_t)sm_count * 4) grid = (uint64_t)sm_count * 4;
    if (grid < 1) grid = 1;
    ep_gather_kernel<<<(unsigned)grid, kGatherWarps * 32, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_scatter(const EpScatterArgs& a, int sm_count, cudaStream_t stream) {
    if (a.hidden % 4 != 0 || a.hidden / 4 > (uint32_t)(kScatterThreads * kScatterWords)) return cudaErrorInvalidValue;
    uint64_t grid = a.cap_items < (uint64_t)sm_count * 4 ? a.cap_items : (uint64_t)sm_count * 4;
    if (grid < 1) grid = 1;
    ep_scatter_kernel<<<(unsigned)grid, kScatterThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_signal(const EpScatterArgs& a, cudaStream_t stream) {
    ep_signal_kernel<<<1, 64, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_publish(EpControl* ctl, uint32_t tokens, cudaStream_t stream) {
    ep_publish_kernel<<<1, 1, 0, stream>>>(ctl, tokens);
    return cudaGetLastError();
}

}  // namespace lbk
