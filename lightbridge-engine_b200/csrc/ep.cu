// ep.cu -- expert-parallel exchange over peer memory (NVLink), no host round trip.
//
// Every rank owns one exchange buffer, mapped into every other rank of the
// node (CUDA IPC, plain peer loads and stores; no multicast):
//   [routing: cap * k lbk_routed][tokens: u32, padded to 256]
//   [Q8_K images: cap * q8b][routed dots: cap * k * H f32]
// A layer step: the home rank routes its tokens into its own buffer
// (routing, images, token count); after a barrier, each rank gathers from
// every buffer the (token, slot) pairs routed to its experts -- their images
// copied over NVLink into a local item list, the count kept on the device;
// computes them (the item kernels read the count on the device); scatters
// each item's row dots straight into the home rank's buffer at
// routed_dots[t * k + j]; after a second barrier the home rank combines in
// ascending expert ID, so no size exchange and no device-to-host read is
// needed, and only the bytes the pairs need cross NVLink.

#include "lbk_kernels.h"
#include "lbk_moe.h"

namespace lbk {

namespace {

constexpr int kGatherWarps = 8;

// One warp per (rank, token): the token's k routing entries; each entry whose
// expert is local becomes an item (slot from an atomic counter), its image
// copied from the home buffer in 16-byte words.
__global__ void __launch_bounds__(kGatherWarps * 32) ep_gather_kernel(EpGatherArgs a) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t pairs_total = (uint64_t)a.world * a.cap;
    for (uint64_t w = (uint64_t)blockIdx.x * kGatherWarps + warp; w < pairs_total;
         w += (uint64_t)gridDim.x * kGatherWarps) {
        const uint32_t s = (uint32_t)(w / a.cap), t = (uint32_t)(w % a.cap);
        const uint8_t* buf = a.peers[s];
        const uint32_t ntok = __ldcg(reinterpret_cast<const uint32_t*>(buf + a.off_ntok));
        if (t >= ntok) continue;
        const lbk_routed* routing = reinterpret_cast<const lbk_routed*>(buf) + (uint64_t)t * a.k;
        uint32_t mine = 0;  // bit j: slot j's expert is local
        uint32_t eid = 0;
        if ((uint32_t)lane < a.k) {
            eid = __ldcg(reinterpret_cast<const uint32_t*>(routing + lane));
            mine = eid >= a.first && eid < a.first + a.count ? 1u : 0u;
        }
        uint32_t mask = __ballot_sync(0xffffffffu, mine != 0u);
        while (mask) {
            const int j = __ffs(mask) - 1;
            mask &= mask - 1;
            const uint32_t e = __shfl_sync(0xffffffffu, eid, j);
            uint32_t slot = 0;
            if (lane == 0) slot = atomicAdd(a.d_count, 1u);
            slot = __shfl_sync(0xffffffffu, slot, 0);
            if (slot >= a.cap_items) continue;  // cannot happen: cap_items = world * cap * k
            if (lane == 0) {
                a.items[slot] = lbk_routed{e - a.first, 0.0f};
                a.returns[slot] = make_uint2(s, t * a.k + (uint32_t)j);
            }
            const uint4* src = reinterpret_cast<const uint4*>(buf + a.off_q8 + (uint64_t)t * a.q8b);
            uint4* dst = reinterpret_cast<uint4*>(a.q8_items + (uint64_t)slot * a.q8b);
            for (uint32_t i = lane; i < a.q8b / 16; i += 32) dst[i] = __ldcg(src + i);
        }
    }
}

// One CTA per item (grid-stride): its H row dots into the home buffer.
__global__ void __launch_bounds__(256) ep_scatter_kernel(EpScatterArgs a) {
    const uint32_t n = __ldcg(a.d_count);
    for (uint32_t i = blockIdx.x; i < n && i < a.cap_items; i += gridDim.x) {
        const uint2 r = a.returns[i];
        const float4* src = reinterpret_cast<const float4*>(a.dots + (uint64_t)i * a.hidden);
        float4* dst = reinterpret_cast<float4*>(a.peers[r.x] + a.off_dots) + (uint64_t)r.y * (a.hidden / 4);
        for (uint32_t q = threadIdx.x; q < a.hidden / 4; q += blockDim.x) dst[q] = __ldcg(src + q);
    }
    __threadfence_system();  // the peer stores are visible before this grid is seen complete
}

__global__ void ep_set_tokens_kernel(uint32_t* p, uint32_t v) { *p = v; }

}  // namespace

cudaError_t launch_ep_gather(const EpGatherArgs& a, int sm_count, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(a.d_count, 0, 4, stream);
    if (e != cudaSuccess) return e;
    const uint64_t warps = (uint64_t)a.world * a.cap;
    uint64_t grid = (warps + kGatherWarps - 1) / kGatherWarps;
    if (grid > (uint64_t)sm_count * 4) grid = (uint64_t)sm_count * 4;
    if (grid < 1) grid = 1;
    ep_gather_kernel<<<(unsigned)grid, kGatherWarps * 32, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_scatter(const EpScatterArgs& a, int sm_count, cudaStream_t stream) {
    uint64_t grid = a.cap_items < (uint64_t)sm_count * 4 ? a.cap_items : (uint64_t)sm_count * 4;
    if (grid < 1) grid = 1;
    ep_scatter_kernel<<<(unsigned)grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_ep_set_tokens(uint32_t* p, uint32_t v, cudaStream_t stream) {
    ep_set_tokens_kernel<<<1, 1, 0, stream>>>(p, v);
    return cudaGetLastError();
}

}  // namespace lbk
