// lbk_moe.h -- launch interface of the fused MoE kernels (moe.cu).
#pragma once

#include "lbk_kernels.h"

namespace lbk {

constexpr int kMoeGateUpWarps = 8;   // warps per gate/up CTA (one CTA per SM)
constexpr int kMoeDownMaxSlots = 9;  // routed top-k + shared, one warp each
constexpr int kMoeGateUpTmaWarps = 16;  // warps per bulk-copy-staged gate/up CTA

struct MoeGateUpArgs {
    uint64_t hidden, ffn;
    int nb_h, nb_f;
    int tpr_h;                       // threads per row over the hidden width
    uint64_t tokens;
    uint64_t k;                      // routed experts per token
    uint64_t experts;
    const uint8_t* const* gate;      // [experts] planar matrices
    const uint8_t* const* up;
    const uint8_t* sgate;            // shared expert
    const uint8_t* sup;
    const lbk_routed* routed;        // [tokens][k]
    const uint8_t* q8x;              // [tokens][nb_h][292]
    float* h;                        // [tokens][k+1][ffn]
    uint8_t* hq;                     // [tokens][k+1][nb_f][292]
    unsigned int* counters;          // [tokens][k+1][nb_f], zero between launches
    uint64_t chunk_r, chunk_s;       // rows per warp (routed / shared slot)
    uint64_t chunks_r, chunks_s;     // chunks per slot
    int bmax_iq, bmax_k;             // rows per tail batch
    uint64_t prod_floats;            // per-warp product buffer
    uint64_t chain_floats;           // per-warp chain + result buffer (>= 9*dots + 64)
    // single-token decode: finish the router here (see router_fused_kernel's defer)
    int defer_topk;
    const float* partials;           // [experts][chunks]
    uint64_t chunks;
    const float* bias;
    float weight_scale;
    lbk_routed* routed_store;        // CTA 0 writes the routing here
    // bulk-copy-staged kernel: CTAs [0, routed_ctas) stream routed slots, the rest the shared expert
    // (no CTA does when has_shared is 0)
    uint32_t routed_ctas;
    int has_shared;
    // down matrices of the layer, prefetched into L2 once the routing is known
    // (null: no prefetch); row strides of the planar down matrices
    const uint8_t* const* down;
    const uint8_t* sdown;
    uint32_t down_rs, sdown_rs;
    // grouped kernels: the routed pairs grouped by expert (moe_group_kernel)
    const uint32_t* grp_n;           // [1] routed groups
    const uint4* grp;                // [groups] {expert, first pair, pairs, 0}
    const uint32_t* grp_pairs;       // [tokens*k] routed index t*k + j, grouped by expert
    uint32_t gsize_r, gsize_s;       // pairs per group: routed / shared expert
    unsigned int* route_flag;        // single token: set (release) once CTA 0 has stored the routing, or null
    // expert-parallel items whose count is only known on the device: read
    // here after the grid dependency (tokens is then the capacity), or null
    const uint32_t* d_items;
    DeviceStatus* status;
    Tables tables;
};

struct MoeDownArgs {
    uint64_t hidden, ffn;
    int nb_f;
    int tpr_f;                       // threads per row over the ffn width
    uint64_t tokens;
    uint64_t k;
    uint64_t experts;
    const uint8_t* const* down;      // [experts] planar matrices
    const uint8_t* sdown;
    const lbk_routed* routed;
    const uint8_t* hq;               // [tokens][k+1][nb_f][292]
    float* out;                      // [tokens][hidden]
    uint64_t rows_per_cta;
    uint64_t wps;                    // warps per slot
    uint64_t prod_floats;
    uint64_t chain_floats;
    // bulk-copy-staged kernel: CTAs [0, routed_ctas) take routed slots, the
    // rest the shared expert; items (token, slot, chunk of rows)
    uint32_t routed_ctas;
    uint64_t chunk_r, chunk_s, chunks_r, chunks_s;
    float* dots;                     // [tokens][dots_slots][hidden] row dots of slot (routed j < k, shared k)
    uint32_t dots_slots;
    int combine;                     // 1: form `out` from the dots (else leave the dots)
    int has_shared;                  // 0: no shared-expert CTAs
    unsigned int* counters;          // [tokens][hidden/64] arrivals, zero between launches
    // grouped kernels (see MoeGateUpArgs)
    const uint32_t* grp_n;
    const uint4* grp;
    const uint32_t* grp_pairs;
    uint32_t gsize_r, gsize_s;
    // single token: the gate/up kernel's routing flag (early copies), or null;
    // the last routed CTA to have read it clears it and route_readers
    unsigned int* route_flag;
    unsigned int* route_readers;
    uint32_t route_polls;            // polls of route_flag before LBK_TIMEOUT
    const uint32_t* d_items;         // see MoeGateUpArgs
    // expert-parallel items returned in place: item t's row dots go straight
    // to (float*)(ret_peers[ret_addr[t].x] + ret_off) + ret_addr[t].y * hidden
    // (its home rank's buffer, over NVLink), then a system-scope fence; or null
    const uint2* ret_addr;
    uint8_t* const* ret_peers;
    uint64_t ret_off;
    DeviceStatus* status;
    Tables tables;
};

constexpr int kMoeDownTmaWarps = 16;   // warps per bulk-copy-staged down CTA
constexpr int kMoeDownCombineRows = 64;  // rows combined by the last arriving warp

bool moe_fused_supported(int gate_type, int shared_gate_type, int down_type, int shared_down_type);
size_t moe_gate_up_fixed_smem(int gate_type, int shared_gate_type);
size_t moe_down_fixed_smem(int down_type, int shared_down_type);
cudaError_t launch_moe_gate_up(int gate_type, int shared_gate_type, const MoeGateUpArgs& a, cudaStream_t stream);
// Bulk-copy-staged gate/up over `ctas` CTAs (planar, nb_h in {8, 16}).
bool moe_gate_up_tma_supported(int gate_type, int shared_gate_type, int nb_h);
// Whether its routed CTAs can finish the router (partials + logits in shared memory).
bool moe_gate_up_tma_defer_fits(int gate_type, uint64_t experts, uint64_t chunks);
cudaError_t launch_moe_gate_up_tma(int gate_type, int shared_gate_type, const MoeGateUpArgs& a, unsigned ctas,
                                   cudaStream_t stream);
cudaError_t launch_moe_down(int down_type, int shared_down_type, const MoeDownArgs& a, cudaStream_t stream);
// Expert-parallel combine of routed row dots [tokens][k][H] and shared row dots [tokens][H].
cudaError_t launch_ep_combine(const lbk_routed* routed, const float* routed_dots, const float* shared_dots, float* out,
                              uint64_t tokens, uint64_t k, uint64_t H, DeviceStatus* status, cudaStream_t stream);
// Bulk-copy-staged down over `ctas` CTAs (planar, nb_f <= 16).
bool moe_down_tma_supported(int down_type, int shared_down_type, int nb_f);
cudaError_t launch_moe_down_tma(int down_type, int shared_down_type, const MoeDownArgs& a, unsigned ctas,
                                cudaStream_t stream);

// Grouped kernels (several tokens per call): the (token, slot) pairs of a
// call are grouped by routed expert, and each weight half block is decoded
// once for all pairs of its group.
struct MoeGroupArgs {
    const lbk_routed* routed;        // [tokens][k]
    uint64_t tokens, k, experts;
    uint32_t gsize;                  // pairs per group at most
    uint32_t* n;                     // [1] groups written
    uint4* groups;                   // [tokens*k] {expert, first pair, pairs, 0}
    uint32_t* pairs;                 // [tokens*k] routed index t*k + j, grouped by expert, ascending in t
    DeviceStatus* status;
    const uint32_t* d_items;         // expert-parallel items counted on the device (k = 1), or null
};

// Pairs per group the grouped kernels of a type pair take (the activations
// of every pair of a group sit in registers), and their warps per CTA.
struct GrpShape {
    uint32_t routed, shared, warps;
};
GrpShape moe_gate_up_grp_shape(int gate_type, int shared_gate_type);
GrpShape moe_down_grp_shape(int down_type, int shared_down_type);
// Whether the grouped kernels take these types / widths (the bulk-copy ones).
bool moe_grouped_supported(int gate_type, int shared_gate_type, int down_type, int shared_down_type, int nb_h, int nb_f);
cudaError_t launch_moe_group(const MoeGroupArgs& a, cudaStream_t stream);

cudaError_t launch_moe_gate_up_grp(int gate_type, int shared_gate_type, const MoeGateUpArgs& a, unsigned ctas,
                                   cudaStream_t stream);
cudaError_t launch_moe_down_grp(int down_type, int shared_down_type, const MoeDownArgs& a, unsigned ctas,
                                cudaStream_t stream);

// Expert-parallel exchange over peer memory (ep.cu).
//
// The control block of an exchange buffer: the token count and the flags
// with which the ranks order a layer step among themselves, without the host.
// `step` is this rank's step number (raised by the publish); `published` is
// the step whose routing and images the buffer holds; done[r] is the step
// whose row dots rank r has finished storing into this buffer.
constexpr uint32_t kEpMaxRanks = 64;
struct EpControl {
    uint32_t tokens;
    uint32_t published;
    uint32_t step;
    uint32_t scatter_ctas;  // CTAs of this rank's scatter that have finished (reset by the last)
    uint32_t pad[12];
    uint32_t done[kEpMaxRanks];
};
static_assert(sizeof(EpControl) <= 512, "control block");
struct EpGatherArgs {
    const uint8_t* const* peers;  // [world] exchange buffers, as this GPU addresses them
    uint32_t world, rank, cap, k, q8b;  // cap: tokens per rank at most
    uint64_t off_ctl, off_q8;     // offsets in an exchange buffer (routing at 0)
    uint32_t first, count;        // this rank's experts [first, first + count)
    uint8_t* q8_items;            // [cap_items][q8b]
    lbk_routed* items;            // [cap_items] local expert ID, coefficient 0
    uint2* returns;               // [cap_items] {home rank, pair t * k + j}
    uint32_t* d_count;            // items gathered (0 at the start: the previous scatter reset it)
    uint32_t cap_items;           // world * cap * k
    uint32_t polls;               // polls of a peer's flag before LBK_TIMEOUT
    DeviceStatus* status;
};
struct EpScatterArgs {
    uint8_t* const* peers;
    uint32_t world, rank;
    uint64_t off_ctl, off_dots;
    const float* dots;            // [cap_items][hidden]
    const uint2* returns;
    uint32_t* d_count;            // reset to 0 by the last CTA, for the next step's gather
    uint32_t cap_items, hidden;
};
cudaError_t launch_ep_gather(const EpGatherArgs& a, int sm_count, cudaStream_t stream);
cudaError_t launch_ep_scatter(const EpScatterArgs& a, int sm_count, cudaStream_t stream);
cudaError_t launch_ep_publish(EpControl* ctl, uint32_t tokens, cudaStream_t stream);
// After items returned in place: reset the item count, release done[rank] =
// step in every rank's buffer (what the scatter's last CTA does).
cudaError_t launch_ep_signal(const EpScatterArgs& a, cudaStream_t stream);
// The home rank's combine once every rank's dots are in (see launch_ep_combine):
// waits at most `polls` polls for done[0, world) to reach this step.
cudaError_t launch_ep_combine_wait(const EpControl* ctl, uint32_t world, uint32_t polls, const lbk_routed* routed,
                                   const float* routed_dots, const float* shared_dots, float* out, uint64_t tokens,
                                   uint64_t k, uint64_t H, DeviceStatus* status, cudaStream_t stream);

}  // namespace lbk
