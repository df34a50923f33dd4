// lbk_tc.h -- grouped row dots on the tcgen05 tensor cores (tc_dots.cu).
#pragma once

#include "lbk_kernels.h"

namespace lbk {

struct TcMatrix {  // layout of lbk_tc_matrix
    const uint8_t* data;  // IQ2_S or IQ3_S, planar rows
    uint32_t rows, nb;
    uint64_t out_offset;  // column of this matrix's first row in a pair's dots
};
static_assert(sizeof(TcMatrix) == 24, "lbk_tc_matrix layout");

struct TcDotsArgs {
    const TcMatrix* mats;
    uint32_t nmat;
    const uint4* jobs;           // per CTA: {matrix, first row (multiple of 128), first pair, pairs <= 32}
    const uint8_t* q8;           // token images, q8_row_bytes apart
    uint64_t q8_row_bytes;
    const uint32_t* pair_tokens; // pair -> token
    float* dots;                 // [pairs][dots_stride]
    uint64_t dots_stride;
    DeviceStatus* status;
    Tables tables;
    // Grouped mode (jobs null): the pairs grouped by expert on the device
    // (moe_group_kernel, groups of at most 32); CTA b is group b / (2 tiles),
    // matrix (b / tiles) % 2 (gate, up) and row tile b % tiles; a CTA past
    // the groups written returns. Gate row r goes to column r, up row r to
    // column rows + r.
    const uint4* groups;         // {expert, first pair, pairs, 0}
    const uint32_t* ngroups;
    const uint8_t* const* gate;  // expert -> planar rows (the down matrices when mats_per_group is 1)
    const uint8_t* const* up;
    uint32_t experts, rows, nb;
    uint32_t mats_per_group;     // 2: gate and up; 1: one matrix per expert
    bool out_by_token;           // a pair's dots go to row pair_tokens[p] instead of p
    // with out_by_token: token r's row goes to (float*)(ret_peers[ret_addr[r].x]
    // + ret_off) + ret_addr[r].y * dots_stride instead (its home rank's buffer),
    // then a system-scope fence; or null
    const uint2* ret_addr;
    uint8_t* const* ret_peers;
    uint64_t ret_off;
};

// SwiGLU and Q8_K of h per grouped pair, from the tensor-core gate/up dots:
// h = swiglu(gate, up) (activation.rs:170-178), quantized per 256-row block
// (quantize_row_q8_k_into) into the image of the pair's item, slot 0 of k + 1.
struct TcSwigluArgs {
    const float* dots;           // [pairs][2 ffn] in grouped order
    const uint32_t* pairs;       // grouped position -> item
    const uint32_t* count;       // items (device)
    uint32_t cap, ffn, nb_f, slots;  // slots = k + 1 of the workspace layout
    uint8_t* hq;
    DeviceStatus* status;
};

int tc_dots_smem_bytes();
// type: LBK_TYPE_IQ2_S (groups of 16 weights, two masked MMAs per 32) or
// LBK_TYPE_IQ3_S (groups of 32, one MMA each; no 0.125 factor)
cudaError_t launch_tc_dots(int type, const TcDotsArgs& a, uint32_t jobs, cudaStream_t stream);
cudaError_t launch_tc_swiglu_quant(const TcSwigluArgs& a, int sm_count, cudaStream_t stream);

}  // namespace lbk
