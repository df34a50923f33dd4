// lbk_tc.h -- grouped row dots on the tcgen05 tensor cores (tc_dots.cu).
#pragma once

#include "lbk_kernels.h"

namespace lbk {

struct TcMatrix {  // layout of lbk_tc_matrix
    const uint8_t* data;  // IQ2_S, planar rows
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
};

int tc_dots_smem_bytes();
cudaError_t launch_tc_dots_iq2(const TcDotsArgs& a, uint32_t jobs, cudaStream_t stream);

}  // namespace lbk
