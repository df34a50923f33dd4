// lbk_host.h -- host-side helpers shared by the C ABI translation units
// (abi.cu owns the thread-local error detail and the layer handle).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lightbridge_kernels.h"

#ifndef LBK_API
#define LBK_API extern "C" __attribute__((visibility("default")))
#endif

namespace lbk {

// Fills the calling thread's lbk_error_detail and returns `status`.
int32_t host_fail(int32_t status, const char* msg, uint64_t index, uint64_t expected, uint64_t actual, uint32_t bits);
// Clears the detail and returns LBK_OK.
int32_t host_ok();
// cudaSetDevice(ctx's device), reported as LBK_CUDA_ERROR on failure.
int32_t host_set_device(lbk_context* ctx);
// lbk_ep_layer_create over `w`, whose device memory is the one allocation
// `owned`: on success the layer frees it on destroy; on failure the caller
// keeps it.
int32_t layer_create_owned(lbk_context* ctx, const lbk_moe_weights* w, uint64_t global_experts, uint64_t first_expert,
                           void* stream, void* owned, lbk_moe_layer** out);

}  // namespace lbk
