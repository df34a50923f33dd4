// lbk_kernels.h -- internal launch interface between the C ABI (abi.cu) and
// the kernel translation units. Not installed; the public surface is
// include/lightbridge_kernels.h.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "lbk_device.cuh"

namespace lbk {

constexpr size_t kMaxSmem = 227 * 1024;

// Raises a kernel's dynamic shared-memory limit on the current device once.
cudaError_t ensure_max_smem(const void* kernel);

// ------------------------------------------------------------------ GEMV

constexpr int kGemvStore = 0;       // y[r] = dot
constexpr int kGemvAccumulate = 1;  // y[r] = y[r] + scale * dot

struct GemvArgs {
    MatrixRef w;
    const float* x;         // f32 input (unless q8_in)
    const uint8_t* q8_in;   // optional pre-quantized Q8_K input
    uint8_t* q8_out;        // optional: receives Q8_K(x)
    float* y;
    float scale;
    int mode;
    int tpr;                // threads per row
    int tail_slots;         // rows per tail batch per warp
    int32_t* block_sums;    // optional per-block integer sums
    // Optional device-side matrix selection (routed experts): when set, the
    // weights are mat_table[sel->expert_id] and the accumulate scale is
    // sel->coefficient.
    const uint8_t* const* mat_table;
    const lbk_routed* sel;
    uint64_t mat_count;     // entries of mat_table
    DeviceStatus* status;
    Tables tables;
};

void gemv_plan(int type, int nb, int* tpr, int* slots);
size_t gemv_smem_required(int type, int nb, int slots);
cudaError_t launch_gemv(int type, int layout, const GemvArgs& a, int sm_count, cudaStream_t stream);

// ------------------------------------------------------------- quantize

cudaError_t launch_quantize_q8k_ws(const float* x, uint64_t n, uint8_t* q8, unsigned long long* scratch_min,
                                   DeviceStatus* status, int sm_count, cudaStream_t stream);

// --------------------------------------------------------------- router

struct RouterArgs {
    const float* w;         // [E][hidden] f32 rows
    const float* x;         // [tokens][hidden]
    float* logits;          // [tokens][E]
    uint64_t hidden, experts, tokens;
    DeviceStatus* status;
};
cudaError_t launch_router(const RouterArgs& a, int mode, int sm_count, cudaStream_t stream);

// Fused router (tree order) + Q8_K quantization of the tokens + top-k in the
// last CTA.
struct RouterFusedArgs {
    RouterArgs r;
    float* partials;        // [tokens][experts][chunks]
    uint8_t* q8x;           // [tokens][hidden/256][292], or null
    unsigned int* counter;  // zero between launches
    const float* bias;
    uint32_t k;
    float weight_scale;
    lbk_routed* routed;     // [tokens][k], or null (logits only)
    int defer;              // 1: leave the chunk partials for the consumer (no last-CTA pass)
    int split;              // 1: logits and top-k in a second launch, one warp per token (set by the launcher)
    unsigned int* zero;     // arrival counters of the launches that follow, zeroed here
    uint64_t zero_words;
};
size_t router_partials_floats(uint64_t hidden, uint64_t experts, uint64_t tokens);
cudaError_t launch_router_fused(const RouterFusedArgs& f, int sm_count, cudaStream_t stream);
// The sequential (bit-identical) logits, the tokens' Q8_K and top-k in one
// launch, for at most 4 tokens and 1024 experts (cudaErrorInvalidValue else).
cudaError_t launch_router_seq_fused(const RouterFusedArgs& f, int sm_count, cudaStream_t stream);

// weighted_rms_norm_into per row (norm.cu): rows x n values.
struct NormArgs {
    const float* x;
    const float* w;      // [n]
    float eps;
    float* out;
    uint64_t rows, n;
    int sequential;      // 1: the reference's single f32 chain (n <= 58K); 0: fixed tree
    DeviceStatus* status;
};
cudaError_t launch_rms_norm(const NormArgs& a, int sm_count, cudaStream_t stream);
// dest += src with residual_add_in_place's checks; key: 8 bytes of scratch.
cudaError_t launch_residual_add(float* dest, const float* src, uint64_t n, unsigned long long* key, DeviceStatus* status,
                                int sm_count, cudaStream_t stream);

struct TopkArgs {
    const float* logits;    // [tokens][E]
    const float* bias;      // [E]
    uint64_t experts, tokens;
    uint32_t k;
    float weight_scale;
    lbk_routed* routed;     // [tokens][k]
    DeviceStatus* status;
};
cudaError_t launch_topk(const TopkArgs& a, cudaStream_t stream);

// ------------------------------------------------------------ layout tools

struct RepackArgs {
    const uint8_t* src;
    uint8_t* dst;
    uint64_t rows;
    int nb;
    int type;
    int to_planar;          // 1: GGUF -> planar, 0: planar -> GGUF
};
cudaError_t launch_repack(const RepackArgs& a, cudaStream_t stream);
cudaError_t launch_build_tables(const uint64_t* iq2s, const uint32_t* iq3s, uint32_t* iq2_img, uint32_t* iq3_img,
                                cudaStream_t stream);
// f32 decode of `rows` consecutive GGUF rows of nb blocks (decode.cu)
struct DecodeArgs {
    int type;                 // Q4_K, Q5_K, IQ2_S or IQ3_S
    const uint8_t* data;      // the range's first row
    uint64_t rows;
    int nb;
    float* out;               // rows * nb * 256
    const uint64_t* iq2s;     // IQ2S_GRID
    const uint32_t* iq3s;     // IQ3S_GRID
    DeviceStatus* status;
};
cudaError_t launch_decode(const DecodeArgs& a, int sm_count, cudaStream_t stream);
cudaError_t launch_validate_scales(int type, int layout, const uint8_t* data, uint64_t rows, int nb,
                                   unsigned long long* scratch_min, DeviceStatus* status, cudaStream_t stream);

// ------------------------------------------------------------- elementwise

// h[i] = swiglu(gate[i], up[i]) with the finite check of apply_swiglu.
cudaError_t launch_swiglu(const float* gate, const float* up, float* h, uint64_t n, DeviceStatus* status,
                          cudaStream_t stream);

}  // namespace lbk
