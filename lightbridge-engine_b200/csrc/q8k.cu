// q8k.cu -- standalone Q8_K activation quantization.
//
// Replaces quantize_row_q8_k_into (bridge-quant-layout/src/q8_k.rs:16-76),
// byte-identical. The reference rejects a row with any non-finite lane before
// writing anything and names the first such lane; a scan kernel finds the
// lowest bad lane with an atomic minimum, and the quantize kernel writes only
// when the scan found none.

#include "lbk_kernels.h"

namespace lbk {

namespace {

__global__ void scan_finite_kernel(const float* x, uint64_t n, unsigned long long* first_bad) {
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        if (!isfinite(x[i])) atomicMin(first_bad, (unsigned long long)i);
}

__global__ void quantize_kernel(const float* x, uint64_t n, uint8_t* q8, const unsigned long long* first_bad,
                                DeviceStatus* status) {
    unsigned long long bad = *first_bad;
    if (bad != ~0ull) {
        if (blockIdx.x == 0 && threadIdx.x == 0) report(status, LBK_NON_FINITE_ACTIVATION, bad, __float_as_uint(x[bad]));
        return;
    }
    const int lane = threadIdx.x & 31;
    const uint64_t nb = n / kQK;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    for (uint64_t b = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); b < nb; b += warps) {
        const float* xb = x + b * kQK + lane * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = xb[i];
        Q8Block q = quantize_q8k_warp(v, lane);
        uint8_t* o = q8 + b * kQ8Bytes;
        uint32_t* ow = reinterpret_cast<uint32_t*>(o + 4);
        ow[lane * 2] = q.q[0];
        ow[lane * 2 + 1] = q.q[1];
        int32_t pair = q.pair_sum + __shfl_xor_sync(0xffffffffu, q.pair_sum, 1);
        if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(o + 260 + lane) = (int16_t)pair;
        if (lane == 0) *reinterpret_cast<float*>(o) = q.d;
    }
}

}  // namespace

cudaError_t launch_quantize_q8k_ws(const float* x, uint64_t n, uint8_t* q8, unsigned long long* scratch_min,
                                   DeviceStatus* status, int sm_count, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(scratch_min, 0xff, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    uint64_t blocks = (n + 255) / 256;
    unsigned grid = (unsigned)(blocks < (uint64_t)sm_count * 4 ? (blocks ? blocks : 1) : (uint64_t)sm_count * 4);
    scan_finite_kernel<<<grid, 256, 0, stream>>>(x, n, scratch_min);
    uint64_t nb = n / kQK;
    uint64_t qgrid = (nb + 7) / 8;
    if (qgrid > (uint64_t)sm_count * 8) qgrid = (uint64_t)sm_count * 8;
    if (qgrid < 1) qgrid = 1;
    quantize_kernel<<<(unsigned)qgrid, 256, 0, stream>>>(x, n, q8, scratch_min, status);
    return cudaGetLastError();
}

}  // namespace lbk
