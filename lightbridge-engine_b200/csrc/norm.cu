// norm.cu -- RMSNorm and residual add of the MoE block (route / finish).
//
// Replaces weighted_rms_norm_into and residual_add_in_place
// (bridge-kernels-reference/src/norm.rs:5-18, :83-100) as hy3_moe_route_token
// and hy3_moe_finish_token use them around the MoE step (layer.rs:588-593,
// :654): the FFN input is normalized before the router, the MoE output is
// added to the hidden state after it.
//
// Both keep the reference's validate-before-write atomicity: every check of a
// call completes before any output is written, and a failed check leaves the
// output untouched (reported through the device status word).

#include "lbk_kernels.h"

namespace lbk {

namespace {

constexpr int kNormThreads = 512;

// One CTA per row: checks (input, weight, scale, outputs; the first failing
// index of the first failing check, the reference's order), then the writes.
// kSeq: the sum of squares is the reference's single f32 chain in index order
// (rms_scale, norm.rs:144-153), bit-identical; else a fixed tree (every thread
// a strided chain, then shuffles and the warps' sums in order), deterministic
// and within 1e-5 of the chain.
template <bool kSeq>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(NormArgs a) {
    extern __shared__ float s_x[];  // kSeq: the row, staged for the chain
    __shared__ float s_warp[kNormThreads / 32];
    __shared__ unsigned long long s_bad;  // (check << 40) | index, minimum wins
    __shared__ float s_scale;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t n = a.n;
    for (uint64_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const float* x = a.x + r * n;
        float* out = a.out + r * n;
        if (tid == 0) s_bad = ~0ull;
        __syncthreads();
        float part = 0.0f;
        for (uint64_t i = tid; i < n; i += kNormThreads) {
            const float v = x[i], w = a.w[i];
            if (!isfinite(v)) atomicMin(&s_bad, (1ull << 40) | i);
            if (!isfinite(w)) atomicMin(&s_bad, (2ull << 40) | i);
            if (kSeq) s_x[i] = v;
            else part = __fadd_rn(part, __fmul_rn(v, v));
        }
        if (!kSeq) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
            if (lane == 0) s_warp[warp] = part;
        }
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            if (kSeq) {
                for (uint64_t i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(s_x[i], s_x[i]));
            } else {
                for (int i = 0; i < kNormThreads / 32; i++) sum = __fadd_rn(sum, s_warp[i]);
            }
            const float mean = __fdiv_rn(sum, (float)n);
            const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            if (!isfinite(scale) && s_bad == ~0ull) s_bad = (3ull << 40);
            s_scale = scale;
        }
        __syncthreads();
        const float scale = s_scale;
        if (s_bad == ~0ull) {
            for (uint64_t i = tid; i < n; i += kNormThreads) {
                const float v = __fmul_rn(__fmul_rn(x[i], scale), a.w[i]);
                if (!isfinite(v)) atomicMin(&s_bad, (4ull << 40) | i);
            }
        }
        __syncthreads();
        const unsigned long long bad = s_bad;
        if (bad != ~0ull) {
            if (tid == 0) {
                const uint64_t i = bad & ((1ull << 40) - 1), kind = bad >> 40;
                const float v = kind == 1 ? x[i] : kind == 2 ? a.w[i] : kind == 3 ? scale : __fmul_rn(__fmul_rn(x[i], scale), a.w[i]);
                report(a.status, LBK_NON_FINITE_VALUE, kind == 3 ? 0 : i, __float_as_uint(v));
            }
        } else {
            for (uint64_t i = tid; i < n; i += kNormThreads) out[i] = __fmul_rn(__fmul_rn(x[i], scale), a.w[i]);
        }
        __syncthreads();
    }
}

// residual_add_in_place's checks over the whole call: dest finite, src finite,
// sums finite, in that order; the smallest (check, index) key wins.
__global__ void residual_check_kernel(const float* dest, const float* src, uint64_t n, unsigned long long* key) {
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const float d = dest[i], s = src[i];
        if (!isfinite(d)) atomicMin(key, (1ull << 40) | i);
        else if (!isfinite(s)) atomicMin(key, (2ull << 40) | i);
        else if (!isfinite(__fadd_rn(d, s))) atomicMin(key, (3ull << 40) | i);
    }
}

__global__ void residual_report_kernel(const float* dest, const float* src, const unsigned long long* key,
                                       DeviceStatus* st) {
    const unsigned long long k = *key;
    if (k == ~0ull) return;
    const uint64_t i = k & ((1ull << 40) - 1), kind = k >> 40;
    const float v = kind == 1 ? dest[i] : kind == 2 ? src[i] : __fadd_rn(dest[i], src[i]);
    report(st, LBK_NON_FINITE_VALUE, i, __float_as_uint(v));
}

// The writes, skipped when any check of the call (or an earlier step of the
// same call) failed.
__global__ void residual_apply_kernel(float* dest, const float* src, uint64_t n, const DeviceStatus* st) {
    if (status_set(st)) return;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        dest[i] = __fadd_rn(dest[i], src[i]);
}

}  // namespace

cudaError_t launch_rms_norm(const NormArgs& a, int sm_count, cudaStream_t stream) {
    uint64_t grid = a.rows < (uint64_t)sm_count * 4 ? a.rows : (uint64_t)sm_count * 4;
    if (grid < 1) grid = 1;
    if (a.sequential) {
        const size_t smem = a.n * sizeof(float);
        if (smem > kMaxSmem) return cudaErrorInvalidValue;
        cudaError_t e = ensure_max_smem(reinterpret_cast<const void*>(rms_norm_kernel<true>));
        if (e != cudaSuccess) return e;
        rms_norm_kernel<true><<<(unsigned)grid, kNormThreads, smem, stream>>>(a);
    } else {
        rms_norm_kernel<false><<<(unsigned)grid, kNormThreads, 0, stream>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_residual_add(float* dest, const float* src, uint64_t n, unsigned long long* key, DeviceStatus* status,
                                int sm_count, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(key, 0xff, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    uint64_t grid = (n + 255) / 256;
    if (grid > (uint64_t)sm_count * 8) grid = (uint64_t)sm_count * 8;
    if (grid < 1) grid = 1;
    residual_check_kernel<<<(unsigned)grid, 256, 0, stream>>>(dest, src, n, key);
    residual_report_kernel<<<1, 1, 0, stream>>>(dest, src, key, status);
    residual_apply_kernel<<<(unsigned)grid, 256, 0, stream>>>(dest, src, n, status);
    return cudaGetLastError();
}

}  // namespace lbk
