// decode.cu -- f32 dequantization of packed rows (GGUF block layout).
//
// Restates the reference's block decoders: decode_row_into
// (bridge-quant-layout/src/k_quants.rs:71-105) over decode_q4_k_validated /
// decode_q5_k_validated (:242-300), decode_iq2_s_validated (iq2_s.rs:9-39)
// and decode_iq3_s_validated (iq3_s.rs:9-53), each f32 product in the
// reference's order with no contraction (explicit _rn operations), so every
// output is bit-identical. One thread writes 8 consecutive outputs of one
// block (a grid index / sign byte of the IQ types, 8 lanes of a K-quant
// sub-block). F32 rows are a bit copy (decode_f32_validated), done by the
// host. The scale scan (launch_validate_scales) runs first; a non-finite
// d / dmin is reported and nothing is written.

#include "lbk_kernels.h"

namespace lbk {

namespace {

__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// k_quants.rs scale_min (:231-240)
__device__ __forceinline__ void scale_min_bytes(const uint8_t* sc, int j, uint32_t& s, uint32_t& m) {
    if (j < 4) {
        s = sc[j] & 0x3f;
        m = sc[j + 4] & 0x3f;
    } else {
        s = (sc[j + 4] & 0x0f) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

__global__ void decode_kernel(DecodeArgs a) {
    const uint64_t items = a.rows * (uint64_t)a.nb * 32;  // 32 runs of 8 outputs per block
    if (status_set(a.status)) return;  // a scale failed validation: write nothing
    for (uint64_t it = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
         it += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t blk = it >> 5;  // row-major blocks of the range
        const int r = (int)(it & 31);  // run of 8 outputs inside the block
        float* out = a.out + blk * 256 + (uint64_t)r * 8;
        float v[8];
        if (a.type == LBK_TYPE_IQ2_S) {
            const uint8_t* e = a.data + blk * 82;
            const float d = f16_at(e);
            const int group = r >> 2, lg = r & 3;
            const uint32_t sc = e[74 + group];
            const uint32_t nib = lg < 2 ? (sc & 0x0f) : (sc >> 4);
            const float scale = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)nib)), 0.25f);
            const uint32_t high = e[66 + group];
            const uint32_t index = e[2 + group * 4 + lg] | ((high << (8 - 2 * lg)) & 0x300u);
            const uint64_t grid = a.iq2s[index];
            const uint32_t signs = e[34 + group * 4 + lg];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float g = (float)((grid >> (8 * i)) & 0xff);
                v[i] = __fmul_rn(__fmul_rn(scale, g), (signs & (1u << i)) ? -1.0f : 1.0f);
            }
        } else if (a.type == LBK_TYPE_IQ3_S) {
            const uint8_t* e = a.data + blk * 110;
            const float d = f16_at(e);
            const int group = r >> 2, lg = r & 3;
            const uint32_t packed = e[106 + (group >> 1)];
            const uint32_t nib = (group & 1) ? (packed >> 4) : (packed & 0x0f);
            const float scale = __fmul_rn(d, (float)(1 + 2 * nib));
            const uint32_t high = e[66 + group];
            const uint32_t i1 = e[2 + group * 8 + lg * 2] | ((high << (8 - 2 * lg)) & 0x100u);
            const uint32_t i2 = e[2 + group * 8 + lg * 2 + 1] | ((high << (7 - 2 * lg)) & 0x100u);
            const uint32_t g1 = a.iq3s[i1], g2 = a.iq3s[i2];
            const uint32_t signs = e[74 + group * 4 + lg];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                v[i] = __fmul_rn(__fmul_rn(scale, (float)((g1 >> (8 * i)) & 0xff)), (signs & (1u << i)) ? -1.0f : 1.0f);
                v[i + 4] = __fmul_rn(__fmul_rn(scale, (float)((g2 >> (8 * i)) & 0xff)),
                                     (signs & (1u << (i + 4))) ? -1.0f : 1.0f);
            }
        } else {  // Q4_K / Q5_K: run r covers outputs 8r .. 8r+7 of sub-block j = r / 4
            const bool q5 = a.type == LBK_TYPE_Q5_K;
            const uint8_t* e = a.data + blk * (q5 ? 176 : 144);
            const float d = f16_at(e), dmin = f16_at(e + 2);
            const int j = r >> 2, group = j >> 1, hi = j & 1, lane0 = (r & 3) * 8;
            uint32_t s, m;
            scale_min_bytes(e + 4, j, s, m);
            const float dj = __fmul_rn(d, (float)s), mj = __fmul_rn(dmin, (float)m);
            const uint8_t* qs = e + (q5 ? 48 : 16) + group * 32;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int lane = lane0 + i;
                uint32_t q = hi ? (qs[lane] >> 4) : (qs[lane] & 0x0f);
                if (q5) q += ((e[16 + lane] >> (2 * group + hi)) & 1u) * 16u;
                v[i] = __fsub_rn(__fmul_rn(dj, (float)q), mj);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) out[i] = v[i];
    }
}

}  // namespace

cudaError_t launch_decode(const DecodeArgs& a, int sm_count, cudaStream_t stream) {
    const uint64_t items = a.rows * (uint64_t)a.nb * 32;
    uint64_t grid = (items + 255) / 256;
    const uint64_t cap = (uint64_t)sm_count * 8;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    decode_kernel<<<(unsigned)grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace lbk
