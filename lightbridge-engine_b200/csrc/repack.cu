// repack.cu -- GGUF <-> planar layout conversion and binary16 scale scans.
//
// The planar layout (described in include/lightbridge_kernels.h) is a byte
// permutation of the GGUF bytes: every field of every block lands in its own
// plane, and Q4_K / Q5_K quant bytes are reordered lane-major inside each
// 32-byte group. IQ2_S / IQ3_S qh words (one per half block) are stored
// bit-transposed (qh_transpose, an involution), and so is every 32-bit word
// of their sign bytes (sign_transpose / sign_untranspose). It exists so that a thread's
// half block is a handful of aligned loads whose bits feed the decoder
// directly; both directions are exact.
//
// The scale scan restates validate_scales (bridge-quant-layout/src/k_quants.rs:178-208)
// over a whole matrix, reporting the first non-finite block in row-major order.

#include "lbk_kernels.h"

namespace lbk {

namespace {

struct Field {
    int src_off;   // offset inside the GGUF block
    int bytes;     // field bytes per block
    int lane_major;  // 1: Q4_K/Q5_K qs or Q5_K qh: permute 32-byte groups;
                     // 2: IQ2_S/IQ3_S qh: transpose each 32-bit word (qh_transpose);
                     // 3: IQ2_S/IQ3_S signs: transpose each 32-bit word (sign_transpose)
};

__host__ __device__ inline int fields_of(int type, Field* f) {
    switch (type) {
        case LBK_TYPE_IQ2_S:  // qs | signs | qh | scales | d
            f[0] = {2, 32, 0};
            f[1] = {34, 32, 3};
            f[2] = {66, 8, 2};
            f[3] = {74, 8, 0};
            f[4] = {0, 2, 0};
            return 5;
        case LBK_TYPE_IQ3_S:  // qs | signs | qh | scales | d
            f[0] = {2, 64, 0};
            f[1] = {74, 32, 3};
            f[2] = {66, 8, 2};
            f[3] = {106, 4, 0};
            f[4] = {0, 2, 0};
            return 5;
        case LBK_TYPE_Q4_K:  // qs (lane-major) | scales | d,dmin
            f[0] = {16, 128, 1};
            f[1] = {4, 12, 0};
            f[2] = {0, 4, 0};
            return 3;
        default:  // Q5_K: qs (lane-major) | qh (lane-major) | scales | d,dmin
            f[0] = {48, 128, 1};
            f[1] = {16, 32, 1};
            f[2] = {4, 12, 0};
            f[3] = {0, 4, 0};
            return 4;
    }
}

// lane-major position of byte j of a 32-byte group: new[4k+i] = old[k+8i]
__host__ __device__ inline int lane_major_pos(int j) {
    int k = j & 7, i = j >> 3;  // old index j = k + 8i
    return 4 * k + i;
}

// One thread per block: its fields move between the GGUF block and the
// block's slots in its row's planes; the thread of block 0 also zeroes the
// row's pad bytes.
__global__ void repack_kernel(RepackArgs a, int block_bytes) {
    Field f[5];
    int nf = fields_of(a.type, f);
    const uint64_t nblk = a.rows * (uint64_t)a.nb;
    const uint64_t rs = planar_row_bytes(block_bytes, a.nb);
    for (uint64_t bi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; bi < nblk; bi += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t row = bi / (uint64_t)a.nb, b = bi % (uint64_t)a.nb;
        uint64_t plane = row * rs;  // start of field plane k inside the planar row
        for (int k = 0; k < nf; k++) {
            const int fb = f[k].bytes;
            if (f[k].lane_major >= 2) {
                for (int j = 0; j < fb; j += 4) {
                    uint64_t g = bi * block_bytes + f[k].src_off + j;
                    uint64_t p = plane + b * fb + j;
                    const uint8_t* s = a.to_planar ? a.src + g : a.src + p;
                    uint8_t* d = a.to_planar ? a.dst + p : a.dst + g;
                    uint32_t w = (uint32_t)s[0] | ((uint32_t)s[1] << 8) | ((uint32_t)s[2] << 16) | ((uint32_t)s[3] << 24);
                    if (f[k].lane_major == 2) w = qh_transpose(w);
                    else w = a.to_planar ? sign_transpose(w) : sign_untranspose(w);
                    for (int i = 0; i < 4; i++) d[i] = (uint8_t)(w >> (8 * i));
                }
                plane += (uint64_t)a.nb * fb;
                continue;
            }
            for (int j = 0; j < fb; j++) {
                int pj = j;
                if (f[k].lane_major) pj = (j & ~31) + lane_major_pos(j & 31);
                uint64_t g = bi * block_bytes + f[k].src_off + j;  // GGUF byte
                uint64_t p = plane + b * fb + pj;                    // planar byte
                if (a.to_planar)
                    a.dst[p] = a.src[g];
                else
                    a.dst[g] = a.src[p];
            }
            plane += (uint64_t)a.nb * fb;
        }
        if (a.to_planar && b == 0)
            for (uint64_t p = row * rs + (uint64_t)a.nb * block_bytes; p < (row + 1) * rs; p++) a.dst[p] = 0;
    }
}

// Bytes of block bi's binary16 d (followed by dmin for the K types).
__device__ __forceinline__ const uint8_t* scale_ptr(int type, int layout, const uint8_t* data, int nb, uint64_t bi) {
    const bool two = type == LBK_TYPE_Q4_K || type == LBK_TYPE_Q5_K;
    const int bb = type == LBK_TYPE_IQ2_S ? 82 : type == LBK_TYPE_IQ3_S ? 110 : type == LBK_TYPE_Q4_K ? 144 : 176;
    const uint64_t dplane = type == LBK_TYPE_IQ2_S ? 80 : type == LBK_TYPE_IQ3_S ? 108 : type == LBK_TYPE_Q4_K ? 140 : 172;
    if (layout != LBK_LAYOUT_PLANAR) return data + bi * bb;
    const uint64_t row = bi / (uint64_t)nb, b = bi % (uint64_t)nb;
    return data + row * planar_row_bytes(bb, nb) + (uint64_t)nb * dplane + b * (two ? 4 : 2);
}

__global__ void scan_scales_kernel(int type, int layout, const uint8_t* data, uint64_t rows, int nb,
                                   unsigned long long* first_bad) {
    const uint64_t nblk = rows * (uint64_t)nb;
    const bool two = type == LBK_TYPE_Q4_K || type == LBK_TYPE_Q5_K;
    for (uint64_t bi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; bi < nblk; bi += (uint64_t)gridDim.x * blockDim.x) {
        const uint8_t* p = scale_ptr(type, layout, data, nb, bi);
        uint32_t d = (uint32_t)p[0] | ((uint32_t)p[1] << 8);
        bool bad = !h_finite(d);
        if (two) bad |= !h_finite((uint32_t)p[2] | ((uint32_t)p[3] << 8));
        if (bad) atomicMin(first_bad, (unsigned long long)bi);
    }
}

__global__ void report_scale_kernel(int type, int layout, const uint8_t* data, uint64_t rows, int nb,
                                    const unsigned long long* first_bad, DeviceStatus* st) {
    unsigned long long bi = *first_bad;
    if (bi == ~0ull) return;
    (void)rows;
    const uint8_t* p = scale_ptr(type, layout, data, nb, bi);
    uint32_t d = (uint32_t)p[0] | ((uint32_t)p[1] << 8);
    uint32_t bits = h_finite(d) ? ((uint32_t)p[2] | ((uint32_t)p[3] << 8)) : d;
    report(st, LBK_NON_FINITE_SCALE, bi, bits);
}

// Replicated shared-memory images of the codebooks: word (entry * 32 + c) =
// entry, for every copy c (see lbk_device.cuh).
__global__ void build_tables_kernel(const uint64_t* iq2s, const uint32_t* iq3s, uint32_t* iq2_img, uint32_t* iq3_img) {
    const int stride = gridDim.x * blockDim.x;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    for (int i = tid; i < kIq2CodeEntries * 32; i += stride) iq2_img[i] = iq2_code_of(iq2s[i >> 5]);
    for (int i = tid; i < kIq3GridEntries * 32; i += stride) iq3_img[i] = iq3s[i >> 5];
}

}  // namespace

cudaError_t launch_build_tables(const uint64_t* iq2s, const uint32_t* iq3s, uint32_t* iq2_img, uint32_t* iq3_img,
                                cudaStream_t stream) {
    build_tables_kernel<<<128, 256, 0, stream>>>(iq2s, iq3s, iq2_img, iq3_img);
    return cudaGetLastError();
}

cudaError_t launch_repack(const RepackArgs& a, cudaStream_t stream) {
    int bb = a.type == LBK_TYPE_IQ2_S ? 82 : a.type == LBK_TYPE_IQ3_S ? 110 : a.type == LBK_TYPE_Q4_K ? 144 : 176;
    uint64_t nblk = a.rows * (uint64_t)a.nb;
    uint64_t grid = (nblk + 255) / 256;
    if (grid > 65535) grid = 65535;
    if (grid < 1) grid = 1;
    repack_kernel<<<(unsigned)grid, 256, 0, stream>>>(a, bb);
    return cudaGetLastError();
}

cudaError_t launch_validate_scales(int type, int layout, const uint8_t* data, uint64_t rows, int nb,
                                   unsigned long long* scratch_min, DeviceStatus* status, cudaStream_t stream) {
    cudaError_t e = cudaMemsetAsync(scratch_min, 0xff, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    uint64_t nblk = rows * (uint64_t)nb;
    uint64_t grid = (nblk + 255) / 256;
    if (grid > 65535) grid = 65535;
    if (grid < 1) grid = 1;
    scan_scales_kernel<<<(unsigned)grid, 256, 0, stream>>>(type, layout, data, rows, nb, scratch_min);
    report_scale_kernel<<<1, 1, 0, stream>>>(type, layout, data, rows, nb, scratch_min, status);
    return cudaGetLastError();
}

}  // namespace lbk
