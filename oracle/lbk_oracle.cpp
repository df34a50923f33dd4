// lbk_oracle.cpp -- CPU restatement of LightBridge's quantized expert path.
//
// TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels and the timed CPU
// baseline. The product never links or calls this file.
//
// Each function cites the reference Rust function it restates (paths inside
// the reference project). Floating-point statements keep the reference's
// operation order; the file is compiled with -ffp-contract=off so no multiply
// is fused into an add (Rust does not contract). expf is the platform libm's,
// as Rust's f32::exp is on Linux.

#include "lbk_oracle.h"
#include "../include/lightbridge_kernels.h"
#include "../lightbridge-engine_b200/csrc/lbk_iq_tables.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

namespace {

constexpr uint64_t kQK = 256;
constexpr uint64_t kQ8Bytes = 292;
constexpr uint64_t kQ8D = 0;
constexpr uint64_t kQ8Qs = 4;
constexpr uint64_t kQ8Sums = 260;

thread_local orc_detail g_detail;

int32_t fail(int32_t status, uint64_t index = 0, uint32_t bits = 0, uint64_t expected = 0,
             uint64_t actual = 0) {
    g_detail.status = status;
    g_detail.index = index;
    g_detail.bits = bits;
    g_detail.expected = expected;
    g_detail.actual = actual;
    return status;
}

int32_t ok() {
    g_detail = orc_detail{};
    return LBK_OK;
}

uint32_t f32_bits(float v) {
    uint32_t b;
    std::memcpy(&b, &v, 4);
    return b;
}

float bits_f32(uint32_t b) {
    float v;
    std::memcpy(&v, &b, 4);
    return v;
}

// Exact IEEE binary16 -> binary32 (the `half` crate's f16::to_f32, pinned by
// bridge-quant-layout/tests/abi.rs:277-300).
float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ffu;
    uint32_t out;
    if (exp == 0) {
        if (man == 0) {
            out = sign;
        } else {
            // subnormal: normalise
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            out = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        out = sign | 0x7f800000u | (man << 13);
    } else {
        out = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    return bits_f32(out);
}

bool half_finite(uint16_t h) { return ((h >> 10) & 0x1f) != 0x1f; }

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
int16_t rdi16(const uint8_t* p) { return (int16_t)rd16(p); }
float rdf32(const uint8_t* p) {
    uint32_t b = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
    return bits_f32(b);
}
float rdf16(const uint8_t* p) { return half_to_float(rd16(p)); }

// nearest_int, q8_k.rs:224-228: round half to even through the 1.5*2^23 magic add.
int32_t nearest_int(float v) {
    float t = v + 12582912.0f;
    int32_t bits = (int32_t)f32_bits(t);
    return (bits & 0x007fffff) - 0x00400000;
}

// layout(), k_quants.rs:34-54
uint64_t block_bytes(int32_t ty) {
    switch (ty) {
        case LBK_TYPE_F32: return 4;
        case LBK_TYPE_Q4_K: return 144;
        case LBK_TYPE_Q5_K: return 176;
        case LBK_TYPE_IQ2_S: return 82;
        case LBK_TYPE_IQ3_S: return 110;
        default: return 0;
    }
}
uint64_t block_elements(int32_t ty) { return ty == LBK_TYPE_F32 ? 1 : kQK; }

bool is_dot_type(int32_t ty) {
    return ty == LBK_TYPE_Q4_K || ty == LBK_TYPE_Q5_K || ty == LBK_TYPE_IQ2_S || ty == LBK_TYPE_IQ3_S;
}

// scale_min, k_quants.rs:231-240
void scale_min(const uint8_t* s, int i, uint8_t* sc, uint8_t* m) {
    if (i < 4) {
        *sc = s[i] & 0x3f;
        *m = s[i + 4] & 0x3f;
    } else {
        *sc = (uint8_t)((s[i + 4] & 0x0f) | ((s[i - 4] >> 6) << 4));
        *m = (uint8_t)((s[i + 4] >> 4) | ((s[i] >> 6) << 4));
    }
}

// validate_scales, k_quants.rs:178-208
int32_t validate_scales(int32_t ty, const uint8_t* enc, uint64_t blocks) {
    uint64_t bb = block_bytes(ty);
    if (ty == LBK_TYPE_F32) return LBK_OK;
    bool two = ty == LBK_TYPE_Q4_K || ty == LBK_TYPE_Q5_K;
    for (uint64_t b = 0; b < blocks; b++) {
        uint16_t d = rd16(enc + b * bb);
        if (!half_finite(d)) return fail(LBK_NON_FINITE_SCALE, b, d);
        if (two) {
            uint16_t dm = rd16(enc + b * bb + 2);
            if (!half_finite(dm)) return fail(LBK_NON_FINITE_SCALE, b, dm);
        }
    }
    return LBK_OK;
}

// ---------------------------------------------------------------- decoders

void decode_q4_k(const uint8_t* e, float* out) {  // k_quants.rs:242-265
    float d = rdf16(e), dmin = rdf16(e + 2);
    const uint8_t* scales = e + 4;
    const uint8_t* q = e + 16;
    for (int g = 0; g < 4; g++) {
        uint8_t s1, m1, s2, m2;
        scale_min(scales, g * 2, &s1, &m1);
        float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        scale_min(scales, g * 2 + 1, &s2, &m2);
        float d2 = d * (float)s2, mm2 = dmin * (float)m2;
        for (int l = 0; l < 32; l++) out[g * 64 + l] = d1 * (float)(q[g * 32 + l] & 0x0f) - mm1;
        for (int l = 0; l < 32; l++) out[g * 64 + 32 + l] = d2 * (float)(q[g * 32 + l] >> 4) - mm2;
    }
}

void decode_q5_k(const uint8_t* e, float* out) {  // k_quants.rs:267-300
    float d = rdf16(e), dmin = rdf16(e + 2);
    const uint8_t* scales = e + 4;
    const uint8_t* qh = e + 16;
    const uint8_t* q = e + 48;
    uint8_t lo = 1, hi = 2;
    for (int g = 0; g < 4; g++) {
        uint8_t s1, m1, s2, m2;
        scale_min(scales, g * 2, &s1, &m1);
        float d1 = d * (float)s1, mm1 = dmin * (float)m1;
        scale_min(scales, g * 2 + 1, &s2, &m2);
        float d2 = d * (float)s2, mm2 = dmin * (float)m2;
        for (int l = 0; l < 32; l++) {
            uint8_t h = (qh[l] & lo) ? 16 : 0;
            out[g * 64 + l] = d1 * (float)((q[g * 32 + l] & 0x0f) + h) - mm1;
        }
        for (int l = 0; l < 32; l++) {
            uint8_t h = (qh[l] & hi) ? 16 : 0;
            out[g * 64 + 32 + l] = d2 * (float)((q[g * 32 + l] >> 4) + h) - mm2;
        }
        lo <<= 2;
        hi <<= 2;
    }
}

void decode_iq2_s(const uint8_t* e, float* out) {  // iq2_s.rs:9-39
    float d = rdf16(e);
    for (int g = 0; g < 8; g++) {
        uint8_t sc = e[74 + g];
        float bs[2] = {d * (0.5f + (float)(sc & 0x0f)) * 0.25f, d * (0.5f + (float)(sc >> 4)) * 0.25f};
        unsigned high = e[66 + g];
        for (int lg = 0; lg < 4; lg++) {
            unsigned low = e[2 + g * 4 + lg];
            unsigned idx = low | ((high << (8 - 2 * lg)) & 0x300);
            uint64_t grid = lbk_iq2s_grid[idx];
            uint8_t signs = e[34 + g * 4 + lg];
            float scale = bs[lg / 2];
            for (int l = 0; l < 8; l++) {
                float sign = (signs & lbk_kmask_iq2xs[l]) == 0 ? 1.0f : -1.0f;
                out[g * 32 + lg * 8 + l] = scale * (float)((grid >> (8 * l)) & 0xff) * sign;
            }
        }
    }
}

void decode_iq3_s(const uint8_t* e, float* out) {  // iq3_s.rs:9-53
    float d = rdf16(e);
    for (int p = 0; p < 4; p++) {
        uint8_t ps = e[106 + p];
        float sc[2] = {d * (float)(1 + 2 * (ps & 0x0f)), d * (float)(1 + 2 * (ps >> 4))};
        for (int h = 0; h < 2; h++) {
            int g = p * 2 + h;
            unsigned high = e[66 + g];
            for (int lg = 0; lg < 4; lg++) {
                unsigned l1 = e[2 + g * 8 + lg * 2], l2 = e[2 + g * 8 + lg * 2 + 1];
                unsigned i1 = l1 | ((high << (8 - 2 * lg)) & 0x100);
                unsigned i2 = l2 | ((high << (7 - 2 * lg)) & 0x100);
                uint32_t g1 = lbk_iq3s_grid[i1], g2 = lbk_iq3s_grid[i2];
                uint8_t signs = e[74 + g * 4 + lg];
                for (int l = 0; l < 4; l++) {
                    float s1 = (signs & lbk_kmask_iq2xs[l]) == 0 ? 1.0f : -1.0f;
                    float s2 = (signs & lbk_kmask_iq2xs[l + 4]) == 0 ? 1.0f : -1.0f;
                    out[g * 32 + lg * 8 + l] = sc[h] * (float)((g1 >> (8 * l)) & 0xff) * s1;
                    out[g * 32 + lg * 8 + l + 4] = sc[h] * (float)((g2 >> (8 * l)) & 0xff) * s2;
                }
            }
        }
    }
}

// ------------------------------------------------------------- scalar dots

// Q4_K / Q5_K lane sums of one block (q8_k.rs:257-312): the 8 per-lane int32
// accumulators and the min correction sum.
void q45_block_ints(int32_t ty, const uint8_t* w, const uint8_t* a, int32_t lane[8], int32_t* min_sum) {
    int8_t q[256];
    if (ty == LBK_TYPE_Q4_K) {
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++) {
                uint8_t p = w[16 + g * 32 + l];
                q[g * 64 + l] = (int8_t)(p & 0x0f);
                q[g * 64 + 32 + l] = (int8_t)(p >> 4);
            }
    } else {
        uint8_t lo = 1, hi = 2;
        for (int g = 0; g < 4; g++) {
            for (int l = 0; l < 32; l++) {
                uint8_t p = w[48 + g * 32 + l];
                uint8_t hb = w[16 + l];
                q[g * 64 + l] = (int8_t)((p & 0x0f) + ((hb & lo) != 0) * 16);
                q[g * 64 + 32 + l] = (int8_t)((p >> 4) + ((hb & hi) != 0) * 16);
            }
            lo <<= 2;
            hi <<= 2;
        }
    }
    uint8_t sc[8], mn[8];
    for (int i = 0; i < 8; i++) scale_min(w + 4, i, &sc[i], &mn[i]);
    int32_t ms = 0;
    for (int g = 0; g < 16; g++) ms += (int32_t)rdi16(a + kQ8Sums + g * 2) * (int32_t)mn[g / 2];
    for (int l = 0; l < 8; l++) lane[l] = 0;
    int off = 0;
    for (int j = 0; j < 8; j++) {
        for (int r = 0; r < 4; r++) {
            for (int l = 0; l < 8; l++) {
                int32_t av = (int8_t)a[kQ8Qs + off + l];
                lane[l] += (int32_t)sc[j] * av * (int32_t)q[off + l];
            }
            off += 8;
        }
    }
    *min_sum = ms;
}

// dot_q4_or_q5_k, q8_k.rs:247-327
float dot_q45(int32_t ty, const uint8_t* w, const uint8_t* q8, uint64_t nb) {
    uint64_t bb = block_bytes(ty);
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sum = 0.0f;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * bb;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        int32_t lane[8], ms;
        q45_block_ints(ty, wb, ab, lane, &ms);
        float dy = rdf32(ab + kQ8D);
        float scale = rdf16(wb) * dy;
        for (int l = 0; l < 8; l++) sums[l] += scale * (float)lane[l];
        float mscale = rdf16(wb + 2) * dy;
        sum -= mscale * (float)ms;
    }
    for (int l = 0; l < 8; l++) sum += sums[l];
    return sum;
}

int32_t iq2s_block_int(const uint8_t* w, const uint8_t* a) {  // q8_k.rs:337-364
    int32_t bsum = 0;
    for (int g = 0; g < 8; g++) {
        uint8_t ps = w[74 + g];
        int32_t s1 = 1 + 2 * (ps & 0x0f), s2 = 1 + 2 * (ps >> 4);
        unsigned high = w[66 + g];
        int32_t sums[2] = {0, 0};
        for (int lg = 0; lg < 4; lg++) {
            unsigned low = w[2 + g * 4 + lg];
            unsigned idx = low | ((high << (8 - 2 * lg)) & 0x300);
            uint64_t grid = lbk_iq2s_grid[idx];
            uint8_t signs = w[34 + g * 4 + lg];
            const uint8_t* act = a + kQ8Qs + g * 32 + lg * 8;
            for (int l = 0; l < 8; l++) {
                int32_t sign = (signs & lbk_kmask_iq2xs[l]) == 0 ? 1 : -1;
                sums[lg / 2] += (int32_t)(int8_t)act[l] * (int32_t)((grid >> (8 * l)) & 0xff) * sign;
            }
        }
        bsum += s1 * sums[0] + s2 * sums[1];
    }
    return bsum;
}

float dot_iq2_s(const uint8_t* w, const uint8_t* q8, uint64_t nb) {  // q8_k.rs:329-370
    float sum = 0.0f;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * 82;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        float scale = rdf16(wb) * rdf32(ab + kQ8D);
        sum += scale * (float)iq2s_block_int(wb, ab);
    }
    return 0.125f * sum;
}

int32_t iq3s_block_int(const uint8_t* w, const uint8_t* a) {  // q8_k.rs:380-428
    int32_t bsum = 0;
    for (int p = 0; p < 4; p++) {
        uint8_t ps = w[106 + p];
        int32_t psc[2] = {2 * (ps & 0x0f) + 1, 2 * (ps >> 4) + 1};
        for (int h = 0; h < 2; h++) {
            int g = p * 2 + h;
            unsigned high = w[66 + g];
            int32_t gs = 0;
            for (int lg = 0; lg < 4; lg++) {
                unsigned l1 = w[2 + g * 8 + lg * 2], l2 = w[2 + g * 8 + lg * 2 + 1];
                unsigned i1 = l1 | ((high << (8 - 2 * lg)) & 0x100);
                unsigned i2 = l2 | ((high << (7 - 2 * lg)) & 0x100);
                uint32_t g1 = lbk_iq3s_grid[i1], g2 = lbk_iq3s_grid[i2];
                uint8_t signs = w[74 + g * 4 + lg];
                const uint8_t* act = a + kQ8Qs + g * 32 + lg * 8;
                for (int l = 0; l < 4; l++) {
                    int32_t s1 = (signs & lbk_kmask_iq2xs[l]) == 0 ? 1 : -1;
                    int32_t s2 = (signs & lbk_kmask_iq2xs[l + 4]) == 0 ? 1 : -1;
                    gs += (int32_t)(int8_t)act[l] * (int32_t)((g1 >> (8 * l)) & 0xff) * s1;
                    gs += (int32_t)(int8_t)act[l + 4] * (int32_t)((g2 >> (8 * l)) & 0xff) * s2;
                }
            }
            bsum += gs * psc[h];
        }
    }
    return bsum;
}

float dot_iq3_s(const uint8_t* w, const uint8_t* q8, uint64_t nb) {  // q8_k.rs:372-434
    float sum = 0.0f;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * 110;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        float scale = rdf16(wb) * rdf32(ab + kQ8D);
        sum += scale * (float)iq3s_block_int(wb, ab);
    }
    return sum;
}

float dot_scalar(int32_t ty, const uint8_t* w, const uint8_t* q8, uint64_t nb) {  // q8_k.rs:163-170
    switch (ty) {
        case LBK_TYPE_Q4_K:
        case LBK_TYPE_Q5_K: return dot_q45(ty, w, q8, nb);
        case LBK_TYPE_IQ2_S: return dot_iq2_s(w, q8, nb);
        default: return dot_iq3_s(w, q8, nb);
    }
}

// --------------------------------------------------------------- AVX2 dots
// Restatement of q8_k.rs:436-731 with the same intrinsic sequence.

__attribute__((target("avx2"))) void lane_sums_i8_32(const int8_t* w, const uint8_t* a, int32_t out[8]) {
    __m256i acc = _mm256_setzero_si256();
    for (int off = 0; off < 32; off += 16) {
        __m128i wi = _mm_loadu_si128((const __m128i*)(w + off));
        __m128i ai = _mm_loadu_si128((const __m128i*)(a + off));
        __m256i w16 = _mm256_cvtepi8_epi16(wi);
        __m256i a16 = _mm256_cvtepi8_epi16(ai);
        __m256i p16 = _mm256_mullo_epi16(w16, a16);
        __m256i lo = _mm256_cvtepi16_epi32(_mm256_castsi256_si128(p16));
        __m256i hi = _mm256_cvtepi16_epi32(_mm256_extracti128_si256(p16, 1));
        acc = _mm256_add_epi32(acc, lo);
        acc = _mm256_add_epi32(acc, hi);
    }
    _mm256_storeu_si256((__m256i*)out, acc);
}

__attribute__((target("avx2"))) int32_t dot_i8_32(const int8_t* w, const uint8_t* a) {
    int32_t l[8];
    lane_sums_i8_32(w, a, l);
    int32_t s = 0;
    for (int i = 0; i < 8; i++) s += l[i];
    return s;
}

__attribute__((target("avx2"))) int32_t dot_i8_16(const int8_t* w, const uint8_t* a) {
    __m128i wi = _mm_loadu_si128((const __m128i*)w);
    __m128i ai = _mm_loadu_si128((const __m128i*)a);
    __m256i p16 = _mm256_mullo_epi16(_mm256_cvtepi8_epi16(wi), _mm256_cvtepi8_epi16(ai));
    __m256i pairs = _mm256_madd_epi16(p16, _mm256_set1_epi16(1));
    int32_t l[8];
    _mm256_storeu_si256((__m256i*)l, pairs);
    int32_t s = 0;
    for (int i = 0; i < 8; i++) s += l[i];
    return s;
}

__attribute__((target("avx2"))) float dot_q45_avx2(int32_t ty, const uint8_t* w, const uint8_t* q8,
                                                   uint64_t nb) {
    uint64_t bb = block_bytes(ty);
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sum = 0.0f;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * bb;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        int8_t q[256];
        if (ty == LBK_TYPE_Q4_K) {
            for (int g = 0; g < 4; g++)
                for (int l = 0; l < 32; l++) {
                    uint8_t p = wb[16 + g * 32 + l];
                    q[g * 64 + l] = (int8_t)(p & 0x0f);
                    q[g * 64 + 32 + l] = (int8_t)(p >> 4);
                }
        } else {
            uint8_t lo = 1, hi = 2;
            for (int g = 0; g < 4; g++) {
                for (int l = 0; l < 32; l++) {
                    uint8_t p = wb[48 + g * 32 + l];
                    uint8_t hb = wb[16 + l];
                    q[g * 64 + l] = (int8_t)((p & 0x0f) + ((hb & lo) != 0) * 16);
                    q[g * 64 + 32 + l] = (int8_t)((p >> 4) + ((hb & hi) != 0) * 16);
                }
                lo <<= 2;
                hi <<= 2;
            }
        }
        uint8_t sc[8], mn[8];
        for (int i = 0; i < 8; i++) scale_min(wb + 4, i, &sc[i], &mn[i]);
        int32_t ms = 0;
        for (int g = 0; g < 16; g++) ms += (int32_t)rdi16(ab + kQ8Sums + g * 2) * (int32_t)mn[g / 2];
        int32_t lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 8; j++) {
            int32_t raw[8];
            lane_sums_i8_32(q + j * 32, ab + kQ8Qs + j * 32, raw);
            for (int l = 0; l < 8; l++) lane[l] += (int32_t)sc[j] * raw[l];
        }
        float dy = rdf32(ab + kQ8D);
        float scale = rdf16(wb) * dy;
        for (int l = 0; l < 8; l++) sums[l] += scale * (float)lane[l];
        float mscale = rdf16(wb + 2) * dy;
        sum -= mscale * (float)ms;
    }
    for (int l = 0; l < 8; l++) sum += sums[l];
    return sum;
}

__attribute__((target("avx2"))) float dot_iq2_s_avx2(const uint8_t* w, const uint8_t* q8, uint64_t nb) {
    float sum = 0.0f;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * 82;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        float scale = rdf16(wb) * rdf32(ab + kQ8D);
        int32_t bsum = 0;
        for (int g = 0; g < 8; g++) {
            uint8_t ps = wb[74 + g];
            int32_t s1 = 1 + 2 * (ps & 0x0f), s2 = 1 + 2 * (ps >> 4);
            unsigned high = wb[66 + g];
            int8_t sg[32];
            for (int lg = 0; lg < 4; lg++) {
                unsigned low = wb[2 + g * 4 + lg];
                unsigned idx = low | ((high << (8 - 2 * lg)) & 0x300);
                uint64_t grid = lbk_iq2s_grid[idx];
                uint8_t signs = wb[34 + g * 4 + lg];
                for (int l = 0; l < 8; l++) {
                    int8_t m = (int8_t)((grid >> (8 * l)) & 0xff);
                    sg[lg * 8 + l] = (signs & lbk_kmask_iq2xs[l]) == 0 ? m : (int8_t)-m;
                }
            }
            const uint8_t* act = ab + kQ8Qs + g * 32;
            int32_t a1 = dot_i8_16(sg, act);
            int32_t a2 = dot_i8_16(sg + 16, act + 16);
            bsum += s1 * a1 + s2 * a2;
        }
        sum += scale * (float)bsum;
    }
    return 0.125f * sum;
}

__attribute__((target("avx2"))) float dot_iq3_s_avx2(const uint8_t* w, const uint8_t* q8, uint64_t nb) {
    float sum = 0.0f;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * 110;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        float scale = rdf16(wb) * rdf32(ab + kQ8D);
        int32_t bsum = 0;
        for (int p = 0; p < 4; p++) {
            uint8_t ps = wb[106 + p];
            int32_t psc[2] = {2 * (ps & 0x0f) + 1, 2 * (ps >> 4) + 1};
            for (int h = 0; h < 2; h++) {
                int g = p * 2 + h;
                unsigned high = wb[66 + g];
                int8_t sg[32];
                for (int lg = 0; lg < 4; lg++) {
                    unsigned l1 = wb[2 + g * 8 + lg * 2], l2 = wb[2 + g * 8 + lg * 2 + 1];
                    unsigned i1 = l1 | ((high << (8 - 2 * lg)) & 0x100);
                    unsigned i2 = l2 | ((high << (7 - 2 * lg)) & 0x100);
                    uint32_t g1 = lbk_iq3s_grid[i1], g2 = lbk_iq3s_grid[i2];
                    uint8_t signs = wb[74 + g * 4 + lg];
                    for (int l = 0; l < 4; l++) {
                        int8_t m1 = (int8_t)((g1 >> (8 * l)) & 0xff), m2 = (int8_t)((g2 >> (8 * l)) & 0xff);
                        sg[lg * 8 + l] = (signs & lbk_kmask_iq2xs[l]) == 0 ? m1 : (int8_t)-m1;
                        sg[lg * 8 + l + 4] = (signs & lbk_kmask_iq2xs[l + 4]) == 0 ? m2 : (int8_t)-m2;
                    }
                }
                bsum += dot_i8_32(sg, ab + kQ8Qs + g * 32) * psc[h];
            }
        }
        sum += scale * (float)bsum;
    }
    return sum;
}

bool have_avx2() { return __builtin_cpu_supports("avx2"); }

float dot_cpu(int32_t ty, const uint8_t* w, const uint8_t* q8, uint64_t nb, int simd) {
    if (simd && have_avx2()) {
        switch (ty) {
            case LBK_TYPE_Q4_K:
            case LBK_TYPE_Q5_K: return dot_q45_avx2(ty, w, q8, nb);
            case LBK_TYPE_IQ2_S: return dot_iq2_s_avx2(w, q8, nb);
            default: return dot_iq3_s_avx2(w, q8, nb);
        }
    }
    return dot_scalar(ty, w, q8, nb);
}

// ------------------------------------------------------------- thread pool
// A bounded pool with dynamic row chunks, standing in for the reference's
// rayon pool (bridge-kernels-cpu/src/lib.rs:75-118).

class Pool {
   public:
    static Pool& get(int threads) {
        static std::mutex mu;
        static std::vector<std::unique_ptr<Pool>> pools;
        std::lock_guard<std::mutex> lock(mu);
        for (auto& p : pools)
            if (p->n_ == threads) return *p;
        pools.emplace_back(new Pool(threads));
        return *pools.back();
    }

    void run(uint64_t count, uint64_t chunk, const std::function<void(uint64_t, uint64_t)>& fn) {
        if (n_ <= 1 || count <= chunk) {
            fn(0, count);
            return;
        }
        std::unique_lock<std::mutex> lock(mu_);
        job_ = &fn;
        count_ = count;
        chunk_ = chunk;
        next_.store(0);
        pending_ = n_ - 1;
        gen_++;
        cv_.notify_all();
        lock.unlock();
        work();
        lock.lock();
        done_cv_.wait(lock, [&] { return pending_ == 0; });
        job_ = nullptr;
    }

    ~Pool() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            stop_ = true;
            gen_++;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }

   private:
    explicit Pool(int n) : n_(n) {
        for (int i = 0; i + 1 < n; i++) threads_.emplace_back([this] { loop(); });
    }

    void work() {
        for (;;) {
            uint64_t s = next_.fetch_add(chunk_);
            if (s >= count_) break;
            uint64_t e = s + chunk_ < count_ ? s + chunk_ : count_;
            (*job_)(s, e);
        }
    }

    void loop() {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lock(mu_);
            cv_.wait(lock, [&] { return gen_ != seen; });
            seen = gen_;
            if (stop_) return;
            lock.unlock();
            work();
            lock.lock();
            if (--pending_ == 0) done_cv_.notify_all();
        }
    }

    int n_;
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(uint64_t, uint64_t)>* job_ = nullptr;
    uint64_t count_ = 0, chunk_ = 1, gen_ = 0;
    std::atomic<uint64_t> next_{0};
    int pending_ = 0;
    bool stop_ = false;
};

int resolve_threads(int threads) {
    if (threads > 0) return threads;
    unsigned h = std::thread::hardware_concurrency();
    return h ? (int)h : 1;
}

void parallel_rows(int threads, uint64_t rows, const std::function<void(uint64_t, uint64_t)>& fn) {
    int t = resolve_threads(threads);
    uint64_t chunk = rows / ((uint64_t)t * 8);
    if (chunk < 1) chunk = 1;
    Pool::get(t).run(rows, chunk, fn);
}

// ------------------------------------------------------------- validation

int32_t matrix_check(const orc_matrix* m) {  // EncodedTensorView::new / PackedMatrix::new, matrix.rs:26-150
    uint64_t bb = block_bytes(m->type);
    if (bb == 0) return fail(LBK_UNSUPPORTED_TYPE, (uint64_t)m->type);
    if (m->input_width == 0 || m->output_width == 0) return fail(LBK_DIMENSION_MISMATCH);
    uint64_t be = block_elements(m->type);
    if (m->input_width % be != 0) return fail(LBK_DIMENSION_MISMATCH, 0, 0, be, m->input_width);
    uint64_t expected = m->input_width / be * bb * m->output_width;
    if (m->bytes != expected) return fail(LBK_ENCODED_LENGTH_MISMATCH, 0, 0, expected, m->bytes);
    return LBK_OK;
}

int32_t check_finite(const float* v, uint64_t n) {
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(v[i])) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(v[i]));
    return LBK_OK;
}

int32_t quantize_impl(const float* x, uint64_t n, uint8_t* out, uint64_t out_len) {
    if (n == 0) return fail(LBK_ZERO_LOGICAL_ELEMENTS);
    if (n % kQK != 0) return fail(LBK_LOGICAL_ELEMENTS_NOT_DIVISIBLE, 0, 0, kQK, n);
    uint64_t nb = n / kQK;
    uint64_t expected = nb * kQ8Bytes;
    if (out_len != expected) return fail(LBK_ENCODED_LENGTH_MISMATCH, 0, 0, expected, out_len);
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(x[i])) return fail(LBK_NON_FINITE_ACTIVATION, i, f32_bits(x[i]));
    for (uint64_t b = 0; b < nb; b++) {
        const float* v = x + b * kQK;
        uint8_t* o = out + b * kQ8Bytes;
        float mx = 0.0f, amax = 0.0f;
        for (uint64_t i = 0; i < kQK; i++) {
            float a = std::fabs(v[i]);
            if (a > amax) {
                amax = a;
                mx = v[i];
            }
        }
        if (amax == 0.0f) {
            std::memset(o, 0, kQ8Bytes);
            continue;
        }
        float iscale = -127.0f / mx;
        for (uint64_t i = 0; i < kQK; i++) {
            int32_t q = nearest_int(iscale * v[i]);
            if (q > 127) q = 127;
            o[kQ8Qs + i] = (uint8_t)(int8_t)q;
        }
        for (int g = 0; g < 16; g++) {
            int32_t s = 0;
            for (int l = 0; l < 16; l++) s += (int8_t)o[kQ8Qs + g * 16 + l];
            int16_t s16 = (int16_t)s;
            o[kQ8Sums + g * 2] = (uint8_t)(s16 & 0xff);
            o[kQ8Sums + g * 2 + 1] = (uint8_t)((uint16_t)s16 >> 8);
        }
        float d = 1.0f / iscale;
        std::memcpy(o + kQ8D, &d, 4);
    }
    return LBK_OK;
}

// validate_vec_dot_q8_k_inner, q8_k.rs:121-161
int32_t dot_validate(int32_t ty, uint64_t w_len, const uint8_t* w, uint64_t q8_len, const uint8_t* q8,
                     uint64_t n) {
    if (!is_dot_type(ty)) return fail(LBK_UNSUPPORTED_TYPE, (uint64_t)ty);
    if (n == 0) return fail(LBK_ZERO_LOGICAL_ELEMENTS);
    if (n % kQK != 0) return fail(LBK_LOGICAL_ELEMENTS_NOT_DIVISIBLE, 0, 0, kQK, n);
    uint64_t nb = n / kQK;
    if (w_len != nb * block_bytes(ty)) return fail(LBK_ENCODED_LENGTH_MISMATCH, 0, 0, nb * block_bytes(ty), w_len);
    if (q8_len != nb * kQ8Bytes) return fail(LBK_ENCODED_LENGTH_MISMATCH, 0, 0, nb * kQ8Bytes, q8_len);
    int32_t st = validate_scales(ty, w, nb);
    if (st) return st;
    for (uint64_t b = 0; b < nb; b++) {
        float d = rdf32(q8 + b * kQ8Bytes);
        if (!std::isfinite(d)) return fail(LBK_NON_FINITE_Q8_SCALE, b, f32_bits(d));
    }
    return LBK_OK;
}

// prepare_llama_q8k, gemv.rs:245-272
int32_t prepare_q8(const orc_matrix* w, const float* x, uint8_t* q8) {
    int32_t st = matrix_check(w);
    if (st) return st;
    st = check_finite(x, w->input_width);
    if (st) return st;
    if (!is_dot_type(w->type)) return fail(LBK_UNSUPPORTED_TYPE, (uint64_t)w->type);
    uint64_t q8_len = w->input_width / kQK * kQ8Bytes;
    st = quantize_impl(x, w->input_width, q8, q8_len);
    if (st) return st;
    uint64_t rb = w->input_width / kQK * block_bytes(w->type);
    for (uint64_t r = 0; r < w->output_width; r++) {
        st = dot_validate(w->type, rb, w->data + r * rb, q8_len, q8, w->input_width);
        if (st) return st;
    }
    return LBK_OK;
}

int32_t gemv_impl(const orc_matrix* w, const float* x, float* y, uint8_t* q8, int simd, int threads,
                  bool accumulate, float scale) {
    int32_t st = prepare_q8(w, x, q8);
    if (st) return st;
    uint64_t nb = w->input_width / kQK;
    uint64_t rb = nb * block_bytes(w->type);
    parallel_rows(threads, w->output_width, [&](uint64_t s, uint64_t e) {
        for (uint64_t r = s; r < e; r++) {
            float d = dot_cpu(w->type, w->data + r * rb, q8, nb, simd);
            if (accumulate)
                y[r] += scale * d;
            else
                y[r] = d;
        }
    });
    return ok();
}

float dot_f32_row(const uint8_t* row, const float* x, uint64_t n) {  // gemv.rs:286-303
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; i++) sum += rdf32(row + i * 4) * x[i];
    return sum;
}

float sigmoid(float v) { return 1.0f / (1.0f + std::exp(-v)); }  // routing.rs:109-111

// Validation of the routed list, moe.rs:282-322
int32_t routed_check(const uint32_t* ids, const float* coefs, uint64_t k, uint64_t expert_count) {
    if (k == 0) return fail(LBK_DIMENSION_MISMATCH, 0, 0, 1, 0);
    for (uint64_t i = 0; i < k; i++) {
        if (!std::isfinite(coefs[i])) return fail(LBK_NON_FINITE_VALUE, 0, f32_bits(coefs[i]));
        if (i > 0) {
            if (ids[i] == ids[i - 1]) return fail(LBK_DUPLICATE_ROUTED_EXPERT, ids[i]);
            if (ids[i] < ids[i - 1]) return fail(LBK_ROUTED_EXPERT_ORDER, ids[i], 0, ids[i - 1], ids[i]);
        }
        if (ids[i] >= expert_count) return fail(LBK_INVALID_PARAMETER, ids[i]);
    }
    return LBK_OK;
}

// swiglu_project_into / expert_swiglu_accumulate_into (activation.rs:65-144)
// for one expert: h = swiglu(gate x, up x); out (=|+=) coef * down h.
int32_t expert_run(const orc_expert* e, const float* x, float* out, bool accumulate, float coef, int simd,
                   int threads) {
    uint64_t hidden = e->gate.output_width;
    std::vector<float> gate(hidden), up(hidden);
    std::vector<uint8_t> q8(e->gate.input_width / kQK * kQ8Bytes);
    int32_t st = gemv_impl(&e->gate, x, gate.data(), q8.data(), simd, threads, false, 0.0f);
    if (st) return st;
    st = gemv_impl(&e->up, x, up.data(), q8.data(), simd, threads, false, 0.0f);
    if (st) return st;
    st = orc_swiglu(gate.data(), up.data(), hidden);
    if (st) return st;
    std::vector<uint8_t> q8h(e->down.input_width / kQK * kQ8Bytes);
    if (accumulate) {
        if (!std::isfinite(coef)) return fail(LBK_NON_FINITE_VALUE, 0, f32_bits(coef));
        st = check_finite(out, e->down.output_width);
        if (st) return st;
        return gemv_impl(&e->down, gate.data(), out, q8h.data(), simd, threads, true, coef);
    }
    return gemv_impl(&e->down, gate.data(), out, q8h.data(), simd, threads, false, 0.0f);
}

}  // namespace

extern "C" {

void orc_last_detail(orc_detail* out) { *out = g_detail; }
uint64_t orc_block_bytes(int32_t type) { return block_bytes(type); }

int32_t orc_quantize_q8k(const float* x, uint64_t n, uint8_t* out, uint64_t out_len) {
    int32_t st = quantize_impl(x, n, out, out_len);
    return st ? st : ok();
}

int32_t orc_decode_row(int32_t type, const uint8_t* enc, uint64_t enc_len, uint64_t n, float* out,
                       uint64_t out_len) {
    uint64_t bb = block_bytes(type);
    if (bb == 0) return fail(LBK_UNSUPPORTED_TYPE, (uint64_t)type);
    if (n == 0) return fail(LBK_ZERO_LOGICAL_ELEMENTS);
    uint64_t be = block_elements(type);
    if (n % be != 0) return fail(LBK_LOGICAL_ELEMENTS_NOT_DIVISIBLE, 0, 0, be, n);
    uint64_t nb = n / be;
    if (enc_len != nb * bb) return fail(LBK_ENCODED_LENGTH_MISMATCH, 0, 0, nb * bb, enc_len);
    if (out_len != nb * be) return fail(LBK_OUTPUT_LENGTH_MISMATCH, 0, 0, nb * be, out_len);
    int32_t st = validate_scales(type, enc, nb);
    if (st) return st;
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* e = enc + b * bb;
        float* o = out + b * be;
        switch (type) {
            case LBK_TYPE_F32: o[0] = rdf32(e); break;
            case LBK_TYPE_Q4_K: decode_q4_k(e, o); break;
            case LBK_TYPE_Q5_K: decode_q5_k(e, o); break;
            case LBK_TYPE_IQ2_S: decode_iq2_s(e, o); break;
            default: decode_iq3_s(e, o); break;
        }
    }
    return ok();
}

int32_t orc_vec_dot(int32_t type, const uint8_t* w, uint64_t w_len, const uint8_t* q8, uint64_t q8_len,
                    uint64_t n, int32_t simd, float* result) {
    int32_t st = dot_validate(type, w_len, w, q8_len, q8, n);
    if (st) return st;
    *result = dot_cpu(type, w, q8, n / kQK, simd);
    return ok();
}

int32_t orc_block_sums(int32_t type, const uint8_t* w, const uint8_t* q8, uint64_t n, int32_t* sums) {
    if (!is_dot_type(type)) return fail(LBK_UNSUPPORTED_TYPE, (uint64_t)type);
    uint64_t nb = n / kQK, bb = block_bytes(type);
    for (uint64_t b = 0; b < nb; b++) {
        const uint8_t* wb = w + b * bb;
        const uint8_t* ab = q8 + b * kQ8Bytes;
        if (type == LBK_TYPE_IQ2_S) {
            sums[b] = iq2s_block_int(wb, ab);
        } else if (type == LBK_TYPE_IQ3_S) {
            sums[b] = iq3s_block_int(wb, ab);
        } else {
            q45_block_ints(type, wb, ab, sums + b * 9, sums + b * 9 + 8);
        }
    }
    return ok();
}

int32_t orc_gemv(const orc_matrix* w, const float* x, float* y, uint8_t* q8_scratch, int32_t simd,
                 int32_t threads) {
    return gemv_impl(w, x, y, q8_scratch, simd, threads, false, 0.0f);
}

int32_t orc_gemv_accumulate_scaled(const orc_matrix* w, const float* x, float* y, float scale,
                                   uint8_t* q8_scratch, int32_t simd, int32_t threads) {
    if (!std::isfinite(scale)) return fail(LBK_NON_FINITE_VALUE, 0, f32_bits(scale));
    int32_t st = matrix_check(w);
    if (st) return st;
    st = check_finite(y, w->output_width);
    if (st) return st;
    return gemv_impl(w, x, y, q8_scratch, simd, threads, true, scale);
}

int32_t orc_gemv_f32(const orc_matrix* w, const float* x, float* y, int32_t threads) {
    if (w->type != LBK_TYPE_F32) return fail(LBK_UNSUPPORTED_TYPE, (uint64_t)w->type);
    int32_t st = matrix_check(w);
    if (st) return st;
    st = check_finite(x, w->input_width);
    if (st) return st;
    uint64_t n = w->input_width;
    for (uint64_t r = 0; r < w->output_width; r++)  // prepare_dequant: weights must be finite
        for (uint64_t i = 0; i < n; i++) {
            float v = rdf32(w->data + (r * n + i) * 4);
            if (!std::isfinite(v)) return fail(LBK_NON_FINITE_VALUE, r * n + i, f32_bits(v));
        }
    parallel_rows(threads, w->output_width, [&](uint64_t s, uint64_t e) {
        for (uint64_t r = s; r < e; r++) y[r] = dot_f32_row(w->data + r * n * 4, x, n);
    });
    return ok();
}

int32_t orc_route_experts(const float* logits, const float* bias, uint64_t expert_count, uint64_t k,
                          float weight_scale, uint32_t* ids, float* coefs) {
    if (k == 0 || k > expert_count) return fail(LBK_ROUTING_TOPK, 0, 0, expert_count, k);
    if (!std::isfinite(weight_scale)) return fail(LBK_NON_FINITE_ROUTING_VALUE, 0, f32_bits(weight_scale));
    for (uint64_t i = 0; i < expert_count; i++) {
        if (!std::isfinite(logits[i])) return fail(LBK_NON_FINITE_ROUTING_VALUE, i, f32_bits(logits[i]));
        if (!std::isfinite(bias[i])) return fail(LBK_NON_FINITE_ROUTING_VALUE, i, f32_bits(bias[i]));
        float score = sigmoid(logits[i]) + bias[i];
        if (!std::isfinite(score)) return fail(LBK_NON_FINITE_ROUTING_VALUE, i, f32_bits(score));
    }
    struct Cand {
        uint32_t id;
        float score, weight;
    };
    std::vector<Cand> c(expert_count);
    for (uint64_t i = 0; i < expert_count; i++) {
        float w = sigmoid(logits[i]);
        c[i] = Cand{(uint32_t)i, w + bias[i], w};
    }
    // Descending score, ties to ascending ID: a total order, so any correct
    // sort gives the reference's sort_unstable_by result.
    std::sort(c.begin(), c.end(), [](const Cand& a, const Cand& b) {
        if (a.score != b.score) return a.score > b.score;
        return a.id < b.id;
    });
    float wsum = 0.0f;
    for (uint64_t i = 0; i < k; i++) wsum += c[i].weight;
    const float floor = 0.000061035156f;  // 2^-14, routing.rs:5
    wsum = wsum < floor ? floor : wsum;   // f32::max with a finite sum
    std::vector<std::pair<uint32_t, float>> sel(k);
    for (uint64_t i = 0; i < k; i++) sel[i] = {c[i].id, c[i].weight / wsum * weight_scale};
    std::sort(sel.begin(), sel.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    for (uint64_t i = 0; i < k; i++) {
        ids[i] = sel[i].first;
        coefs[i] = sel[i].second;
    }
    return ok();
}

int32_t orc_swiglu(float* gate, const float* up, uint64_t n) {
    // apply_swiglu, activation.rs:170-178. The reference rejects after writing
    // earlier lanes (its caller discards the scratch); same here.
    for (uint64_t i = 0; i < n; i++) {
        float g = gate[i];
        float act = g / (1.0f + std::exp(-g));
        float v = act * up[i];
        if (!std::isfinite(v)) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(v));
        gate[i] = v;
    }
    return LBK_OK;
}

int32_t orc_moe_routed(const orc_expert* experts, uint64_t expert_count, const orc_expert* shared,
                       const uint32_t* ids, const float* coefs, uint64_t k, const float* x, float* out,
                       int32_t preflight, int32_t simd, int32_t threads) {
    int32_t st = routed_check(ids, coefs, k, expert_count);
    if (st) return st;
    uint64_t n_out = shared->down.output_width;
    if (preflight) {  // moe.rs:315-329: every expert once into scratch
        std::vector<float> scratch(n_out);
        for (uint64_t i = 0; i < k; i++) {
            st = expert_run(&experts[ids[i]], x, scratch.data(), false, 0.0f, simd, threads);
            if (st) return st;
        }
        st = expert_run(shared, x, scratch.data(), false, 0.0f, simd, threads);
        if (st) return st;
    }
    for (uint64_t i = 0; i < n_out; i++) out[i] = 0.0f;  // moe.rs:331
    for (uint64_t i = 0; i < k; i++) {
        st = expert_run(&experts[ids[i]], x, out, true, coefs[i], simd, threads);
        if (st) return st;
    }
    st = expert_run(shared, x, out, true, 1.0f, simd, threads);
    return st ? st : ok();
}

int32_t orc_moe_token(const orc_expert* experts, uint64_t expert_count, const orc_expert* shared,
                      const orc_matrix* router, const float* bias, uint64_t k, float weight_scale,
                      const float* x, float* out, uint32_t* ids, float* coefs, int32_t preflight,
                      int32_t simd, int32_t threads) {
    std::vector<float> logits(router->output_width);
    int32_t st = orc_gemv_f32(router, x, logits.data(), threads);
    if (st) return st;
    st = orc_route_experts(logits.data(), bias, expert_count, k, weight_scale, ids, coefs);
    if (st) return st;
    return orc_moe_routed(experts, expert_count, shared, ids, coefs, k, x, out, preflight, simd, threads);
}

int32_t orc_rms_norm(const float* input, uint64_t n, const float* weight, uint64_t weight_len, float epsilon,
                     float* out, uint64_t out_len) {
    // validate_norm_call (norm.rs:102-114) -> validate_norm_lengths (:116-131),
    // validate_epsilon (:133-142), then the input and weight values
    if (n == 0) return fail(LBK_INVALID_PARAMETER);
    if (weight_len != n) return fail(LBK_DIMENSION_MISMATCH, 0, 0, n, weight_len);
    if (out_len != n) return fail(LBK_DIMENSION_MISMATCH, 0, 0, n, out_len);
    if (!std::isfinite(epsilon)) return fail(LBK_NON_FINITE_VALUE, 0, f32_bits(epsilon));
    if (!(epsilon > 0.0f)) return fail(LBK_INVALID_PARAMETER);
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(input[i])) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(input[i]));
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(weight[i])) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(weight[i]));
    // rms_scale (:144-153): one f32 chain of squares, f32 mean, 1 / sqrt(mean + eps)
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; i++) sum += input[i] * input[i];  // -ffp-contract=off: no fused multiply-add
    const float mean = sum / (float)n;
    const float scale = 1.0f / std::sqrt(mean + epsilon);
    if (!std::isfinite(scale)) return fail(LBK_NON_FINITE_VALUE, 0, f32_bits(scale));
    for (uint64_t i = 0; i < n; i++) {
        const float v = input[i] * scale * weight[i];
        if (!std::isfinite(v)) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(v));
    }
    for (uint64_t i = 0; i < n; i++) out[i] = input[i] * scale * weight[i];
    return ok();
}

int32_t orc_residual_add(float* dest, uint64_t n, const float* src, uint64_t src_len) {
    if (src_len != n) return fail(LBK_DIMENSION_MISMATCH, 0, 0, n, src_len);
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(dest[i])) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(dest[i]));
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(src[i])) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(src[i]));
    for (uint64_t i = 0; i < n; i++) {
        const float v = dest[i] + src[i];
        if (!std::isfinite(v)) return fail(LBK_NON_FINITE_VALUE, i, f32_bits(v));
    }
    for (uint64_t i = 0; i < n; i++) dest[i] += src[i];
    return ok();
}

float orc_f16_to_f32(uint16_t bits) { return half_to_float(bits); }
int32_t orc_nearest_int(float v) { return nearest_int(v); }
float orc_expf(float v) { return std::exp(v); }
int32_t orc_hw_threads(void) { return resolve_threads(0); }

const uint8_t* orc_table_bytes(int32_t which, uint64_t* len) {
    switch (which) {
        case 0: *len = sizeof(lbk_kmask_iq2xs); return lbk_kmask_iq2xs;
        case 1: *len = sizeof(lbk_iq2s_grid); return (const uint8_t*)lbk_iq2s_grid;
        default: *len = sizeof(lbk_iq3s_grid); return (const uint8_t*)lbk_iq3s_grid;
    }
}

}  // extern "C"
