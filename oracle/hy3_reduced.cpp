// hy3_reduced.cpp -- CPU restatement of the reference's reduced two-block Hy3
// model pieces that sit around the expert path: its deterministic weights,
// the DequantF32 GEMV mode, per-head RMSNorm, NeoX YaRN RoPE, one-token causal
// GQA attention and softmax.
//
// TEST INFRASTRUCTURE ONLY: with the functions of lbk_oracle.cpp these run the
// reduced model token by token so that the reference's named SHA-256 outputs
// (bridge-test-model/tests/fixtures/hy3-oracle-v1.json, checked by
// bridge-test-model/tests/hy3_logits.rs:69-112) pin the oracle, and the
// device path can be dropped in for the GEMVs, norms, routing and experts.
// The product never links or calls this file.
//
// Floating-point statements keep the reference's operation order; the file is
// compiled with -ffp-contract=off -fno-builtin so that no multiply is fused and
// no libm call is folded at compile time: expf, sinf, cosf, logf, powf and
// sqrtf are the platform libm's at run time, as Rust's f32 methods are on
// Linux.

#include "lbk_oracle.h"
#include "../include/lightbridge_kernels.h"

#include <cmath>
#include <cstring>
#include <vector>

namespace {

uint32_t bits_of(float v) {
    uint32_t b;
    std::memcpy(&b, &v, 4);
    return b;
}

// xorshift64, bridge-test-model/src/hy3.rs:758-762.
uint64_t xorshift64(uint64_t v) {
    v ^= v << 13;
    v ^= v >> 7;
    return v ^ (v << 17);
}

bool finite_all(const float* v, uint64_t n, uint64_t* bad) {
    for (uint64_t i = 0; i < n; i++)
        if (!std::isfinite(v[i])) {
            *bad = i;
            return false;
        }
    return true;
}

// rms_scale, bridge-kernels-reference/src/norm.rs:144-153.
float rms_scale(const float* v, uint64_t n, float eps) {
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; i++) sum += v[i] * v[i];
    float mean = sum / (float)n;
    return 1.0f / sqrtf(mean + eps);
}

uint64_t row_bytes_of(const orc_matrix* w) { return w->input_width / 256 * orc_block_bytes(w->type); }

// dot_dequant_row, bridge-kernels-reference/src/gemv.rs:305-328: one f32
// chain over the decoded row, block after block.
int32_t dequant_dots(const orc_matrix* w, const float* x, std::vector<float>& dots) {
    const uint64_t n = w->input_width, rb = row_bytes_of(w);
    std::vector<float> row(n);
    dots.assign(w->output_width, 0.0f);
    // prepare_dequant (gemv.rs:215-243): every decoded weight must be finite
    // before any output is computed.
    for (uint64_t r = 0; r < w->output_width; r++) {
        int32_t st = orc_decode_row(w->type, w->data + r * rb, rb, n, row.data(), n);
        if (st) return st;
        uint64_t bad;
        if (!finite_all(row.data(), n, &bad)) return LBK_NON_FINITE_VALUE;
        float sum = 0.0f;
        for (uint64_t i = 0; i < n; i++) sum += row[i] * x[i];
        dots[r] = sum;
    }
    return LBK_OK;
}

int32_t dequant_check(const orc_matrix* w, const float* x) {
    if (w->input_width == 0 || w->input_width % 256 != 0) return LBK_DIMENSION_MISMATCH;
    if (orc_block_bytes(w->type) == 0) return LBK_UNSUPPORTED_TYPE;
    if (w->bytes != row_bytes_of(w) * w->output_width) return LBK_DIMENSION_MISMATCH;
    uint64_t bad;
    if (!finite_all(x, w->input_width, &bad)) return LBK_NON_FINITE_VALUE;
    return LBK_OK;
}

}  // namespace

extern "C" {

// f16::from_f32 of the `half` crate (the reduced model's scale encoding,
// hy3.rs:104-108): IEEE binary32 -> binary16, round to nearest, ties to even,
// subnormals and overflow to infinity included.
uint16_t orc_f32_to_f16(float v) {
    const uint32_t x = bits_of(v);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u)  // infinity, or NaN kept quiet with its top payload bits
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u | ((a >> 13) & 0x3ffu) : 0u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // >= 65520 rounds to infinity
    const int e = (int)(a >> 23) - 127;
    if (e >= -14) {  // normal binary16: drop 13 mantissa bits
        const uint32_t mant = a & 0x7fffffu;
        uint32_t h = ((uint32_t)(e + 15) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  // a carry moves into the exponent
        return (uint16_t)(sign | h);
    }
    if (e < -25) return (uint16_t)sign;  // below half the smallest subnormal
    // subnormal: the value in units of 2^-24 is the 24-bit significand >> (-e - 1)
    const uint32_t mant = (a & 0x7fffffu) | 0x800000u;
    const uint32_t s = (uint32_t)(-e - 1);  // 14 .. 24
    uint32_t h = mant >> s;
    const uint32_t rem = mant & ((1u << s) - 1u), half = 1u << (s - 1u);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

// OwnedMatrix::quantized, hy3.rs:68-117: every block's bytes from one
// xorshift64 stream seeded with seed | 1 (byte = state >> 24), then d (and
// dmin for Q4_K / Q5_K) overwritten with a small magnitude that cycles with
// row + block + (seed & 7).
int32_t orc_hy3_fill_matrix(int32_t type, uint64_t input_width, uint64_t output_width, uint64_t seed, uint8_t* out,
                            uint64_t out_len) {
    const uint64_t bb = orc_block_bytes(type);
    if (bb == 0 || type == LBK_TYPE_F32) return LBK_UNSUPPORTED_TYPE;
    if (input_width == 0 || input_width % 256 != 0) return LBK_DIMENSION_MISMATCH;
    const uint64_t blocks = input_width / 256, rb = blocks * bb;
    if (out_len != rb * output_width) return LBK_DIMENSION_MISMATCH;
    uint64_t state = seed | 1u;
    for (uint64_t row = 0; row < output_width; row++)
        for (uint64_t b = 0; b < blocks; b++) {
            uint8_t* enc = out + row * rb + b * bb;
            for (uint64_t i = 0; i < bb; i++) {
                state = xorshift64(state);
                enc[i] = (uint8_t)(state >> 24);
            }
            const float magnitude = 0.00035f + (float)((row + b + (seed & 7u)) % 11u) * 0.000025f;
            const uint16_t d = orc_f32_to_f16(magnitude);
            enc[0] = (uint8_t)(d & 0xffu);
            enc[1] = (uint8_t)(d >> 8);
            if (type == LBK_TYPE_Q4_K || type == LBK_TYPE_Q5_K) {
                const uint16_t m = orc_f32_to_f16(magnitude * 0.125f);
                enc[2] = (uint8_t)(m & 0xffu);
                enc[3] = (uint8_t)(m >> 8);
            }
        }
    return LBK_OK;
}

// embeddings(), hy3.rs:731-740: n values from one xorshift64 stream.
void orc_hy3_embeddings(float* out, uint64_t n) {
    uint64_t state = 0x9e3779b97f4a7c15ull;
    for (uint64_t i = 0; i < n; i++) {
        state = xorshift64(state);
        const float centered = (float)((uint32_t)(state >> 40) & 0xffffu) / 65535.0f - 0.5f;
        out[i] = centered * 0.5f;
    }
}

// norm_weights(), hy3.rs:742-746.
void orc_hy3_norm_weights(uint64_t length, uint64_t seed, float* out) {
    for (uint64_t i = 0; i < length; i++) out[i] = 0.95f + (float)((i * 17u + seed) % 101u) * 0.001f;
}

// gemv_dequant_f32_into, gemv.rs:33-41 (prepare_dequant :215-243,
// compute_dequant_into :274-284).
int32_t orc_gemv_dequant(const orc_matrix* w, const float* x, float* y) {
    int32_t st = dequant_check(w, x);
    if (st) return st;
    std::vector<float> dots;
    if ((st = dequant_dots(w, x, dots))) return st;
    std::memcpy(y, dots.data(), dots.size() * sizeof(float));
    return LBK_OK;
}

// gemv_accumulate_scaled_into in DequantF32 mode, gemv.rs:117-121 and :138-144:
// y[r] += scale * dot_dequant_row(r).
int32_t orc_gemv_dequant_accumulate_scaled(const orc_matrix* w, const float* x, float* y, float scale) {
    if (!std::isfinite(scale)) return LBK_NON_FINITE_VALUE;
    uint64_t bad;
    if (!finite_all(y, w->output_width, &bad)) return LBK_NON_FINITE_VALUE;
    int32_t st = dequant_check(w, x);
    if (st) return st;
    std::vector<float> dots;
    if ((st = dequant_dots(w, x, dots))) return st;
    for (uint64_t r = 0; r < w->output_width; r++) y[r] += scale * dots[r];
    return LBK_OK;
}

// weighted_head_rms_norm_in_place, norm.rs:36-81: each head_dim chunk scaled
// by its own rms_scale and the shared weight; nothing written unless every
// output is finite.
int32_t orc_head_rms_norm(float* values, uint64_t n, const float* weight, uint64_t head_dim, float eps) {
    if (head_dim == 0) return LBK_INVALID_PARAMETER;
    if (n % head_dim != 0) return LBK_DIMENSION_MISMATCH;
    if (!std::isfinite(eps)) return LBK_NON_FINITE_VALUE;
    if (eps <= 0.0f) return LBK_INVALID_PARAMETER;
    uint64_t bad;
    if (!finite_all(values, n, &bad) || !finite_all(weight, head_dim, &bad)) return LBK_NON_FINITE_VALUE;
    for (uint64_t h = 0; h < n; h += head_dim) {
        const float scale = rms_scale(values + h, head_dim, eps);
        if (!std::isfinite(scale)) return LBK_NON_FINITE_VALUE;
        for (uint64_t i = 0; i < head_dim; i++)
            if (!std::isfinite(values[h + i] * scale * weight[i])) return LBK_NON_FINITE_VALUE;
    }
    for (uint64_t h = 0; h < n; h += head_dim) {
        const float scale = rms_scale(values + h, head_dim, eps);
        for (uint64_t i = 0; i < head_dim; i++) values[h + i] = values[h + i] * scale * weight[i];
    }
    return LBK_OK;
}

// apply_neox_yarn_rope_in_place, rope.rs:121-190, with correction_dimensions
// (:192-204) and yarn_ramp (:206-209): pair i of each head is (i, i + d/2);
// the angle runs from the position by theta_scale = base^(-2/d) per pair,
// interpolated by the frequency scale and mixed back toward extrapolation by
// the YaRN ramp; cos and sin are scaled by the YaRN magnitude.
int32_t orc_rope_neox_yarn(float* values, uint64_t head_count, uint64_t position, const orc_rope* p) {
    if (p->head_dim == 0 || p->head_dim % 2 != 0) return LBK_INVALID_PARAMETER;
    if (p->context_length == 0 || p->original_context == 0) return LBK_INVALID_PARAMETER;
    const float fields[6] = {p->base, p->freq_scale, p->ext_factor, p->attn_factor, p->beta_fast, p->beta_slow};
    for (float f : fields)
        if (!std::isfinite(f)) return LBK_NON_FINITE_VALUE;
    if (p->base <= 0.0f || p->freq_scale <= 0.0f || p->ext_factor < 0.0f || p->attn_factor <= 0.0f ||
        p->beta_fast <= 0.0f || p->beta_slow <= 0.0f)
        return LBK_INVALID_PARAMETER;
    if (position >= p->context_length) return LBK_INVALID_PARAMETER;  // KernelError::PositionOutOfRange
    const uint64_t d = p->head_dim, n = head_count * d;
    uint64_t bad;
    if (!finite_all(values, n, &bad)) return LBK_NON_FINITE_VALUE;

    const float pi = 3.14159265358979323846f;
    auto correction = [&](float rotations) {
        return (float)d * logf((float)p->original_context / (rotations * 2.0f * pi)) / (2.0f * logf(p->base));
    };
    const float low = fmaxf(floorf(correction(p->beta_fast)), 0.0f);
    const float high = fminf(ceilf(correction(p->beta_slow)), (float)d - 1.0f);
    const float theta_scale = powf(p->base, -2.0f / (float)d);
    const float magnitude =
        p->ext_factor == 0.0f ? p->attn_factor : p->attn_factor * (1.0f + 0.1f * logf(1.0f / p->freq_scale));
    const uint64_t half = d / 2;
    auto ramp = [&](uint64_t i0) {
        float t = ((float)(i0 / 2) - low) / fmaxf(high - low, 0.001f);
        t = t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
        return 1.0f - t;
    };
    for (int pass = 0; pass < 2; pass++) {  // pass 0 validates every output, pass 1 writes
        for (uint64_t h = 0; h < n; h += d) {
            float* head = values + h;
            float theta_extrap = (float)position;
            for (uint64_t pair = 0; pair < half; pair++) {
                const float theta_interp = p->freq_scale * theta_extrap;
                const float mix = ramp(pair * 2) * p->ext_factor;
                const float theta = theta_interp * (1.0f - mix) + theta_extrap * mix;
                const float c = cosf(theta) * magnitude, s = sinf(theta) * magnitude;
                const float first = head[pair], second = head[pair + half];
                const float a = first * c - second * s, b = first * s + second * c;
                if (pass == 0) {
                    if (!std::isfinite(a) || !std::isfinite(b)) return LBK_NON_FINITE_VALUE;
                } else {
                    head[pair] = a;
                    head[pair + half] = b;
                }
                theta_extrap *= theta_scale;
            }
        }
    }
    return LBK_OK;
}

// causal_gqa_attention_into for one token, attention.rs:28-87: query head q
// reads KV head q / (q_heads / kv_heads); scores over the `stored` cached
// tokens plus this token, each a sequential dot times 1/sqrt(dim); a stable
// softmax; each output lane a sequential sum of (weight / denominator) *
// value. cache_keys / cache_values hold [token][kv_head][dim] rows; the caller
// appends this token's keys and values afterwards (cache.append_tokens).
int32_t orc_gqa_attention(const float* cache_keys, const float* cache_values, uint64_t stored, uint64_t q_heads,
                          uint64_t kv_heads, uint64_t dim, const float* q, const float* k, const float* v,
                          float* out) {
    if (q_heads == 0 || kv_heads == 0 || q_heads % kv_heads != 0 || dim == 0) return LBK_INVALID_PARAMETER;
    uint64_t bad;
    if (!finite_all(q, q_heads * dim, &bad) || !finite_all(k, kv_heads * dim, &bad) ||
        !finite_all(v, kv_heads * dim, &bad))
        return LBK_NON_FINITE_VALUE;
    const uint64_t per = q_heads / kv_heads, tokens = stored + 1;
    const float scale = 1.0f / sqrtf((float)dim);
    std::vector<float> scores(tokens), staged(q_heads * dim);
    auto key_row = [&](uint64_t t, uint64_t h) { return t < stored ? cache_keys + (t * kv_heads + h) * dim : k + h * dim; };
    auto value_row = [&](uint64_t t, uint64_t h) {
        return t < stored ? cache_values + (t * kv_heads + h) * dim : v + h * dim;
    };
    for (uint64_t qh = 0; qh < q_heads; qh++) {
        const uint64_t kvh = qh / per;
        const float* query = q + qh * dim;
        for (uint64_t t = 0; t < tokens; t++) {
            const float* key = key_row(t, kvh);
            float dot = 0.0f;
            for (uint64_t i = 0; i < dim; i++) dot += query[i] * key[i];
            scores[t] = dot * scale;
            if (!std::isfinite(scores[t])) return LBK_NON_FINITE_VALUE;
        }
        float maximum = -INFINITY;
        for (uint64_t t = 0; t < tokens; t++) maximum = fmaxf(maximum, scores[t]);
        float denominator = 0.0f;
        for (uint64_t t = 0; t < tokens; t++) {
            scores[t] = expf(scores[t] - maximum);
            denominator += scores[t];
        }
        if (!std::isfinite(denominator)) return LBK_NON_FINITE_VALUE;
        for (uint64_t lane = 0; lane < dim; lane++) {
            float attended = 0.0f;
            for (uint64_t t = 0; t < tokens; t++) attended += (scores[t] / denominator) * value_row(t, kvh)[lane];
            if (!std::isfinite(attended)) return LBK_NON_FINITE_VALUE;
            staged[qh * dim + lane] = attended;
        }
    }
    std::memcpy(out, staged.data(), staged.size() * sizeof(float));
    return LBK_OK;
}

// softmax_into, softmax.rs:5-53 (every lane unmasked).
int32_t orc_softmax(const float* logits, uint64_t n, float* out) {
    uint64_t bad;
    if (!finite_all(logits, n, &bad)) return LBK_NON_FINITE_VALUE;
    if (n == 0) return LBK_OK;
    float maximum = -INFINITY;
    for (uint64_t i = 0; i < n; i++) maximum = fmaxf(maximum, logits[i]);
    float sum = 0.0f;
    for (uint64_t i = 0; i < n; i++) sum += expf(logits[i] - maximum);
    if (!std::isfinite(sum)) return LBK_NON_FINITE_VALUE;
    if (sum == 0.0f) return LBK_INVALID_PARAMETER;
    for (uint64_t i = 0; i < n; i++) out[i] = expf(logits[i] - maximum) / sum;
    return LBK_OK;
}

}  // extern "C"
