/*
 * lbk_oracle.h -- CPU restatement of the reference's quantized expert path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA kernels
 * are compared against, and the timed CPU baseline ("port" of the reference's
 * AVX2 path). Nothing in the product links, loads or calls it; only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg
 * may use it.
 *
 * The reference (KB01111/LightBridge-Engine) is a Rust workspace that cannot
 * be compiled in this environment (no cargo / rustc), so each function here
 * restates the cited Rust function step by step, in the same f32 operation
 * order, compiled with -ffp-contract=off -fno-fast-math (Rust never contracts
 * a*b+c into an FMA). Parity of this restatement is pinned by the reference's
 * own golden vectors (crates/bridge-quant-layout/tests/fixtures/, copied to
 * tests/golden/) and its table SHA-256 locks.
 *
 * Status codes are the lbk_status values of include/lightbridge_kernels.h.
 */
#ifndef LBK_ORACLE_H
#define LBK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_detail {
    int32_t status;
    uint64_t index;
    uint32_t bits;
    uint64_t expected;
    uint64_t actual;
} orc_detail;

typedef struct orc_matrix {
    int32_t type;          /* GGML discriminant */
    uint64_t input_width;
    uint64_t output_width;
    const uint8_t* data;   /* GGUF layout, output_width rows */
    uint64_t bytes;
} orc_matrix;

typedef struct orc_expert {
    orc_matrix gate, up, down;
} orc_expert;

void orc_last_detail(orc_detail* out);
uint64_t orc_block_bytes(int32_t type);

/* q8_k.rs:16-76 */
int32_t orc_quantize_q8k(const float* x, uint64_t n, uint8_t* out, uint64_t out_len);
/* k_quants.rs:71-105 with the block decoders k_quants.rs:242-300, iq2_s.rs:9-39, iq3_s.rs:9-53 */
int32_t orc_decode_row(int32_t type, const uint8_t* enc, uint64_t enc_len, uint64_t n, float* out,
                       uint64_t out_len);
/* vec_dot_q8_k (simd=0, q8_k.rs:80-89) / vec_dot_q8_k_cpu (simd=1, :103-119) */
int32_t orc_vec_dot(int32_t type, const uint8_t* w, uint64_t w_len, const uint8_t* q8, uint64_t q8_len,
                    uint64_t n, int32_t simd, float* result);
/* Per-super-block int32 sums feeding the f32 tail (1 per block for IQ2_S/IQ3_S;
 * 8 lane sums + min sum per block for Q4_K/Q5_K). No validation. */
int32_t orc_block_sums(int32_t type, const uint8_t* w, const uint8_t* q8, uint64_t n, int32_t* sums);

/* gemv_into for a quantized matrix in CpuParallelQ8K (simd=1) or LlamaQ8K
 * (simd=0) mode: gemv.rs:56-70 / :43-54 with prepare_llama_q8k :245-272.
 * q8_scratch receives Q8_K(x). threads<=0 uses the hardware count. */
int32_t orc_gemv(const orc_matrix* w, const float* x, float* y, uint8_t* q8_scratch, int32_t simd,
                 int32_t threads);
/* gemv_accumulate_scaled_into, gemv.rs:117-174 */
int32_t orc_gemv_accumulate_scaled(const orc_matrix* w, const float* x, float* y, float scale,
                                   uint8_t* q8_scratch, int32_t simd, int32_t threads);
/* F32 row GEMV, one sequential chain per row: gemv.rs:72-86, dot_f32_row :286-303 */
int32_t orc_gemv_f32(const orc_matrix* w, const float* x, float* y, int32_t threads);
/* route_experts_into, bridge-model-hy3/src/routing.rs:25-107 */
int32_t orc_route_experts(const float* logits, const float* bias, uint64_t expert_count, uint64_t k,
                          float weight_scale, uint32_t* ids, float* coefs);
/* apply_swiglu, activation.rs:170-178 (in place on gate) */
int32_t orc_swiglu(float* gate, const float* up, uint64_t n);
/* moe_routed_by_id_into, moe.rs:64-147 (preflight=1 runs every expert twice,
 * as the reference does; preflight=0 is the single-pass variant). */
int32_t orc_moe_routed(const orc_expert* experts, uint64_t expert_count, const orc_expert* shared,
                       const uint32_t* ids, const float* coefs, uint64_t k, const float* x, float* out,
                       int32_t preflight, int32_t simd, int32_t threads);
/* Route + finish for one token: router F32 GEMV (gemv.rs:72-86), route_experts_into,
 * moe_routed_by_id_into (layer.rs:583-603, :610-659 without norm / residual). */
int32_t orc_moe_token(const orc_expert* experts, uint64_t expert_count, const orc_expert* shared,
                      const orc_matrix* router, const float* bias, uint64_t k, float weight_scale,
                      const float* x, float* out, uint32_t* ids, float* coefs, int32_t preflight,
                      int32_t simd, int32_t threads);

/* Test hooks. */
// weighted_rms_norm_into (bridge-kernels-reference/src/norm.rs:5-18): out is
// written only when every check passes (validation :102-143, rms_scale
// :144-153). weight_len and out_len are the slice lengths the reference checks.
int32_t orc_rms_norm(const float* input, uint64_t n, const float* weight, uint64_t weight_len, float epsilon,
                     float* out, uint64_t out_len);
// residual_add_in_place (norm.rs:83-100): dest += src, or nothing on error.
int32_t orc_residual_add(float* dest, uint64_t n, const float* src, uint64_t src_len);

/* Reduced Hy3 model pieces (hy3_reduced.cpp): the deterministic weights of
 * bridge-test-model/src/hy3.rs and the non-expert steps of its token
 * (bridge-kernels-reference/src/layer.rs:309-472), for the end-to-end pin
 * against bridge-test-model/tests/fixtures/hy3-oracle-v1.json. */
uint16_t orc_f32_to_f16(float v);
int32_t orc_hy3_fill_matrix(int32_t type, uint64_t input_width, uint64_t output_width, uint64_t seed, uint8_t* out,
                            uint64_t out_len);
void orc_hy3_embeddings(float* out, uint64_t n);
void orc_hy3_norm_weights(uint64_t length, uint64_t seed, float* out);
int32_t orc_gemv_dequant(const orc_matrix* w, const float* x, float* y);
int32_t orc_gemv_dequant_accumulate_scaled(const orc_matrix* w, const float* x, float* y, float scale);
int32_t orc_head_rms_norm(float* values, uint64_t n, const float* weight, uint64_t head_dim, float eps);
/* Hy3RopeParams, rope.rs:8-18 */
typedef struct orc_rope {
    uint64_t head_dim, context_length, original_context;
    float base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow;
} orc_rope;
int32_t orc_rope_neox_yarn(float* values, uint64_t head_count, uint64_t position, const orc_rope* p);
int32_t orc_gqa_attention(const float* cache_keys, const float* cache_values, uint64_t stored, uint64_t q_heads,
                          uint64_t kv_heads, uint64_t dim, const float* q, const float* k, const float* v,
                          float* out);
int32_t orc_softmax(const float* logits, uint64_t n, float* out);

float orc_f16_to_f32(uint16_t bits);
int32_t orc_nearest_int(float v);
float orc_expf(float v);
int32_t orc_hw_threads(void);
/* Pointers to the codebooks compiled into the oracle (for the SHA-256 lock test). */
const uint8_t* orc_table_bytes(int32_t which, uint64_t* len);

#ifdef __cplusplus
}
#endif

#endif
