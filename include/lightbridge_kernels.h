/*
 * lightbridge_kernels.h -- C ABI of the B200 (sm_100a) quantized routed-MoE
 * expert kernels.
 *
 * This is the drop-in boundary for LightBridge's quantized expert hot path:
 * packed IQ2_S / IQ3_S / Q4_K / Q5_K weight rows dotted against Q8_K
 * activations inside the Hy3 routed + shared SwiGLU expert FFN with top-k
 * routing. The reference (a Rust workspace) exposes this path as Rust
 * functions over borrowed slices; every entry point below names the reference
 * function it replaces (path:line inside the reference project).
 *
 * Conventions (kept from the reference):
 *  - Caller-owned outputs and scratch. No entry point allocates on the hot
 *    path; scratch sizes are queryable (lbk_required_q8k_bytes,
 *    lbk_moe_workspace_bytes).
 *  - All host-checkable validation (types, widths, lengths, finite scalars,
 *    routed-expert order) happens before anything is launched; on a non-zero
 *    status nothing was written.
 *  - Device pointers only (except where a parameter says "host"). Launches are
 *    stream-ordered and asynchronous. Conditions that need device data
 *    (non-finite activations, non-finite weight scales, non-finite SwiGLU
 *    values) are recorded in a device status word that the caller reads with
 *    lbk_context_sync_status(); kernels that write outputs check it first, so
 *    outputs of a launch whose inputs failed validation are left unchanged.
 *  - Packed weights use the GGUF byte layout unchanged (LBK_LAYOUT_GGUF), or
 *    the row-planar device layout produced by lbk_repack (LBK_LAYOUT_PLANAR),
 *    which has an exact byte-for-byte inverse (lbk_unpack).
 *  - Matrices follow GGML order [input_width, output_width]: output row r is
 *    input_width/256 consecutive packed blocks.
 *  - A context is bound to one device. Distinct contexts may be used from
 *    different host threads; one context is not reentrant.
 */
#ifndef LIGHTBRIDGE_KERNELS_H
#define LIGHTBRIDGE_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LBK_ABI_VERSION 1

/* GGML type discriminants (reference: crates/bridge-core/src/ggml_type.rs:9-30). */
typedef enum lbk_ggml_type {
    LBK_TYPE_F32 = 0,
    LBK_TYPE_Q4_K = 12,
    LBK_TYPE_Q5_K = 13,
    LBK_TYPE_Q8_K = 15,
    LBK_TYPE_IQ3_S = 21,
    LBK_TYPE_IQ2_S = 22
} lbk_ggml_type;

/* Block constants (reference: bridge-quant-layout/src/q8_k.rs:7-12,
 * src/k_quants.rs:7-13). */
#define LBK_QK_K 256
#define LBK_Q8K_BLOCK_BYTES 292
#define LBK_Q4K_BLOCK_BYTES 144
#define LBK_Q5K_BLOCK_BYTES 176
#define LBK_IQ2S_BLOCK_BYTES 82
#define LBK_IQ3S_BLOCK_BYTES 110

/* Status codes. Values 1..29 map one-to-one onto the reference error variants
 * QuantError (bridge-quant-layout/src/error.rs:9-60), KernelError
 * (bridge-kernels-reference/src/error.rs:6-58) and the routing errors of
 * Hy3Error (bridge-model-hy3/src/routing.rs:25-107). */
typedef enum lbk_status {
    LBK_OK = 0,
    LBK_UNSUPPORTED_TYPE = 1,
    LBK_ZERO_LOGICAL_ELEMENTS = 2,
    LBK_LOGICAL_ELEMENTS_NOT_DIVISIBLE = 3,
    LBK_ARITHMETIC_OVERFLOW = 4,
    LBK_ENCODED_LENGTH_MISMATCH = 5,
    LBK_OUTPUT_LENGTH_MISMATCH = 6,
    LBK_NON_FINITE_SCALE = 7,        /* packed binary16 d / dmin */
    LBK_NON_FINITE_ACTIVATION = 8,   /* Q8_K quantizer input */
    LBK_NON_FINITE_Q8_SCALE = 9,     /* encoded Q8_K d */
    LBK_DIMENSION_MISMATCH = 10,
    LBK_SCRATCH_TOO_SMALL = 11,
    LBK_NON_FINITE_VALUE = 12,       /* GEMV input, coefficient, SwiGLU value ... */
    LBK_ROUTED_EXPERT_ORDER = 13,
    LBK_DUPLICATE_ROUTED_EXPERT = 14,
    LBK_INVALID_PARAMETER = 15,
    LBK_ROUTING_TOPK = 16,
    LBK_ROUTING_LENGTH = 17,
    LBK_NON_FINITE_ROUTING_VALUE = 18,
    LBK_CUDA_ERROR = 30,
    LBK_TIMEOUT = 31,
    LBK_NO_DEVICE = 32,
    LBK_FORMAT_ERROR = 33,  /* GGUF container or Hy3 schema; kind in detail.bits (lbk_gguf_error) */
    LBK_IO_ERROR = 34       /* a GGUF file could not be opened or read */
} lbk_status;

/* Packed weight byte layouts. */
typedef enum lbk_layout {
    LBK_LAYOUT_GGUF = 0,   /* GGUF / reference block layout, unchanged */
    LBK_LAYOUT_PLANAR = 1  /* row-planar, 16-byte row stride (see lbk_repack) */
} lbk_layout;

/* Router dot-product order. */
typedef enum lbk_router_mode {
    /* One sequential f32 chain per row, in lane order: bit-identical to the
     * reference F32 GEMV (bridge-kernels-reference/src/gemv.rs:286-303). */
    LBK_ROUTER_SEQUENTIAL = 0,
    /* Fixed-shape tree reduction: deterministic, within 1e-5 relative of the
     * sequential order, and much faster. */
    LBK_ROUTER_TREE = 1
} lbk_router_mode;

/* Detail of the last failure, host- or device-detected. */
typedef struct lbk_error_detail {
    int32_t status;        /* lbk_status */
    int32_t cuda_error;    /* cudaError_t when status == LBK_CUDA_ERROR */
    uint64_t index;        /* block / lane / expert index, where meaningful */
    uint32_t bits;         /* offending value bits, where meaningful */
    uint64_t expected;     /* expected length / width, where meaningful */
    uint64_t actual;       /* actual length / width, where meaningful */
    char message[160];
} lbk_error_detail;

typedef struct lbk_context lbk_context;

/* One packed matrix in device memory. Its byte length must be exactly
 * output_width * (input_width / 256) * block_bytes(type) in the GGUF layout,
 * lbk_planar_bytes in the planar layout. */
typedef struct lbk_matrix {
    int32_t type;            /* lbk_ggml_type */
    int32_t layout;          /* lbk_layout */
    uint64_t input_width;    /* GGML ne[0]: logical elements per row */
    uint64_t output_width;   /* GGML ne[1]: rows */
    const void* data;        /* device pointer */
    uint64_t bytes;          /* encoded byte length */
} lbk_matrix;

/* A SwiGLU expert (reference: SwiGluExpert, activation.rs:5-47). */
typedef struct lbk_expert {
    lbk_matrix gate;
    lbk_matrix up;
    lbk_matrix down;
} lbk_expert;

/* A routed selection (reference: RoutedExpert, bridge-model-hy3/src/routing.rs). */
typedef struct lbk_routed {
    uint32_t expert_id;
    float coefficient;
} lbk_routed;

/* ---------------------------------------------------------------- context */

int32_t lbk_abi_version(void);

/* Name of the backend, "cuda_sm100a_q8_k"; the CPU backend of the reference is
 * named by CpuCapabilities::backend_name (bridge-kernels-cpu/src/lib.rs:50-56). */
const char* lbk_backend_name(void);

/* Creates a context on `device` (also loads the IQ codebooks into device
 * memory and allocates the device status word). Not on the hot path. */
int32_t lbk_context_create(int32_t device, lbk_context** out);
int32_t lbk_context_destroy(lbk_context* ctx);

/* Synchronizes `stream` (a cudaStream_t, NULL = legacy default), reads and
 * clears the device status word. Returns its status; fills `detail` if given. */
int32_t lbk_context_sync_status(lbk_context* ctx, void* stream, lbk_error_detail* detail);

/* Detail of the last host-side failure of any call on this thread. */
void lbk_last_error_detail(lbk_error_detail* out);

/* ------------------------------------------------------------- sizes */

/* reference: required_q8_k_bytes, bridge-kernels-reference/src/gemv.rs:18-31 */
int32_t lbk_required_q8k_bytes(uint64_t input_width, uint64_t* bytes);

/* Encoded byte length of a [input_width, output_width] matrix of `type`
 * (reference: EncodedTensorView::new, matrix.rs:26-78). */
int32_t lbk_matrix_bytes(int32_t type, uint64_t input_width, uint64_t output_width, uint64_t* bytes);

/* Byte length of the same matrix in the planar device layout (rows padded
 * to 16 bytes, see lbk_repack); no counterpart in the reference. */
int32_t lbk_planar_bytes(int32_t type, uint64_t input_width, uint64_t output_width, uint64_t* bytes);

/* ------------------------------------------------------------- kernels */

/* Q8_K activation quantization of x[n] into q8[n/256*292].
 * reference: quantize_row_q8_k_into, bridge-quant-layout/src/q8_k.rs:16-76.
 * Non-finite input is reported through the device status word
 * (LBK_NON_FINITE_ACTIVATION, first lane index) and q8 is left unchanged. */
int32_t lbk_quantize_q8k(lbk_context* ctx, const float* x, uint64_t n, uint8_t* q8,
                         uint64_t q8_bytes, void* stream);

/* Dot products of `rows` packed rows (each input_width wide) with one Q8_K
 * activation row, writing f32 results -- the per-row result of
 * vec_dot_q8_k / vec_dot_q8_k_cpu (q8_k.rs:80-119), bit-identical.
 * If block_sums is non-NULL it receives the per-super-block int32 sums that
 * feed the f32 tail: 1 per block for IQ2_S / IQ3_S, 9 per block (8 lane sums,
 * then the min sum) for Q4_K / Q5_K. */
int32_t lbk_vec_dot_q8k(lbk_context* ctx, const lbk_matrix* w, const uint8_t* q8, uint64_t q8_bytes,
                        float* out, int32_t* block_sums, void* stream);

/* y = W x with x quantized to Q8_K into caller scratch.
 * reference: gemv_into (CpuParallelQ8K), bridge-kernels-reference/src/gemv.rs:88-115,
 * and gemv_cpu_parallel_q8k_into (:56-70). */
int32_t lbk_gemv(lbk_context* ctx, const lbk_matrix* w, const float* x, float* y,
                 uint8_t* q8_scratch, uint64_t q8_scratch_bytes, void* stream);

/* y[r] += scale * dot(W_r, Q8_K(x)), non-contracted multiply then add.
 * reference: gemv_accumulate_scaled_into, gemv.rs:117-174. `scale` is
 * checked on the host; non-finite y is reported via the status word. */
int32_t lbk_gemv_accumulate_scaled(lbk_context* ctx, const lbk_matrix* w, const float* x, float* y,
                                   float scale, uint8_t* q8_scratch, uint64_t q8_scratch_bytes,
                                   void* stream);

/* Router logits for `tokens` tokens: logits[t*E + e] = dot(router_e, x_t),
 * router an F32 [hidden, E] matrix.
 * reference: gemv_into on an F32 matrix, gemv.rs:72-86 and :286-303. */
int32_t lbk_router_logits(lbk_context* ctx, const lbk_matrix* router, const float* x, uint64_t tokens,
                          float* logits, int32_t mode, void* stream);

/* Hy3 top-k routing of `tokens` rows of E logits: sigmoid, + selection bias for
 * the ranking only, ties to ascending ID, renormalise over the top k with the
 * 2^-14 floor, scale by weight_scale, output sorted by expert ID.
 * reference: route_experts_into, bridge-model-hy3/src/routing.rs:25-107. */
int32_t lbk_route_topk(lbk_context* ctx, const float* logits, const float* selection_bias,
                       uint64_t expert_count, uint64_t tokens, uint32_t k, float weight_scale,
                       lbk_routed* routed, void* stream);

/* f32 decode of rows [first_row, first_row + rows) of a packed matrix in the
 * GGUF layout into out[rows * input_width], bit-identical to the reference:
 * decode_row_into (bridge-quant-layout/src/k_quants.rs:71-105) per row over
 * the block decoders (k_quants.rs:242-300, iq2_s.rs:9-39, iq3_s.rs:9-53;
 * F32 rows are copied bit for bit). Every d / dmin of the range is checked
 * first: a non-finite one is reported through the status word
 * (LBK_NON_FINITE_SCALE, index = block within the range) and nothing is
 * written. A planar matrix is refused (lbk_unpack converts it). */
int32_t lbk_decode_rows(lbk_context* ctx, const lbk_matrix* w, uint64_t first_row, uint64_t rows, float* out,
                        void* stream);

/* SwiGLU expert, accumulated: dst += coefficient * down(swiglu(gate x, up x)).
 * reference: expert_swiglu_accumulate_into, activation.rs:104-144.
 * Workspace: lbk_expert_workspace_bytes. */
int32_t lbk_expert_workspace_bytes(const lbk_expert* expert, uint64_t* bytes);
int32_t lbk_expert_swiglu_accumulate(lbk_context* ctx, const lbk_expert* expert, const float* x,
                                     float* dst, float coefficient, void* workspace,
                                     uint64_t workspace_bytes, void* stream);

/* --------------------------------------------------------- MoE layer */

/* One layer's expert table, mirroring Hy3MoeWeights
 * (bridge-kernels-reference/src/layer.rs:28-36). Routed expert e's gate, up
 * and down matrices are experts[e]; the matrices stay resident in device
 * memory for the life of the layer handle. */
typedef struct lbk_moe_weights {
    const lbk_expert* experts;   /* host array of expert_count descriptors */
    uint64_t expert_count;
    lbk_expert shared;           /* always-on shared expert, coefficient 1.0 */
    lbk_matrix router;           /* F32 [hidden, expert_count] */
    const float* selection_bias; /* device, expert_count floats */
    uint32_t top_k;              /* expert_used_count */
    float weight_scale;          /* Hy3 expert_weights_scale (2.826 default) */
} lbk_moe_weights;

typedef struct lbk_moe_layer lbk_moe_layer;

/* Registers a layer's resident expert table: checks every shape and type
 * (SwiGluExpert::new, activation.rs:13-22; widths of moe.rs:272-314), scans
 * every binary16 scale once (validate_scales, k_quants.rs:178-208) -- the
 * reference re-validates every row on every call (gemv.rs:268-270); here that
 * happens once at registration -- uploads the expert pointer table, and picks
 * the fused sm_100a kernels when every matrix is in the planar layout with a
 * supported type combination (else the per-expert kernels). Synchronizes
 * `stream`. Not on the hot path. */
int32_t lbk_moe_layer_create(lbk_context* ctx, const lbk_moe_weights* w, void* stream, lbk_moe_layer** out);
int32_t lbk_moe_layer_destroy(lbk_moe_layer* layer);
/* 1 when the fused kernels are used, 0 for the per-expert path. */
int32_t lbk_moe_layer_fused(const lbk_moe_layer* layer);

/* Token count from which lbk_moe_forward / lbk_moe_routed (and, counted in
 * items, lbk_ep_items_forward; in tokens, lbk_ep_combine) run the grouped
 * kernels on a fused planar layer: the call's (token, slot) pairs are grouped
 * by expert and each weight half block is decoded once for every pair of its
 * group. Results are bit-identical either way; only the speed differs.
 * min_tokens 0 turns grouping off; the default is 8 for whole layers and 0
 * (off) for expert-parallel layers (lbk_ep_layer_create, or lbk_moe_layer_load
 * of a rank's share), whose passes measured no faster grouped. No counterpart
 * in the reference, which runs each routed expert per token
 * (moe_routed_by_id_into, moe.rs:64-147). */
int32_t lbk_moe_layer_set_grouping(lbk_moe_layer* layer, uint64_t min_tokens);

/* Expert-parallel items (lbk_ep_items_forward_counted) on the grouped kernels
 * run their gate/up projections on the tcgen05 tensor cores (IQ2_S gate/up:
 * int8 MMA, one accumulator per 16-weight scale group, see
 * lbk_tc_grouped_dots) when the expected pairs per expert -- cap_items / the
 * global expert count -- reach `min_pairs_per_expert` (default 4; 0: never).
 * SwiGLU and Q8_K(h) follow per pair, and an IQ3_S or IQ2_S down projection
 * runs on the tensor cores too (else on the grouped kernel); results are
 * bit-identical either way. No counterpart in the reference,
 * which runs each routed expert once per token (moe.rs:64-147). */
int32_t lbk_moe_layer_set_tensor_cores(lbk_moe_layer* layer, uint64_t min_pairs_per_expert);

/* Bound of a single-token call's wait for its routing: the down kernel polls
 * the flag with which the gate/up kernel publishes the routing (so that it can
 * request its first rows before the gate/up grid ends) at most `polls` times
 * (default 2^20, far beyond the few microseconds the publication takes). A
 * wait that runs out is reported as LBK_TIMEOUT through the status word and
 * the call's output is left unwritten; the kernels still finish (the wait has
 * no copy in flight), so the workspace and the context stay usable. No
 * counterpart in the reference, whose calls are synchronous. */
int32_t lbk_moe_layer_set_wait_limit(lbk_moe_layer* layer, uint32_t polls);

/* Workspace bytes for `tokens` tokens. The workspace must be zero-filled once
 * before its first use (its first 16 bytes hold an arrival counter that every
 * completed call leaves at zero; the rest is rewritten by every call), so one
 * workspace of the largest size serves calls of any layer and token count. */
int32_t lbk_moe_workspace_bytes(const lbk_moe_layer* layer, uint64_t tokens, uint64_t* bytes);

/* Full routed-MoE FFN for `tokens` tokens (x: tokens*hidden f32): router
 * logits, top-k routing, then per token
 *   out = 0; out += coef_e * expert_e(x) for routed e in ascending ID;
 *   out += 1.0 * shared(x)
 * -- the combine order of moe_routed_by_id_into
 * (bridge-kernels-reference/src/moe.rs:64-147); together this is
 * hy3_moe_route_token + hy3_moe_finish_token (layer.rs:473-659) without the
 * FFN norm and the residual add. `routed_out` (device, tokens*top_k entries,
 * may be NULL) receives the routing. */
int32_t lbk_moe_forward(lbk_moe_layer* layer, const float* x, uint64_t tokens, float* out,
                        lbk_routed* routed_out, int32_t router_mode, void* workspace,
                        uint64_t workspace_bytes, void* stream);

/* Kernel-level tracing: while enabled, lbk_moe_forward records CUDA events
 * around its router, gate/up and down launches (three event records per call;
 * they are captured into CUDA graphs like the launches).
 * lbk_moe_layer_trace_read returns the three durations of the most recent
 * traced call (ms), after synchronizing on its last event. */
int32_t lbk_moe_layer_trace(lbk_moe_layer* layer, int32_t enable);
int32_t lbk_moe_layer_trace_read(lbk_moe_layer* layer, float ms[3]);

/* Same combine for a caller-supplied routing (device `routed`, tokens*top_k
 * entries, IDs strictly ascending per token, finite coefficients; checked on
 * the device, reported through the status word). reference:
 * moe_routed_by_id_into, moe.rs:64-147. */
int32_t lbk_moe_routed(lbk_moe_layer* layer, const float* x, uint64_t tokens, const lbk_routed* routed,
                       float* out, void* workspace, uint64_t workspace_bytes, void* stream);

/* ---------------------------------------- MoE block: norm and residual */

/* weighted_rms_norm_into (bridge-kernels-reference/src/norm.rs:5-18) on each
 * of `rows` rows of n values: out = (x * scale) * weight with scale =
 * 1 / sqrt(mean(x^2) + epsilon). mode LBK_ROUTER_SEQUENTIAL sums the squares
 * in one f32 chain as the reference does (bit-identical); LBK_ROUTER_TREE in
 * a fixed tree (within 1e-5). Validate before write: a non-finite input,
 * weight, scale or output is reported through the status word and the row's
 * output is not written; n == 0 or epsilon <= 0 -> LBK_INVALID_PARAMETER,
 * non-finite epsilon -> LBK_NON_FINITE_VALUE (host checks). */
int32_t lbk_rms_norm(lbk_context* ctx, const float* x, const float* weight, uint64_t n, uint64_t rows, float epsilon,
                     float* out, int32_t mode, void* stream);
/* residual_add_in_place (norm.rs:83-100): dest += src over n values, written
 * only when every check of the call (dest finite, src finite, sums finite, in
 * that order) passes and the status word is clear. */
int32_t lbk_residual_add(lbk_context* ctx, float* dest, const float* src, uint64_t n, void* stream);

/* The FFN half of a Hy3 block for `tokens` tokens: hidden[t] +=
 * MoE(RMSNorm(hidden[t], ffn_norm, epsilon)), i.e. the FFN part of
 * hy3_moe_route_token (RMSNorm, router, top-k; layer.rs:588-608) followed by
 * hy3_moe_finish_token (experts, combine, residual add; layer.rs:610-659)
 * with the experts HBM-resident, so no payload is streamed between the two.
 * router_mode selects the order of both the norm's sum and the router logits.
 * hidden is written only if every step succeeded. */
int32_t lbk_moe_block_workspace_bytes(const lbk_moe_layer* layer, uint64_t tokens, uint64_t* bytes);
int32_t lbk_moe_block_forward(lbk_moe_layer* layer, float* hidden, const float* ffn_norm, float epsilon,
                              uint64_t tokens, lbk_routed* routed_out, int32_t router_mode, void* workspace,
                              uint64_t workspace_bytes, void* stream);

/* The same block in the reference's two phases, for a runtime that acts on
 * the routing between them. Route: the FFN part of hy3_moe_route_token
 * (layer.rs:473-605 from the FFN RMSNorm on: norm, router, top-k); the
 * routing (tokens*top_k entries) stays in the block workspace and is copied to
 * routed_out when that is not null. Finish: hy3_moe_finish_token
 * (layer.rs:610-659): `selected` (device, tokens*top_k entries) must equal the
 * route phase's routing in expert IDs and coefficient bits, checked on the
 * device before anything is written (a mismatch is reported through the
 * status word as LBK_INVALID_PARAMETER at the first differing entry and
 * leaves hidden untouched); then the experts, the combine and hidden +=
 * delta. The phase is kept per workspace as the reference keeps it per
 * scratch: a second route on a workspace before its finish, or a finish
 * without a route, returns LBK_INVALID_PARAMETER; a finish with another token
 * count returns LBK_DIMENSION_MISMATCH (host checks, before any launch). The
 * phase ends when finish has been enqueued; device-side failures of finish
 * surface at the next status sync, as for every call. Workspace: as
 * lbk_moe_block_workspace_bytes. */
int32_t lbk_moe_block_route(lbk_moe_layer* layer, const float* hidden, const float* ffn_norm, float epsilon,
                            uint64_t tokens, lbk_routed* routed_out, int32_t router_mode, void* workspace,
                            uint64_t workspace_bytes, void* stream);
int32_t lbk_moe_block_finish(lbk_moe_layer* layer, float* hidden, uint64_t tokens, const lbk_routed* selected,
                             void* workspace, uint64_t workspace_bytes, void* stream);

/* ------------------------------------------------ expert parallelism */

/* A rank's layer for expert parallelism: w->experts holds this rank's
 * resident experts, the global experts [first_expert, first_expert +
 * w->expert_count) of a router (w->router) over global_experts; the router
 * and the shared expert are whole. Such a layer runs only through lbk_ep_*.
 * No counterpart in the reference, whose MoE step runs every expert on one
 * host (bridge-runtime/src/hy3_scalar.rs:561-628). Needs planar layers with
 * hidden 2048 or 4096. */
int32_t lbk_ep_layer_create(lbk_context* ctx, const lbk_moe_weights* w, uint64_t global_experts,
                            uint64_t first_expert, void* stream, lbk_moe_layer** out);
/* Bytes of one token's Q8_K image as lbk_ep_route writes it and
 * lbk_ep_items_forward / lbk_ep_combine read it (opaque, 16-byte aligned). */
int32_t lbk_ep_q8_bytes(const lbk_moe_layer* layer, uint64_t* bytes);
/* Workspace for lbk_ep_* calls over `count` tokens or items (zero-filled once). */
int32_t lbk_ep_workspace_bytes(const lbk_moe_layer* layer, uint64_t count, uint64_t* bytes);
/* Home rank: routing of `tokens` tokens (routed[tokens*k], global expert IDs
 * in ascending order, as lbk_moe_forward) and their Q8_K images
 * (q8[tokens * lbk_ep_q8_bytes]). reference: hy3_moe_route_token's router and
 * route_experts_into (layer.rs:576-603, routing.rs:25-107). */
int32_t lbk_ep_route(lbk_moe_layer* layer, const float* x, uint64_t tokens, lbk_routed* routed, uint8_t* q8,
                     void* workspace, uint64_t workspace_bytes, void* stream);
/* Expert rank: for each item i, the row dots of resident expert
 * items_routed[i].expert_id (local index; the coefficient is ignored) on the
 * token image q8_items[i]: dots[i*H + r] = down_r(SwiGLU(gate, up)) before any
 * coefficient. reference: expert_swiglu_accumulate_into's projection
 * (activation.rs:104-144). */
int32_t lbk_ep_items_forward(lbk_moe_layer* layer, const uint8_t* q8_items, const lbk_routed* items_routed,
                             uint64_t items, float* dots, void* workspace, uint64_t workspace_bytes, void* stream);
/* Home rank: out[t] = 0; += c_j * routed_dots[t][j] in the routing's order
 * (ascending ID); += 1.0 * shared(t) -- moe_routed_by_id_into's accept pass
 * (moe.rs:116-147), bit-identical to lbk_moe_forward on one GPU.
 * routed_dots: [tokens][k][H] as returned by the expert ranks. */
int32_t lbk_ep_combine(lbk_moe_layer* layer, const uint8_t* q8, uint64_t tokens, const lbk_routed* routed,
                       const float* routed_dots, float* out, void* workspace, uint64_t workspace_bytes, void* stream);

/* Expert-parallel exchange over peer memory: no collective, no size exchange
 * and no device-to-host read in a layer step, so a step can be captured in a
 * CUDA graph (none of this has a counterpart in the reference, whose MoE step
 * runs every expert on one host).
 *
 * Peer buffers: lbk_peer_alloc allocates and zero-fills `bytes` of device
 * memory and returns its 64-byte interprocess handle; another process of the
 * node maps it with lbk_peer_open (plain peer loads and stores over NVLink;
 * no multicast object) and unmaps it with lbk_peer_close; the owner frees it
 * with lbk_peer_free.
 *
 * Exchange buffer of a rank (lbk_ep_exchange_layout, `cap` tokens per rank at
 * most; zero-filled before the first step): the routing, a 512-byte control
 * block (token count and step flags), the Q8_K images and the routed row dots
 * returned by the other ranks. `peers` is a device array of `world` (at most
 * 64) buffer pointers as this GPU addresses them, indexed by rank. A layer
 * step, every call on every rank once, in this order, on one stream:
 *   lbk_ep_publish   route this rank's tokens into its own buffer and
 *                    publish them (this rank's step number + 1);
 *   lbk_ep_gather    wait until every rank has published this step, then
 *                    collect the pairs routed to this rank's experts: items
 *                    (local expert ID), their Q8_K images, their return
 *                    addresses {rank, t * k + j} (uint64 each) and their
 *                    count, on the device (`count` is zero-filled before the
 *                    first step; lbk_ep_scatter resets it for the next);
 *   lbk_ep_items_forward_counted  the items' row dots (as
 *                    lbk_ep_items_forward, the count read on the device;
 *                    cap_items = world * cap * k bounds it);
 *   lbk_ep_scatter   each item's dots into its home rank's buffer, then flag
 *                    this rank's step done in every buffer (or, instead of
 *                    these two, lbk_ep_items_return: the items' down rows
 *                    stored in place);
 *   lbk_ep_combine_exchange  on the home rank: wait until every rank's dots
 *                    of this step are in, then combine from its buffer's
 *                    routing, images and dots, bit-identical to
 *                    lbk_moe_forward on one GPU (a rank without tokens still
 *                    calls it: the wait frees its buffer for the next step).
 *                    `shared_dots` null: the shared expert is computed here
 *                    first; otherwise they are lbk_ep_shared's output, which
 *                    needs only the publication and so can run on a second
 *                    stream (with its own workspace) while the pairs are
 *                    exchanged.
 * The waits poll at most the layer's wait limit
 * (lbk_moe_layer_set_wait_limit) times; one that runs out is reported as
 * LBK_TIMEOUT through the status word (index 8: gather, 9: combine; bits: the
 * step) and the kernels still finish. */
typedef struct lbk_ep_exchange {
    uint64_t routing, control, q8, dots, total; /* byte offsets in a buffer, its size */
    uint64_t q8_bytes;                          /* one token's Q8_K image */
} lbk_ep_exchange;
int32_t lbk_peer_alloc(lbk_context* ctx, uint64_t bytes, void** ptr, uint8_t handle[64]);
int32_t lbk_peer_free(lbk_context* ctx, void* ptr);
int32_t lbk_peer_open(lbk_context* ctx, const uint8_t handle[64], void** ptr);
int32_t lbk_peer_close(lbk_context* ctx, void* ptr);
int32_t lbk_ep_exchange_layout(const lbk_moe_layer* layer, uint64_t cap, lbk_ep_exchange* out);
int32_t lbk_ep_publish(lbk_moe_layer* layer, const float* x, uint64_t tokens, void* xbuf, uint64_t cap, void* workspace,
                       uint64_t workspace_bytes, void* stream);
int32_t lbk_ep_gather(lbk_moe_layer* layer, const void* const* peers, uint32_t world, uint32_t rank, uint64_t cap,
                      uint8_t* q8_items, lbk_routed* items, uint64_t* returns, uint32_t* count, uint64_t cap_items,
                      void* stream);
int32_t lbk_ep_items_forward_counted(lbk_moe_layer* layer, const uint8_t* q8_items, const lbk_routed* items,
                                     const uint32_t* count, uint64_t cap_items, float* dots, void* workspace,
                                     uint64_t workspace_bytes, void* stream);
int32_t lbk_ep_scatter(lbk_moe_layer* layer, void* const* peers, uint32_t world, uint32_t rank, uint64_t cap,
                       const float* dots, const uint64_t* returns, uint32_t* count, uint64_t cap_items, void* stream);
int32_t lbk_ep_shared(lbk_moe_layer* layer, void* xbuf, uint64_t cap, uint64_t tokens, float* shared_dots,
                      void* workspace, uint64_t workspace_bytes, void* stream);
/* lbk_ep_items_forward_counted and lbk_ep_scatter in one call, with no local
 * copy of the dots: the down kernels store each item's row dots straight into
 * its home rank's buffer at its return address (peer stores, then a system
 * fence), and a one-CTA kernel then resets `count` and flags this rank's step
 * done in every buffer. Same results bit for bit; one kernel and one round
 * trip of the dots fewer. */
int32_t lbk_ep_items_return(lbk_moe_layer* layer, void* const* peers, uint32_t world, uint32_t rank, uint64_t cap,
                            const uint8_t* q8_items, const lbk_routed* items, const uint64_t* returns, uint32_t* count,
                            uint64_t cap_items, void* workspace, uint64_t workspace_bytes, void* stream);
int32_t lbk_ep_combine_exchange(lbk_moe_layer* layer, void* xbuf, uint32_t world, uint64_t cap, uint64_t tokens,
                                const float* shared_dots, float* out, void* workspace, uint64_t workspace_bytes,
                                void* stream);

/* lbk_moe_forward without a caller workspace and without any allocation: the
 * workspace is a fixed 1 MiB array of this library's device memory, one per
 * device. No counterpart in the reference (its moe_routed_by_id_into takes
 * caller scratch, moe.rs:64-71). For callers that cannot allocate device
 * memory: an FFI host holding only device pointers handed to it, with no
 * device allocator of its own, and decode loops in which cudaMalloc / cudaFree
 * would synchronize the device.
 *   - Returns LBK_SCRATCH_TOO_SMALL (detail: expected = bytes needed) when the
 *     layer's workspace for `tokens` exceeds 1 MiB (hidden 4096, ffn 1536,
 *     top-8 fits up to 4 tokens).
 *   - The first call on a device looks up the array and zero-fills it
 *     synchronously; make it before any stream capture on that device. The
 *     array's first 16 bytes (an arrival counter) must be zero when a call
 *     starts; every call that runs to completion leaves them at zero.
 *   - Calls that overlap in time on one device (any stream, thread or layer)
 *     share the array and race: serialize them. */
int32_t lbk_moe_forward_no_alloc(lbk_moe_layer* layer, const float* x, uint64_t tokens, float* out,
                                 lbk_routed* routed_out, int32_t router_mode, void* stream);

/* ------------------------------------------------------- layout tools */

/* Converts a GGUF-layout matrix into the planar device layout
 * (lbk_planar_bytes long). Planar layout: rows at a stride of
 * ceil16(nb * block_bytes) bytes (nb = input_width/256; the pad bytes are
 * zero), each row a sequence of field planes over its nb blocks:
 *   IQ2_S: qs[nb][32] | signs[nb][32] | qh[nb][8] | scales[nb][8] | d[nb][2]
 *   IQ3_S: qs[nb][64] | signs[nb][32] | qh[nb][8] | scales[nb][4] | d[nb][2]
 *   Q4_K : qs[nb][128] | scales[nb][12] | d,dmin[nb][4]
 *   Q5_K : qs[nb][128] | qh[nb][32] | scales[nb][12] | d,dmin[nb][4]
 * Inside a block, Q4_K / Q5_K qs (and Q5_K qh) bytes are lane-major per
 * 32-byte group (new[4k+i] = old[k+8i]), and each little-endian 32-bit word
 * of the IQ2_S / IQ3_S qh field is stored as the transpose of its 4x4 matrix
 * of 2-bit cells (cell (r, c) at bit 8r+2c moves to bit 8c+2r). Every row
 * starts 16-byte aligned, so any run of rows is one contiguous aligned copy. */
int32_t lbk_repack(lbk_context* ctx, const lbk_matrix* src_gguf, void* dst_planar, uint64_t dst_bytes,
                   void* stream);
/* Exact inverse of lbk_repack (dst_bytes = lbk_matrix_bytes). */
int32_t lbk_unpack(lbk_context* ctx, const lbk_matrix* src_planar, void* dst_gguf, uint64_t dst_bytes,
                   void* stream);

/* Scans every binary16 d (and dmin) of a matrix; non-finite scales are
 * reported through the status word as LBK_NON_FINITE_SCALE with the global
 * block index. reference: validate_scales, k_quants.rs:178-208. */
int32_t lbk_validate_matrix(lbk_context* ctx, const lbk_matrix* w, void* stream);

/* ------------------------------------------------------ GGUF residency */

/* A GGUF split set opened for reading (bridge-gguf-split GgufSet,
 * src/lib.rs:155-159): every shard's header parsed and checked, the tensors
 * of all shards in one directory. Payloads are read only by
 * lbk_moe_layer_load. */
typedef struct lbk_gguf lbk_gguf;

/* Failure kinds of LBK_FORMAT_ERROR / LBK_IO_ERROR, in lbk_error_detail.bits.
 * They follow GgufError (bridge-gguf/src/error.rs:8-110), CoreError
 * (bridge-core/src/error.rs:6-22), SplitError (bridge-gguf-split/src/lib.rs:
 * 95-153), MetadataError and the Hy3 schema / config errors; the detail's
 * message is the reference's text for the same failure. */
typedef enum lbk_gguf_error {
    LBK_GGUF_IO = 1,
    LBK_GGUF_TRUNCATED = 2,
    LBK_GGUF_BAD_MAGIC = 3,
    LBK_GGUF_UNSUPPORTED_VERSION = 4,
    LBK_GGUF_LIMIT_EXCEEDED = 5,
    LBK_GGUF_INVALID_UTF8 = 6,
    LBK_GGUF_INVALID_BOOLEAN = 7,
    LBK_GGUF_UNKNOWN_VALUE_TYPE = 8,
    LBK_GGUF_NESTED_ARRAY = 9,
    LBK_GGUF_INVALID_DIMENSION_COUNT = 10,
    LBK_GGUF_INVALID_DIMENSION_LIMIT = 11,
    LBK_GGUF_DUPLICATE_METADATA_KEY = 12,
    LBK_GGUF_INVALID_ALIGNMENT = 13,
    LBK_GGUF_ALIGNMENT_WRONG_TYPE = 14,
    LBK_GGUF_ARITHMETIC_OVERFLOW = 15,
    LBK_GGUF_DATA_OFFSET_BEYOND_FILE = 16,
    LBK_GGUF_TENSOR_OFFSET_MISMATCH = 17,
    LBK_GGUF_TENSOR_PADDING_OVERFLOW = 18,
    LBK_GGUF_TENSOR_EXTENT_OVERFLOW = 19,
    LBK_GGUF_TENSOR_DATA_END_OVERFLOW = 20,
    LBK_GGUF_TENSOR_DATA_SECTION_TRUNCATED = 21,
    LBK_GGUF_UNKNOWN_GGML_TYPE = 22,
    LBK_GGUF_ZERO_TENSOR_DIMENSION = 23,
    LBK_GGUF_NOT_BLOCK_ALIGNED = 24,
    LBK_GGUF_TENSOR_OUT_OF_BOUNDS = 25,
    /* split sets */
    LBK_GGUF_NOT_A_FILE = 30,
    LBK_GGUF_INVALID_NUMBERED_FILENAME = 31,
    LBK_GGUF_MISSING_SPLIT_METADATA = 32,
    LBK_GGUF_SPLIT_METADATA_DISAGREEMENT = 33,
    LBK_GGUF_NUMBERED_SINGLE_SHARD = 34,
    LBK_GGUF_MISSING_SHARD = 35,
    LBK_GGUF_SHARD_ESCAPES_PARENT = 36,
    LBK_GGUF_DUPLICATE_TENSOR_NAME = 37,
    LBK_GGUF_HETEROGENEOUS_VERSION = 38,
    LBK_GGUF_HETEROGENEOUS_ENDIANNESS = 39,
    LBK_GGUF_HETEROGENEOUS_ALIGNMENT = 40,
    LBK_GGUF_UNALIGNED_TENSOR_OFFSET = 41,
    LBK_GGUF_NEGATIVE_AGGREGATE_TENSOR_COUNT = 42,
    LBK_GGUF_AGGREGATE_TENSOR_COUNT_DISAGREEMENT = 43,
    LBK_GGUF_AGGREGATE_TENSOR_DIRECTORY_DISAGREEMENT = 44,
    /* metadata and the Hy3 MoE block schema */
    LBK_GGUF_METADATA_MISSING = 50,
    LBK_GGUF_METADATA_WRONG_TYPE = 51,
    LBK_GGUF_METADATA_VALUE = 52,
    LBK_GGUF_NON_FINITE_METADATA = 53,
    LBK_GGUF_MISSING_TENSOR = 54,
    LBK_GGUF_TENSOR_SHAPE = 55,
    LBK_GGUF_TENSOR_TYPE = 56,
    LBK_GGUF_EXPERT_PAYLOAD_NOT_DIVISIBLE = 57,
    LBK_GGUF_BLOCK_OUT_OF_RANGE = 58,
    LBK_GGUF_EXPERT_RANGE = 59,
    LBK_GGUF_SHARED_WIDTH = 60,
    LBK_GGUF_BIG_ENDIAN_PAYLOAD = 61
} lbk_gguf_error;

/* Reader limits (ReaderLimits, bridge-gguf/src/reader.rs:21-42). */
typedef struct lbk_gguf_limits {
    uint32_t max_dimensions;       /* <= 4 */
    uint64_t max_string_bytes;     /* per string */
    uint64_t max_array_elements;   /* aggregate over the file */
    uint64_t max_tensors;
    uint64_t max_metadata_entries;
    uint64_t max_metadata_bytes;   /* metadata section and tensor names */
} lbk_gguf_limits;

/* The primary shard's header facts, and the set's totals. */
typedef struct lbk_gguf_file_info {
    uint32_t version;       /* 2 or 3 */
    uint32_t big_endian;    /* "FUGG" magic */
    uint64_t alignment;     /* general.alignment, default 32 */
    uint64_t shard_count;
    uint64_t tensor_count;  /* all shards */
    uint64_t metadata_count;
    uint64_t data_offset;
    uint64_t file_len;
} lbk_gguf_file_info;

/* One tensor of the directory (TensorLocation, bridge-gguf-split). */
typedef struct lbk_gguf_tensor {
    int32_t type;             /* ggml type discriminant */
    uint32_t n_dims;
    uint64_t dims[4];         /* ne[0..3], 1 past n_dims */
    uint32_t shard;           /* 0-based shard ordinal */
    uint64_t offset;          /* absolute byte offset in its shard */
    uint64_t relative_offset; /* offset within the shard's data section */
    uint64_t bytes;           /* encoded payload bytes */
    uint64_t name_len;
} lbk_gguf_tensor;

/* One metadata value of the primary shard. */
typedef struct lbk_gguf_value {
    uint32_t type;          /* 0 U8 1 I8 2 U16 3 I16 4 U32 5 I32 6 F32 7 Bool 8 String 9 Array 10 U64 11 I64 12 F64 */
    uint32_t element_type;  /* arrays */
    uint64_t count;         /* arrays: elements; strings: bytes */
    uint64_t u;             /* integers (signed ones sign-extended), bools; raw bits of floats */
    double f;               /* F32 / F64 values */
} lbk_gguf_value;

void lbk_gguf_default_limits(lbk_gguf_limits* out);
/* Opens the split set `entry` belongs to (open_set): a `<prefix>-NNNNN-of-
 * MMMMM.gguf` name opens all MMMMM shards beside it (each with split.no and
 * split.count), any other name one file. limits NULL = the defaults. */
int32_t lbk_gguf_open(const char* entry, const lbk_gguf_limits* limits, lbk_gguf** out);
int32_t lbk_gguf_close(lbk_gguf* gguf);
int32_t lbk_gguf_info(const lbk_gguf* gguf, lbk_gguf_file_info* out);
/* Tensor `index` in directory order; its name NUL-terminated into name
 * (name_cap bytes, truncated) when name is not NULL. */
int32_t lbk_gguf_tensor_at(const lbk_gguf* gguf, uint64_t index, lbk_gguf_tensor* out, char* name,
                           uint64_t name_cap);
int32_t lbk_gguf_find_tensor(const lbk_gguf* gguf, const char* name, uint64_t* index);
int32_t lbk_gguf_metadata(const lbk_gguf* gguf, const char* key, lbk_gguf_value* out);
int32_t lbk_gguf_metadata_string(const lbk_gguf* gguf, const char* key, char* buf, uint64_t cap, uint64_t* len);

/* Builds an HBM-resident MoE layer from block `block` of a Hy3 GGUF set:
 * checks general.architecture and the hy_v3.* configuration (resolve_config,
 * bridge-model-hy3/src/config.rs:57-109) and the block's eight MoE tensors
 * (schema.rs:200-258: router [H, E] and exp_probs_b [E] F32, stacked experts
 * [H, F, E] / [F, H, E], shared expert), reads the router, the bias, the
 * shared expert and routed experts [first_expert, first_expert +
 * expert_count) -- each expert one slab of its stacked tensor
 * (checked_expert_slab, schema.rs:524-580) -- repacks them to the planar
 * layout and registers the layer as lbk_moe_layer_create (all experts) or
 * lbk_ep_layer_create (a share) would. expert_count 0 = to the last expert.
 * The layer owns its device memory. Weight types: IQ2_S, IQ3_S, Q4_K, Q5_K.
 * Synchronizes `stream`; not on the hot path. */
int32_t lbk_moe_layer_load(lbk_context* ctx, const lbk_gguf* gguf, uint32_t block, uint64_t first_expert,
                           uint64_t expert_count, void* stream, lbk_moe_layer** out);

/* Grouped row dots of IQ2_S or IQ3_S matrices on the tcgen05 tensor cores
 * (int8 MMA, one int32 accumulator per scale group: 16 weights for IQ2_S,
 * 32 for IQ3_S): the row dots of a group of tokens against one matrix,
 * bit-identical to lbk_gemv per token (dot_iq2_s / dot_iq3_s,
 * bridge-quant-layout/src/q8_k.rs:339-434, chained as gemv_into,
 * gemv.rs:88-115). The same kernel runs the expert-parallel items' gate/up
 * and down (lbk_moe_layer_set_tensor_cores); this entry exposes it for any
 * grouping. All pointers are device memory:
 *   type            LBK_TYPE_IQ2_S or LBK_TYPE_IQ3_S (else LBK_UNSUPPORTED_TYPE);
 *   mats[nmat]      planar matrices of that type and the column of each
 *                   one's first row in a pair's dots;
 *   jobs[njobs][4]  per job {matrix, first row (a multiple of 128), first
 *                   pair, pairs (1..32)}: one CTA computes 128 rows of the
 *                   matrix for those pairs;
 *   q8              token images (the layout lbk_ep_route writes: per 256
 *                   block 304 bytes -- 256 qs, 16 int16 bsums, f32 d, 12
 *                   bytes of padding), q8_row_bytes apart;
 *   pair_tokens     pair -> token;
 *   dots            [pairs][dots_stride] f32 (only the jobs' rows written).
 * A malformed job is reported as LBK_INVALID_PARAMETER (index: the job). */
typedef struct lbk_tc_matrix {
    const void* data;
    uint32_t rows, blocks; /* blocks: 256-weight blocks per row */
    uint64_t out_offset;
} lbk_tc_matrix;
int32_t lbk_tc_grouped_dots(lbk_context* ctx, int32_t type, const lbk_tc_matrix* mats, uint32_t nmat,
                            const uint32_t* jobs, uint32_t njobs, const uint8_t* q8, uint64_t q8_row_bytes,
                            const uint32_t* pair_tokens, float* dots, uint64_t dots_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LIGHTBRIDGE_KERNELS_H */
