"""The reference's reduced two-block Hy3 model, run token by token.

TEST INFRASTRUCTURE: the end-to-end pin of the expert path. The reference
checks this model's named f32 outputs by SHA-256
(bridge-test-model/tests/hy3_logits.rs:69-112 against
tests/fixtures/hy3-oracle-v1.json, copied to tests/golden/): block 0 is dense
(attention + one SwiGLU expert), block 1 is MoE (attention, Q4_K router,
top-2 of 4 routed experts and a shared expert), then the output RMSNorm, the
IQ3_S vocabulary projection and softmax.

The weights are generated exactly as bridge-test-model/src/hy3.rs:268-321
does (through the oracle's restatement of its generators). A token runs
through `evaluate_token` with an `ops` object that supplies the GEMVs, RMSNorms,
residual adds and the two feed-forward halves: `OracleOps` is the reference's
CPU path in one execution mode; the GPU test supplies the device path through
the C-ABI. Per-head norm, RoPE, attention and softmax always run in the oracle
(they are outside the expert path).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

import oracle as orc

# hy3.rs:21-31 and reduced_config (:705-729)
HIDDEN = 256
Q_HEADS, KV_HEADS, HEAD_DIM = 4, 2, 64
DENSE_FFN = EXPERT_FFN = 256
EXPERTS, USED = 4, 2
VOCAB = 32
CONTEXT = 1024
EPS = 1.0e-5
WEIGHT_SCALE = 1.75
# Hy3RopeParams::from_config (rope.rs:21-82): YaRN factor 4 over 256 original tokens
ROPE = orc.Rope(HEAD_DIM, CONTEXT, CONTEXT // 4, 10000.0, 0.25, 1.0, 1.0, 32.0, 1.0)

BLOCK_OUTPUTS = ("attention_normalized", "queries", "keys", "values", "attention_context", "attention_delta",
                 "attention_residual", "ffn_normalized", "ffn_delta")
MODES = ("dequant_f32", "llama_q8_k")

Q4, Q5, I2, I3 = orc.TYPE_Q4_K, orc.TYPE_Q5_K, orc.TYPE_IQ2_S, orc.TYPE_IQ3_S


@dataclass
class Mat:
    ty: int
    in_w: int
    out_w: int
    data: np.ndarray  # GGUF layout bytes


@dataclass
class Expert:
    gate: Mat
    up: Mat
    down: Mat


@dataclass
class Attention:
    input_norm: np.ndarray
    query: Mat
    query_norm: np.ndarray
    key: Mat
    key_norm: np.ndarray
    value: Mat
    output: Mat


def _mat(ty: int, in_w: int, out_w: int, seed: int) -> Mat:
    return Mat(ty, in_w, out_w, orc.hy3_fill_matrix(ty, in_w, out_w, seed))


def _expert(types, seed: int, ffn: int) -> Expert:
    """OwnedExpert::new, hy3.rs:138-144."""
    return Expert(_mat(types[0], HIDDEN, ffn, seed), _mat(types[1], HIDDEN, ffn, seed + 1),
                  _mat(types[2], ffn, HIDDEN, seed + 2))


def _attention(types, seed: int) -> Attention:
    """OwnedAttention::new, hy3.rs:167-187."""
    return Attention(
        input_norm=orc.hy3_norm_weights(HIDDEN, seed),
        query=_mat(types[0], HIDDEN, Q_HEADS * HEAD_DIM, seed + 1),
        query_norm=orc.hy3_norm_weights(HEAD_DIM, seed + 2),
        key=_mat(types[1], HIDDEN, KV_HEADS * HEAD_DIM, seed + 3),
        key_norm=orc.hy3_norm_weights(HEAD_DIM, seed + 4),
        value=_mat(types[2], HIDDEN, KV_HEADS * HEAD_DIM, seed + 5),
        output=_mat(types[3], Q_HEADS * HEAD_DIM, HIDDEN, seed + 6),
    )


class ReducedHy3:
    """ReducedHy3Model::new, hy3.rs:268-321."""

    def __init__(self):
        self.embeddings = orc.hy3_embeddings(VOCAB * HIDDEN).reshape(VOCAB, HIDDEN)
        self.dense_attention = _attention([Q4, Q5, I2, I3], 0x1001)
        self.dense_ffn_norm = orc.hy3_norm_weights(HIDDEN, 0x1101)
        self.dense_expert = _expert([I2, Q4, Q5], 0x1201, DENSE_FFN)
        self.moe_attention = _attention([I3, I2, Q5, Q4], 0x2001)
        self.moe_ffn_norm = orc.hy3_norm_weights(HIDDEN, 0x2101)
        self.router = _mat(Q4, HIDDEN, EXPERTS, 0x2201)
        self.selection_bias = np.array([0.025, -0.0125, 0.0375, -0.02], dtype=np.float32)
        self.experts = [_expert([I2, Q5, I3], 0x2301 + 0x100 * e, EXPERT_FFN) for e in range(EXPERTS)]
        self.shared = _expert([I2, I3, Q4], 0x2701, EXPERT_FFN)
        self.output_norm = orc.hy3_norm_weights(HIDDEN, 0x3001)
        self.output = _mat(I3, HIDDEN, VOCAB, 0x3101)


@dataclass
class Session:
    """ReducedHy3Session (hy3.rs:646-687): position and the per-block f32 KV
    rows ([token][kv_head][dim], PagedKvCache stores them unchanged)."""

    position: int = 0
    keys: list = field(default_factory=lambda: [[], []])
    values: list = field(default_factory=lambda: [[], []])


class OracleOps:
    """The reference's CPU kernels in one execution mode: DequantF32 (decode
    then one f32 chain per row, gemv.rs:33-41) or LlamaQ8K (Q8_K activations,
    the scalar vec_dot_q8_k, gemv.rs:43-54)."""

    def __init__(self, mode: str):
        assert mode in MODES
        self.mode = mode

    def rms_norm(self, x, weight):
        return orc.rms_norm(x, weight, EPS)

    def residual_add(self, dest, src):
        st = orc.residual_add_status(dest, src)
        assert st == 0, st

    def gemv(self, m: Mat, x):
        if self.mode == "dequant_f32":
            return orc.gemv_dequant(m.ty, m.in_w, m.out_w, m.data, x)
        return orc.gemv(m.ty, m.in_w, m.out_w, m.data, x, simd=False, threads=1)[0]

    def _accumulate(self, m: Mat, x, y, scale):
        if self.mode == "dequant_f32":
            orc.gemv_dequant_accumulate_scaled(m.ty, m.in_w, m.out_w, m.data, x, y, scale)
        else:
            orc.gemv_accumulate_scaled(m.ty, m.in_w, m.out_w, m.data, x, y, scale, simd=False, threads=1)

    def dense_ffn(self, e: Expert, x):
        """swiglu_project_into, activation.rs:65-102."""
        act = orc.swiglu(self.gemv(e.gate, x), self.gemv(e.up, x))
        return self.gemv(e.down, act)

    def _expert_accumulate(self, e: Expert, x, y, coefficient):
        """expert_swiglu_accumulate_into, activation.rs:104-144."""
        act = orc.swiglu(self.gemv(e.gate, x), self.gemv(e.up, x))
        self._accumulate(e.down, act, y, coefficient)

    def moe_ffn(self, model: ReducedHy3, x):
        """Router GEMV and route_experts_into (layer.rs:588-605), then
        moe_selected_into (moe.rs:29-58): routed experts in ascending ID, then
        the shared expert at 1.0. Returns (delta, ids, coefficients)."""
        logits = self.gemv(model.router, x)
        ids, coefs = orc.route_experts(logits, model.selection_bias, USED, WEIGHT_SCALE)
        out = np.zeros(HIDDEN, dtype=np.float32)
        for i, c in zip(ids, coefs):
            self._expert_accumulate(model.experts[int(i)], x, out, c)
        self._expert_accumulate(model.shared, x, out, 1.0)
        return out, ids, coefs


def evaluate_token(model: ReducedHy3, session: Session, ops, token: int) -> dict:
    """ReducedHy3Model::evaluate_token (hy3.rs:433-530) with
    hy3_block_forward_token / hy3_moe_route_token + finish
    (layer.rs:309-472, :473-659). Returns every named output of the
    reference's record, plus "selected_experts", "coefficients" and
    "greedy_id"."""
    if not 0 <= token < VOCAB:
        raise ValueError(f"token ID {token} is outside vocabulary size {VOCAB}")
    if session.position >= CONTEXT:
        raise ValueError("position out of range")
    out = {}
    hidden = model.embeddings[token].copy()
    blocks = [(model.dense_attention, model.dense_ffn_norm), (model.moe_attention, model.moe_ffn_norm)]
    for layer, (att, ffn_norm) in enumerate(blocks):
        rec = {}
        rec["attention_normalized"] = ops.rms_norm(hidden, att.input_norm)
        q = ops.gemv(att.query, rec["attention_normalized"])
        k = ops.gemv(att.key, rec["attention_normalized"])
        v = ops.gemv(att.value, rec["attention_normalized"])
        q = orc.head_rms_norm(q, att.query_norm, HEAD_DIM, EPS)
        k = orc.head_rms_norm(k, att.key_norm, HEAD_DIM, EPS)
        rec["queries"] = orc.rope_neox_yarn(q, Q_HEADS, session.position, ROPE)
        rec["keys"] = orc.rope_neox_yarn(k, KV_HEADS, session.position, ROPE)
        rec["values"] = np.asarray(v, dtype=np.float32)
        stored = len(session.keys[layer])
        ck = np.concatenate(session.keys[layer]) if stored else np.zeros(0, np.float32)
        cv = np.concatenate(session.values[layer]) if stored else np.zeros(0, np.float32)
        rec["attention_context"] = orc.gqa_attention(ck, cv, stored, Q_HEADS, KV_HEADS, HEAD_DIM, rec["queries"],
                                                     rec["keys"], rec["values"])
        session.keys[layer].append(rec["keys"].copy())
        session.values[layer].append(rec["values"].copy())
        rec["attention_delta"] = ops.gemv(att.output, rec["attention_context"])
        ops.residual_add(hidden, rec["attention_delta"])
        rec["attention_residual"] = hidden.copy()
        rec["ffn_normalized"] = ops.rms_norm(hidden, ffn_norm)
        if layer == 0:
            rec["ffn_delta"] = ops.dense_ffn(model.dense_expert, rec["ffn_normalized"])
        else:
            rec["ffn_delta"], ids, coefs = ops.moe_ffn(model, rec["ffn_normalized"])
            out["selected_experts"] = [int(i) for i in ids]
            out["coefficients"] = np.asarray(coefs, dtype=np.float32)
        ops.residual_add(hidden, rec["ffn_delta"])
        for name in BLOCK_OUTPUTS:
            out[f"block{layer}.{name}"] = np.asarray(rec[name], dtype=np.float32)
    out["final.hidden"] = hidden.copy()
    out["final.normalized"] = ops.rms_norm(hidden, model.output_norm)
    out["final.logits"] = np.asarray(ops.gemv(model.output, out["final.normalized"]), dtype=np.float32)
    out["final.probabilities"] = orc.softmax(out["final.logits"])
    logits = out["final.logits"]
    greedy = 0
    for i in range(1, logits.size):  # greedy_id, hy3.rs:748-756: first strict maximum
        if logits[i] > logits[greedy]:
            greedy = i
    out["greedy_id"] = greedy
    session.position += 1
    return out


def f32_hash(values) -> str:
    """f32_hash of hy3_logits.rs:32-38: SHA-256 of the little-endian bits."""
    return hashlib.sha256(np.ascontiguousarray(values, dtype="<f4").tobytes()).hexdigest()


def hashes(record: dict) -> dict:
    return {k: f32_hash(v) for k, v in record.items() if k.startswith(("block", "final."))}


def assert_close(got, want, atol, rtol):
    """assert_close of llama_logits.rs:34-43: |got - want| <= atol + rtol |want| (f32)."""
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape
    tol = np.float32(atol) + np.float32(rtol) * np.abs(want)
    bad = np.nonzero(np.abs(got - want) > tol)[0]
    assert bad.size == 0, f"values {bad[:8]}: got {got[bad[:8]]}, want {want[bad[:8]]}"
