"""Pins the oracle end to end on the reference's reduced two-block Hy3 model.

For both execution modes (DequantF32 and LlamaQ8K) and the teacher-forced
tokens [3, 7], every named f32 output of both blocks and of the head must have
the SHA-256 the reference records (bridge-test-model/tests/hy3_logits.rs:69-112,
fixture hy3-oracle-v1.json copied to tests/golden/), with the same selected
experts and greedy token. This checks the weight generators, RMSNorm, the
per-head norm, YaRN RoPE, GQA attention over the KV rows, both GEMV modes,
routing, the expert combine and softmax together. The other tests mirror the
reference's session tests (hy3_logits.rs:114-164).
"""

import json

import numpy as np
import pytest

import hy3_model as hm
import oracle as orc
from conftest import REPO

FIXTURE = json.loads((REPO / "tests/golden/hy3-oracle-v1.json").read_text())
LLAMA = json.loads((REPO / "tests/golden/hy3-llama-oracle-v1.json").read_text())



def test_fixture_shape():
    assert FIXTURE["format"] == "lightbridge-reduced-hy3-oracle-v1"
    assert FIXTURE["token_ids"] == [3, 7]
    assert [m["mode"] for m in FIXTURE["modes"]] == list(hm.MODES)


@pytest.mark.parametrize("mode", hm.MODES)
def test_two_step_sequence_matches_reference_hashes(mode):
    model = hm.ReducedHy3()
    steps = next(m["steps"] for m in FIXTURE["modes"] if m["mode"] == mode)
    session = hm.Session()
    for step in steps:
        rec = hm.evaluate_token(model, session, hm.OracleOps(mode), step["token_id"])
        assert abs(float(np.sum(rec["final.probabilities"], dtype=np.float32)) - 1.0) <= 1e-5
        assert rec["final.logits"].size == hm.VOCAB and rec["final.hidden"].size == hm.HIDDEN
        assert rec["selected_experts"] == step["selected_experts"]
        assert rec["greedy_id"] == step["greedy_id"]
        assert hm.hashes(rec) == step["hashes"]
    assert session.position == 2
    assert [len(k) for k in session.keys] == [2, 2]


def test_llama_q8k_mode_matches_llama_cpp_logits():
    """The same model run by llama.cpp b10153 (llama_logits.rs:45-71): the
    LlamaQ8K logits within 3e-4 + 3e-4 |want| and probabilities within
    5e-5 + 5e-5 |want|, same selected experts and greedy tokens."""
    assert LLAMA["format"] == "lightbridge-llama-hy3-oracle-v1"
    model = hm.ReducedHy3()
    session = hm.Session()
    for step in LLAMA["steps"]:
        rec = hm.evaluate_token(model, session, hm.OracleOps("llama_q8_k"), step["token_id"])
        assert rec["selected_experts"] == step["selected_experts"]
        assert rec["greedy_id"] == step["greedy_id"]
        hm.assert_close(rec["final.logits"], step["logits"], 3.0e-4, 3.0e-4)
        hm.assert_close(rec["final.probabilities"], step["probabilities"], 5.0e-5, 5.0e-5)


def test_execution_modes_are_numerically_distinct():
    model = hm.ReducedHy3()
    a = hm.evaluate_token(model, hm.Session(), hm.OracleOps("dequant_f32"), 3)
    b = hm.evaluate_token(model, hm.Session(), hm.OracleOps("llama_q8_k"), 3)
    assert hm.f32_hash(a["final.logits"]) != hm.f32_hash(b["final.logits"])


def test_fresh_session_repeats_the_first_token():
    model = hm.ReducedHy3()
    ops = hm.OracleOps("dequant_f32")
    s = hm.Session()
    first = hm.f32_hash(hm.evaluate_token(model, s, ops, 5)["final.logits"])
    hm.evaluate_token(model, s, ops, 9)
    again = hm.f32_hash(hm.evaluate_token(model, hm.Session(), ops, 5)["final.logits"])
    assert first == again


def test_invalid_token_rejected_before_session_changes():
    s = hm.Session()
    with pytest.raises(ValueError):
        hm.evaluate_token(hm.ReducedHy3(), s, hm.OracleOps("dequant_f32"), hm.VOCAB)
    assert s.position == 0 and s.keys == [[], []]


def test_one_changed_expert_byte_changes_only_what_follows_it():
    """A planted change in routed expert 2's down matrix (selected for token
    3) must change block 1's FFN delta hash but not its normalized input."""
    model = hm.ReducedHy3()
    model.experts[2].down.data[200] ^= 0x10
    step = FIXTURE["modes"][1]["steps"][0]
    rec = hm.evaluate_token(model, hm.Session(), hm.OracleOps("llama_q8_k"), step["token_id"])
    h = hm.hashes(rec)
    assert h["block1.ffn_normalized"] == step["hashes"]["block1.ffn_normalized"]
    assert h["block1.ffn_delta"] != step["hashes"]["block1.ffn_delta"]


def test_f32_to_f16_rounds_to_nearest_even():
    rng = np.random.default_rng(3)
    v = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    edge = np.array([65504, 65519.99, 65520, 1e-8, 2 ** -25, 2 ** -24, 3 * 2 ** -26, 6e-5, -0.0, 0.00035, 4.375e-5],
                    np.float32)
    v = np.concatenate([v[np.abs(v) < 65520], edge])
    got = np.array([orc.f32_to_f16(x) for x in v], np.uint16)
    with np.errstate(over="ignore"):  # 65520 rounds to infinity
        want = v.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(got, want)
