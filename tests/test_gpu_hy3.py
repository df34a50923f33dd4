"""GPU end-to-end pin on the reference's reduced two-block Hy3 model.

The reduced model (bridge-test-model/src/hy3.rs) runs the teacher-forced
tokens [3, 7] in the LlamaQ8K execution mode with every quantized GEMV (the
Q4_K / Q5_K / IQ2_S / IQ3_S attention projections, the Q4_K router and the
IQ3_S vocabulary projection), every RMSNorm and residual add, the dense
block's SwiGLU expert, the top-2 routing and block 1's routed + shared expert
combine on the device through the C ABI (lbk_gemv, lbk_rms_norm,
lbk_residual_add, lbk_expert_swiglu_accumulate, lbk_route_topk,
lbk_moe_routed on a registered layer). Per-head norm, RoPE, attention and
softmax stay on the host (they are outside the expert path). Every named
output must have the SHA-256 the reference records for this mode
(hy3_logits.rs:69-112 over hy3-oracle-v1.json), so the device results are bit
for bit the reference's, through two blocks and a KV cache.

The reduced router is a Q4_K matrix (the layer's own router is F32), so the
logits come from lbk_gemv and the routing from lbk_route_topk; the layer is
registered with the router decoded to F32 and runs only the experts.
"""

import json

import numpy as np
import pytest
import torch

import hy3_model as hm
import lbk
import oracle as orc
from conftest import REPO
from gpu_helpers import clean_status, ctx, dev, host, planar_dev

pytestmark = pytest.mark.gpu

FIXTURE = json.loads((REPO / "tests/golden/hy3-oracle-v1.json").read_text())
LLAMA = json.loads((REPO / "tests/golden/hy3-llama-oracle-v1.json").read_text())


class DeviceOps:
    """The LlamaQ8K path on the device; matrices in the GGUF or planar layout."""

    def __init__(self, model: hm.ReducedHy3, layout: int):
        self.layout = layout
        self._mats = {}
        self._keep = []
        self.calls = 0
        self.ws = None
        self.moe_layer = self._layer(model)

    def _matrix(self, m: hm.Mat) -> lbk.Matrix:
        key = id(m)
        if key not in self._mats:
            t = planar_dev(m.ty, m.data, m.in_w) if self.layout == lbk.LAYOUT_PLANAR else dev(m.data)
            self._keep.append(t)
            self._mats[key] = lbk.matrix(m.ty, m.in_w, m.out_w, t, self.layout)
        return self._mats[key]

    def _expert(self, e: hm.Expert) -> lbk.Expert:
        return lbk.Expert(self._matrix(e.gate), self._matrix(e.up), self._matrix(e.down))

    def _layer(self, model: hm.ReducedHy3) -> lbk.MoeLayer:
        r = model.router
        router_f32 = np.concatenate([
            orc.decode_row(r.ty, r.data[i * r.data.size // r.out_w:(i + 1) * r.data.size // r.out_w], r.in_w)
            for i in range(r.out_w)
        ]).astype(np.float32)
        rt = dev(router_f32)
        self.bias = dev(model.selection_bias)
        self._keep += [rt, self.bias]
        rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, hm.HIDDEN, hm.EXPERTS, rt.data_ptr(), rt.numel() * 4)
        layer = lbk.MoeLayer(ctx(), [self._expert(e) for e in model.experts], self._expert(model.shared), rm,
                             self.bias, hm.USED, hm.WEIGHT_SCALE)
        self.layer_ws = torch.zeros(layer.workspace_bytes(1), dtype=torch.uint8, device="cuda")
        return layer

    def rms_norm(self, x, weight):
        out = torch.empty(hm.HIDDEN, device="cuda")
        ctx().rms_norm(dev(x), dev(weight), hm.HIDDEN, 1, hm.EPS, out, lbk.ROUTER_SEQUENTIAL)
        self.calls += 1
        return host(out)

    def residual_add(self, dest, src):
        d = dev(dest)
        ctx().residual_add(d, dev(src), dest.size)
        self.calls += 1
        dest[:] = host(d)

    def gemv(self, m: hm.Mat, x):
        y = torch.empty(m.out_w, device="cuda")
        ctx().gemv(self._matrix(m), dev(np.asarray(x, np.float32)), y)
        self.calls += 1
        return host(y)

    def _accumulate(self, e: hm.Expert, x, out, coefficient):
        ex = self._expert(e)
        ws = torch.zeros(ctx().expert_workspace_bytes(ex), dtype=torch.uint8, device="cuda")
        ctx().expert_swiglu_accumulate(ex, x, out, float(coefficient), ws)
        self.calls += 1

    def dense_ffn(self, e: hm.Expert, x):
        out = torch.zeros(hm.HIDDEN, device="cuda")  # 0 + 1.0 * dot == dot
        self._accumulate(e, dev(x), out, 1.0)
        return host(out)

    def moe_ffn(self, model: hm.ReducedHy3, x):
        xd = dev(np.asarray(x, np.float32))
        logits = dev(self.gemv(model.router, x))
        routed = torch.zeros(hm.USED * 2, dtype=torch.int32, device="cuda")
        ctx().route_topk(logits, self.bias, hm.EXPERTS, 1, hm.USED, hm.WEIGHT_SCALE, routed)
        out = torch.full((hm.HIDDEN,), float("nan"), device="cuda")
        self.moe_layer.routed(xd, 1, routed, out, self.layer_ws)
        self.calls += 2
        r = host(routed)
        return host(out), r[0::2].view(np.uint32), r[1::2].view(np.float32)


@pytest.mark.parametrize("layout", [lbk.LAYOUT_GGUF, lbk.LAYOUT_PLANAR], ids=["gguf", "planar"])
def test_reduced_model_device_path_matches_reference_hashes(layout):
    model = hm.ReducedHy3()
    ops = DeviceOps(model, layout)
    steps = next(m["steps"] for m in FIXTURE["modes"] if m["mode"] == "llama_q8_k")
    session = hm.Session()
    for step in steps:
        rec = hm.evaluate_token(model, session, ops, step["token_id"])
        clean_status()
        assert rec["selected_experts"] == step["selected_experts"]
        assert rec["greedy_id"] == step["greedy_id"]
        got = hm.hashes(rec)
        bad = sorted(k for k in step["hashes"] if got[k] != step["hashes"][k])
        assert not bad, f"token {step['token_id']}: {bad}"
        # and within llama_logits.rs:45-71's tolerances of llama.cpp's run
        llama = next(x for x in LLAMA["steps"] if x["token_id"] == step["token_id"])
        assert rec["selected_experts"] == llama["selected_experts"]
        hm.assert_close(rec["final.logits"], llama["logits"], 3.0e-4, 3.0e-4)
        hm.assert_close(rec["final.probabilities"], llama["probabilities"], 5.0e-5, 5.0e-5)
    assert ops.calls > 0
    ops.moe_layer.close()


def test_reduced_model_block1_ffn_through_the_layer_equals_the_oracle_record():
    """Block 1's FFN on the device from the oracle's own ffn_normalized, for
    both tokens: the routed + shared combine equals the oracle bit for bit."""
    model = hm.ReducedHy3()
    ops = DeviceOps(model, lbk.LAYOUT_PLANAR)
    session = hm.Session()
    for token in (3, 7):
        rec = hm.evaluate_token(model, session, hm.OracleOps("llama_q8_k"), token)
        delta, ids, coefs = ops.moe_ffn(model, rec["block1.ffn_normalized"])
        clean_status()
        assert list(ids) == rec["selected_experts"]
        np.testing.assert_array_equal(coefs.view(np.uint32), rec["coefficients"].view(np.uint32))
        np.testing.assert_array_equal(delta.view(np.uint32), rec["block1.ffn_delta"].view(np.uint32))
    ops.moe_layer.close()
