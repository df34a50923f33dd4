"""GPU parity of the routed + shared SwiGLU MoE layer against the CPU oracle
(route_experts_into + moe_routed_by_id_into, i.e. hy3_moe_route_token /
hy3_moe_finish_token without norm and residual).

Bars (north star): top-k expert IDs identical; f32 outputs within 1e-5
relative (norm-wise). Stages that call exp (sigmoid, SwiGLU) use CUDA's
double exp rounded to f32 where the reference uses the platform expf, so
the layer output is held to the tolerance; every integer sum and every
exp-free f32 tail is bit-exact (tests/test_gpu_quant_dot.py).
Also covers the combine order of bridge-kernels-reference/tests/moe.rs:106-153
and validate-before-write (moe.rs:156-244).
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
from gpu_helpers import (bits, clean_status, ctx, dev, errs, expect_status, host, make_layer_np, moe_term_magnitude,
                         rel_err, topk_margins, upload_layer)

pytestmark = pytest.mark.gpu

TOL = 1e-5


def run_forward(layer, xs, mode=lbk.ROUTER_TREE):
    T, H = xs.shape
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.full((T * H,), float("nan"), device="cuda")
    routed = torch.zeros(T * layer.top_k * 2, dtype=torch.int32, device="cuda")
    layer.forward(dev(xs.reshape(-1)), T, out, ws, routed_out=routed, router_mode=mode)
    clean_status()
    r = host(routed).reshape(T, layer.top_k, 2)
    return host(out).reshape(T, H), r[:, :, 0].astype(np.uint32), r[:, :, 1].view(np.float32)


def oracle_tokens(router, experts, shared, xs, k):
    """Oracle outputs, routing and (for the tolerance) each output row's term magnitude."""
    table = orc.ExpertTable(experts, shared, router=router, hidden=xs.shape[1])
    E = len(experts)
    outs, ids, coefs, mags = [], [], [], []
    for x in xs:
        o, i, c = orc.moe_token(table, np.zeros(E, np.float32), k, 2.826, x)
        outs.append(o)
        ids.append(i)
        coefs.append(c)
        mags.append(moe_term_magnitude(table, i, c, x))
    return np.stack(outs), np.stack(ids), np.stack(coefs), np.stack(mags)


@pytest.mark.parametrize("layout", [lbk.LAYOUT_PLANAR, lbk.LAYOUT_GGUF])
@pytest.mark.parametrize("H,F,E,k,T", [(512, 256, 8, 2, 1), (1024, 512, 16, 4, 3), (768, 768, 12, 3, 2)])
def test_small_layers_match_oracle(H, F, E, k, T, layout):
    rng = np.random.default_rng(H + F + E + k)
    router, experts, shared = make_layer_np(rng, H, F, E)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    layer, keep = upload_layer(router, experts, shared, layout, k)
    assert layer.fused == (layout == lbk.LAYOUT_PLANAR)
    for mode in (lbk.ROUTER_TREE, lbk.ROUTER_SEQUENTIAL):
        out, ids, coefs = run_forward(layer, xs, mode)
        want, wids, wcoefs, mag = oracle_tokens(router, experts, shared, xs, k)
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_allclose(coefs, wcoefs, rtol=1e-6)
        assert rel_err(out, want, mag) <= TOL, errs(out, want, mag)
    layer.close()


def test_fused_and_per_expert_paths_are_bit_identical():
    rng = np.random.default_rng(77)
    H, F, E, k, T = 1024, 512, 16, 4, 2
    router, experts, shared = make_layer_np(rng, H, F, E)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    lp, kp = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    lg, kg = upload_layer(router, experts, shared, lbk.LAYOUT_GGUF, k)
    a, ia, _ = run_forward(lp, xs, lbk.ROUTER_SEQUENTIAL)
    b, ib, _ = run_forward(lg, xs, lbk.ROUTER_SEQUENTIAL)
    np.testing.assert_array_equal(ia, ib)
    np.testing.assert_array_equal(bits(a), bits(b))
    lp.close()
    lg.close()


@pytest.mark.parametrize("H,F,E,k,T", [(2048, 512, 8, 2, 1), (4096, 768, 12, 4, 3), (2048, 256, 16, 8, 1)])
def test_bulk_staged_gate_up_matches_oracle_and_per_expert_path(H, F, E, k, T):
    """Hidden widths of 8 or 16 blocks take the bulk-copy-staged gate/up
    kernel (routed and shared CTA roles); the result must equal the oracle to
    the tolerance and the per-expert GGUF path bit for bit."""
    rng = np.random.default_rng(H + 3 * F + E + k + T)
    router, experts, shared = make_layer_np(rng, H, F, E)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    lp, kp = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    lg, kg = upload_layer(router, experts, shared, lbk.LAYOUT_GGUF, k)
    want, wids, wcoefs, mag = oracle_tokens(router, experts, shared, xs, k)
    for mode in (lbk.ROUTER_TREE, lbk.ROUTER_SEQUENTIAL):
        out, ids, coefs = run_forward(lp, xs, mode)
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_allclose(coefs, wcoefs, rtol=1e-6)
        assert rel_err(out, want, mag) <= TOL, errs(out, want, mag)
        ref, rids, _ = run_forward(lg, xs, mode)
        np.testing.assert_array_equal(ids, rids)
        np.testing.assert_array_equal(bits(out), bits(ref))
    lp.close()
    lg.close()


@pytest.mark.parametrize("H,F,E,k", [(2048, 512, 8, 2), (1024, 512, 16, 4)])
def test_one_workspace_serves_every_token_count(H, F, E, k):
    """A workspace zero-filled once and sized for the largest call stays valid
    across calls with different token counts (its regions move with T)."""
    rng = np.random.default_rng(H + F + 11 * k)
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    ws = torch.zeros(layer.workspace_bytes(4), dtype=torch.uint8, device="cuda")
    for T, mode in [(1, lbk.ROUTER_TREE), (4, lbk.ROUTER_TREE), (2, lbk.ROUTER_SEQUENTIAL), (1, lbk.ROUTER_SEQUENTIAL),
                    (3, lbk.ROUTER_TREE), (1, lbk.ROUTER_TREE)]:
        xs = rng.standard_normal((T, H)).astype(np.float32)
        want, wids, _ = run_forward(layer, xs, mode)  # fresh workspace
        out = torch.full((T * H,), float("nan"), device="cuda")
        routed = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
        layer.forward(dev(xs.reshape(-1)), T, out, ws, routed_out=routed, router_mode=mode)
        clean_status()
        np.testing.assert_array_equal(host(routed).reshape(T, k, 2)[:, :, 0].astype(np.uint32), wids)
        np.testing.assert_array_equal(bits(host(out).reshape(T, H)), bits(want))
    layer.close()


@pytest.mark.parametrize("H,F,E,k", [(2048, 512, 16, 4), (4096, 1536, 192, 8)])
def test_queued_single_token_calls_on_one_workspace(H, F, E, k):
    """Single-token calls queued back to back on one workspace, with no host
    synchronization between them and routing that changes from call to call,
    plus several-token calls between them: every output and routing equals a
    fresh-workspace run bit for bit. A routing flag or routing left over from
    an earlier call would stream the wrong experts here."""
    rng = np.random.default_rng(H + E + 31 * k)
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    plan = [3] + [1] * 12 + [3, 1, 2, 1, 1]
    xs = [rng.standard_normal((T, H)).astype(np.float32) for T in plan]
    wants = [run_forward(layer, x) for x in xs]  # each on a fresh workspace
    ws = torch.zeros(layer.workspace_bytes(max(plan)), dtype=torch.uint8, device="cuda")
    xd = [dev(x.reshape(-1)) for x in xs]
    outs = [torch.full((T * H,), float("nan"), device="cuda") for T in plan]
    routs = [torch.zeros(T * k * 2, dtype=torch.int32, device="cuda") for T in plan]
    torch.cuda.synchronize()
    for T, x, o, r in zip(plan, xd, outs, routs):
        layer.forward(x, T, o, ws, routed_out=r)
    clean_status()
    singles = [i for i, T in enumerate(plan) if T == 1]
    changed = sum(not np.array_equal(wants[a][1], wants[b][1]) for a, b in zip(singles, singles[1:]))
    assert changed >= len(singles) // 2, "routing should change between the queued calls"
    for i, T in enumerate(plan):
        want, wids, _ = wants[i]
        ids = host(routs[i]).reshape(T, k, 2)[:, :, 0].astype(np.uint32)
        np.testing.assert_array_equal(ids, wids, err_msg=f"call {i}")
        np.testing.assert_array_equal(bits(host(outs[i]).reshape(T, H)), bits(want), err_msg=f"call {i}")
    layer.close()


def test_routing_wait_that_runs_out_reports_timeout():
    """The down kernel's bounded wait for the single-token routing flag (a
    wait with no copy in flight) made to run out with a zero poll limit:
    LBK_TIMEOUT through the status word, the output left unwritten, and the
    workspace and context still usable for the next call."""
    rng = np.random.default_rng(15)
    H, F, E, k = 2048, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    x = rng.standard_normal((1, H)).astype(np.float32)
    want, wids, _ = run_forward(layer, x)
    ws = torch.zeros(layer.workspace_bytes(1), dtype=torch.uint8, device="cuda")
    sentinel = np.full(H, 7.5, np.float32)
    out = dev(sentinel)
    layer.set_wait_limit(0)
    layer.forward(dev(x.reshape(-1)), 1, out, ws)
    d = expect_status(31)
    assert d.index == 4
    np.testing.assert_array_equal(host(out), sentinel)
    layer.set_wait_limit(1 << 20)
    for _ in range(2):
        out2 = torch.full((H,), float("nan"), device="cuda")
        layer.forward(dev(x.reshape(-1)), 1, out2, ws)
        clean_status()
        np.testing.assert_array_equal(bits(host(out2)), bits(want[0]))
    layer.close()


def test_caller_supplied_routing_and_combine_order():
    rng = np.random.default_rng(5)
    H, F, E, k = 512, 256, 8, 3
    router, experts, shared = make_layer_np(rng, H, F, E)
    x = rng.standard_normal((1, H)).astype(np.float32)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    ids = np.array([1, 4, 6], np.uint32)
    coefs = np.array([0.25, 0.75, -1.5], np.float32)
    rt = np.zeros(k * 2, np.int32)
    rt[0::2] = ids.view(np.int32)
    rt[1::2] = coefs.view(np.int32)
    ws = torch.zeros(layer.workspace_bytes(1), dtype=torch.uint8, device="cuda")
    out = torch.zeros(H, device="cuda")
    layer.routed(dev(x.reshape(-1)), 1, dev(rt), out, ws)
    clean_status()
    table = orc.ExpertTable(experts, shared)
    want = orc.moe_routed(table, ids, coefs, x[0], preflight=True)
    assert rel_err(host(out), want) <= TOL
    layer.close()


@pytest.mark.parametrize(
    "ids,code", [([3, 3, 5], 14), ([4, 2, 5], 13), ([1, 2, 99], 15)]
)
def test_bad_routing_rejected_before_output_write(ids, code):
    rng = np.random.default_rng(6)
    H, F, E, k = 512, 256, 8, 3
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    rt = np.zeros(k * 2, np.int32)
    rt[0::2] = np.array(ids, np.uint32).view(np.int32)
    rt[1::2] = np.ones(k, np.float32).view(np.int32)
    ws = torch.zeros(layer.workspace_bytes(1), dtype=torch.uint8, device="cuda")
    sentinel = np.full(H, -4.25, np.float32)
    out = dev(sentinel)
    layer.routed(dev(rng.standard_normal(H).astype(np.float32)), 1, dev(rt), out, ws)
    expect_status(code)
    np.testing.assert_array_equal(host(out), sentinel)
    layer.close()


def test_non_finite_token_leaves_output_unchanged():
    rng = np.random.default_rng(8)
    H, F, E, k = 512, 256, 8, 2
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    x = rng.standard_normal(H).astype(np.float32)
    x[100] = np.inf
    ws = torch.zeros(layer.workspace_bytes(1), dtype=torch.uint8, device="cuda")
    sentinel = np.full(H, 9.0, np.float32)
    out = dev(sentinel)
    layer.forward(dev(x), 1, out, ws)
    expect_status(12)
    np.testing.assert_array_equal(host(out), sentinel)
    # the workspace stays usable: a clean call afterwards is correct
    x[100] = 0.5
    out2 = torch.zeros(H, device="cuda")
    layer.forward(dev(x), 1, out2, ws)
    clean_status()
    want, _, _, mag = oracle_tokens(router, experts, shared, x[None], k)
    assert rel_err(host(out2), want[0], mag[0]) <= TOL
    layer.close()


def test_config3_layer_single_token():
    """hidden 4096, 192 experts (IQ2_S gate/up, IQ3_S down,
    FFN 1536), shared Q4_K expert, F32 router N(0, 0.02), top-8, seed 2."""
    rng = np.random.default_rng(2)
    H, F, E, k = 4096, 1536, 192, 8
    router, experts, shared = make_layer_np(rng, H, F, E)
    xs = rng.standard_normal((2, H)).astype(np.float32)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    assert layer.fused
    want, wids, wcoefs, mag = oracle_tokens(router, experts, shared, xs, k)
    margins = topk_margins(router, xs, np.zeros(E, np.float32), k)
    print(f"config 3: 8th/9th selection-score margins {margins}")
    for mode in (lbk.ROUTER_TREE, lbk.ROUTER_SEQUENTIAL):
        out, ids, coefs = run_forward(layer, xs, mode)
        np.testing.assert_array_equal(ids, wids)
        np.testing.assert_allclose(coefs, wcoefs, rtol=1e-6)
        assert rel_err(out, want, mag) <= TOL, errs(out, want, mag)
        print(f"config 3, router mode {mode}: {errs(out, want, mag)}")
    layer.close()


# The checkpoint's per-layer types (bridge-model-hy3/src/schema.rs:200-258):
# routed gate/up and shared gate/up IQ2_S; routed down IQ3_S in layers <= 5,
# IQ2_S after; shared down IQ3_S in layers <= 4, IQ2_S after.
CHECKPOINT_TYPES = [
    (orc.TYPE_IQ2_S, orc.TYPE_IQ3_S, orc.TYPE_IQ2_S, orc.TYPE_IQ3_S),  # layers 1-4
    (orc.TYPE_IQ2_S, orc.TYPE_IQ3_S, orc.TYPE_IQ2_S, orc.TYPE_IQ2_S),  # layer 5
    (orc.TYPE_IQ2_S, orc.TYPE_IQ2_S, orc.TYPE_IQ2_S, orc.TYPE_IQ2_S),  # layers 6+
]


@pytest.mark.parametrize("types", CHECKPOINT_TYPES)
@pytest.mark.parametrize("H,F,E,k,T", [(4096, 1536, 24, 8, 1), (2048, 512, 16, 4, 3)])
def test_checkpoint_types_take_the_fused_kernels(types, H, F, E, k, T):
    """Layers of the checkpoint's type mix run on the bulk-copy kernels (IQ
    shared-expert roles with their own tables): oracle to the tolerance, the
    per-expert GGUF path bit for bit."""
    gty, dty, sty, sdty = types
    rng = np.random.default_rng(H + F + E + k + T + sdty)
    router, experts, shared = make_layer_np(rng, H, F, E, gty=gty, dty=dty, sty=sty, sdty=sdty)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    lp, kp = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    lg, kg = upload_layer(router, experts, shared, lbk.LAYOUT_GGUF, k)
    assert lp.fused and not lg.fused
    want, wids, _, mag = oracle_tokens(router, experts, shared, xs, k)
    out, ids, _ = run_forward(lp, xs)
    np.testing.assert_array_equal(ids, wids)
    assert rel_err(out, want, mag) <= TOL, errs(out, want, mag)
    ref, rids, _ = run_forward(lg, xs)
    np.testing.assert_array_equal(bits(out), bits(ref))
    lp.close()
    lg.close()
