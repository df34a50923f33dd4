"""GPU parity of the grouped MoE kernels (calls of several tokens).

With grouping on, the (token, slot) pairs of a call are grouped by routed
expert and every weight half block is decoded once for all pairs of its
group. Each pair's integer block sums, f32 block products and row tails are
the ones of the per-(token, slot) kernels, so the layer output must equal the
ungrouped path bit for bit, and the CPU oracle (moe_routed_by_id_into,
bridge-kernels-reference/src/moe.rs:64-147) to the layer tolerance.
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
from gpu_helpers import (bits, clean_status, dev, errs, expect_status, host, make_layer_np, moe_term_magnitude, rel_err,
                         topk_margins, upload_layer)

pytestmark = pytest.mark.gpu

TOL = 1e-5


def forward(layer, xs, mode=lbk.ROUTER_SEQUENTIAL):
    T, H = xs.shape
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.full((T * H,), float("nan"), device="cuda")
    routed = torch.zeros(T * layer.top_k * 2, dtype=torch.int32, device="cuda")
    layer.forward(dev(xs.reshape(-1)), T, out, ws, routed_out=routed, router_mode=mode)
    clean_status()
    r = host(routed).reshape(T, layer.top_k, 2)
    return host(out).reshape(T, H), r[:, :, 0].astype(np.uint32)


def routed_call(layer, xs, ids, coefs):
    T, H = xs.shape
    k = ids.shape[1]
    rt = np.zeros((T, k, 2), np.int32)
    rt[:, :, 0] = ids.astype(np.uint32).view(np.int32)
    rt[:, :, 1] = coefs.astype(np.float32).view(np.int32)
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.full((T * H,), float("nan"), device="cuda")
    layer.routed(dev(xs.reshape(-1)), T, dev(rt.reshape(-1)), out, ws)
    return out


def grouped_and_plain(layer, fn):
    layer.set_grouping(2)
    a = fn()
    layer.set_grouping(0)
    b = fn()
    layer.set_grouping(8)
    return a, b


@pytest.mark.parametrize(
    "H,F,E,k,T,types",
    [
        (2048, 512, 16, 4, 9, None),
        (4096, 768, 12, 4, 8, None),
        (2048, 256, 16, 8, 17, None),
        (4096, 1536, 24, 8, 33, (orc.TYPE_IQ2_S, orc.TYPE_IQ3_S, orc.TYPE_IQ2_S, orc.TYPE_IQ3_S)),
        (2048, 512, 16, 4, 10, (orc.TYPE_IQ2_S, orc.TYPE_IQ3_S, orc.TYPE_IQ2_S, orc.TYPE_IQ2_S)),
        (2048, 512, 16, 4, 11, (orc.TYPE_IQ2_S, orc.TYPE_IQ2_S, orc.TYPE_IQ2_S, orc.TYPE_IQ2_S)),
        (2048, 512, 16, 2, 12, (orc.TYPE_Q4_K, orc.TYPE_Q4_K, orc.TYPE_Q4_K, orc.TYPE_Q4_K)),
        (2048, 512, 16, 2, 13, (orc.TYPE_IQ2_S, orc.TYPE_IQ2_S, orc.TYPE_Q4_K, orc.TYPE_Q4_K)),
    ],
)
def test_grouped_equals_ungrouped_and_oracle(H, F, E, k, T, types):
    rng = np.random.default_rng(H + F + E + k + T)
    kw = {} if types is None else dict(gty=types[0], dty=types[1], sty=types[2], sdty=types[3])
    router, experts, shared = make_layer_np(rng, H, F, E, **kw)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    assert layer.fused
    for mode in (lbk.ROUTER_SEQUENTIAL, lbk.ROUTER_TREE):
        (a, ia), (b, ib) = grouped_and_plain(layer, lambda: forward(layer, xs, mode))
        np.testing.assert_array_equal(ia, ib)
        np.testing.assert_array_equal(bits(a), bits(b))
    table = orc.ExpertTable(experts, shared, router=router, hidden=H)
    for t in (0, T // 2, T - 1):  # oracle on a few tokens (seconds each at these sizes)
        want, wids, wc = orc.moe_token(table, np.zeros(E, np.float32), k, 2.826, xs[t])
        np.testing.assert_array_equal(ia[t], wids)
        mag = moe_term_magnitude(table, wids, wc, xs[t])
        assert rel_err(a[t], want, mag) <= TOL, errs(a[t], want, mag)
    layer.close()


def test_config3_shapes_64_tokens():
    """BASELINE config 4's layer (hidden 4096, 192 experts, FFN 1536, IQ2_S
    gate/up, IQ3_S down, shared Q4_K, top-8) at 64 tokens, seed 3: grouped
    equals ungrouped bit for bit; every token against the oracle (single pass,
    moe_routed_by_id_into without the preflight, which does not change the
    result)."""
    rng = np.random.default_rng(3)
    H, F, E, k, T = 4096, 1536, 192, 8, 64
    router, experts, shared = make_layer_np(rng, H, F, E)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    (a, ia), (b, ib) = grouped_and_plain(layer, lambda: forward(layer, xs, lbk.ROUTER_TREE))
    np.testing.assert_array_equal(ia, ib)
    np.testing.assert_array_equal(bits(a), bits(b))
    table = orc.ExpertTable(experts, shared, router=router, hidden=H)
    margins = topk_margins(router, xs, np.zeros(E, np.float32), k)
    print(f"config 4: 8th/9th selection-score margin min {margins.min():.3e}, median {np.median(margins):.3e}")
    worst = 0.0
    for t in range(T):
        want, wids, wc = orc.moe_token(table, np.zeros(E, np.float32), k, 2.826, xs[t], preflight=False)
        np.testing.assert_array_equal(ia[t], wids, err_msg=f"token {t}")
        mag = moe_term_magnitude(table, wids, wc, xs[t])
        assert rel_err(a[t], want, mag) <= TOL, f"token {t}: " + errs(a[t], want, mag)
        worst = max(worst, rel_err(a[t], want, mag))
    print(f"config 4: 64 tokens against the oracle, worst element-wise relative error {worst:.3e}")
    layer.close()


@pytest.mark.parametrize("T", [8, 21, 40])
def test_skewed_routing_splits_groups(T):
    """Every token routed to the same few experts: each expert's pairs are cut
    into several groups, every pair still computed exactly once."""
    rng = np.random.default_rng(100 + T)
    H, F, E, k = 2048, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    ids = np.tile(np.array([1, 5, 6, 14], np.uint32), (T, 1))
    ids[::3] = np.array([0, 5, 9, 14], np.uint32)  # some pairs elsewhere
    coefs = rng.uniform(-1.5, 1.5, (T, k)).astype(np.float32)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    a, b = grouped_and_plain(layer, lambda: host(routed_call(layer, xs, ids, coefs)))
    clean_status()
    np.testing.assert_array_equal(bits(a), bits(b))
    table = orc.ExpertTable(experts, shared)
    for t in (0, 1, T - 1):
        want = orc.moe_routed(table, ids[t], coefs[t], xs[t], preflight=True)
        assert rel_err(a.reshape(T, H)[t], want) <= TOL
    layer.close()


def test_grouped_bad_routing_leaves_output_unchanged():
    """An expert ID outside the layer in one token of a grouped call is
    reported (InvalidParameter) and no output row is written."""
    rng = np.random.default_rng(9)
    H, F, E, k, T = 2048, 512, 16, 3, 12
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    layer.set_grouping(2)
    ids = np.tile(np.array([1, 2, 3], np.uint32), (T, 1))
    ids[7] = np.array([1, 2, 99], np.uint32)
    rt = np.zeros((T, k, 2), np.int32)
    rt[:, :, 0] = ids.view(np.int32)
    rt[:, :, 1] = np.ones((T, k), np.float32).view(np.int32)
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    sentinel = np.full(T * H, -4.25, np.float32)
    out = dev(sentinel)
    layer.routed(dev(rng.standard_normal(T * H).astype(np.float32)), T, dev(rt.reshape(-1)), out, ws)
    expect_status(15)
    np.testing.assert_array_equal(host(out), sentinel)
    layer.close()


def test_workspace_reused_across_grouped_and_single_token_calls():
    """One zero-filled workspace sized for the largest call serves grouped
    calls and single-token calls in any order, bit-identical to fresh ones."""
    rng = np.random.default_rng(12)
    H, F, E, k = 2048, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    ws = torch.zeros(layer.workspace_bytes(24), dtype=torch.uint8, device="cuda")
    for T, mode in [(24, lbk.ROUTER_TREE), (1, lbk.ROUTER_TREE), (9, lbk.ROUTER_SEQUENTIAL), (16, lbk.ROUTER_TREE),
                    (1, lbk.ROUTER_SEQUENTIAL), (8, lbk.ROUTER_TREE)]:
        xs = rng.standard_normal((T, H)).astype(np.float32)
        want, wids = forward(layer, xs, mode)
        out = torch.full((T * H,), float("nan"), device="cuda")
        routed = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
        layer.forward(dev(xs.reshape(-1)), T, out, ws, routed_out=routed, router_mode=mode)
        clean_status()
        np.testing.assert_array_equal(host(routed).reshape(T, k, 2)[:, :, 0].astype(np.uint32), wids)
        np.testing.assert_array_equal(bits(host(out).reshape(T, H)), bits(want))
    layer.close()
