"""GPU parity of the MoE block's RMSNorm and residual add (lbk_rms_norm,
lbk_residual_add) and of the whole FFN block (lbk_moe_block_forward) against
the CPU oracle: weighted_rms_norm_into and residual_add_in_place
(bridge-kernels-reference/src/norm.rs:5-18, :83-100) around the MoE step of
hy3_moe_route_token / hy3_moe_finish_token (layer.rs:588-659).

Bars: the sequential-order norm bit-identical to the reference's f32 chain,
the tree order within 1e-5 relative; the residual add exact; the block output
within 1e-5 relative (its SwiGLU and sigmoid call exp) with identical routing.
Every error leaves its output untouched (tests/norm.rs:48-81).
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
from gpu_helpers import (bits, clean_status, ctx, dev, errs, expect_status, host, make_layer_np, moe_term_magnitude,
                         rel_err, upload_layer)

pytestmark = pytest.mark.gpu

TOL = 1e-5


def norm_dev(x, w, eps, mode, out_init=np.nan):
    rows, n = x.shape
    out = torch.full((rows * n,), float(out_init), device="cuda")
    ctx().rms_norm(dev(x.reshape(-1)), dev(w), n, rows, eps, out, mode)
    return out


@pytest.mark.parametrize("n", [4096, 2048, 1536, 100, 7])
def test_rms_norm_matches_oracle(n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((3, n)) * 1.7).astype(np.float32)
    w = (rng.random(n) * 2 - 0.5).astype(np.float32)
    eps = 1e-6
    want = np.stack([orc.rms_norm(r, w, eps) for r in x])
    seq = host(norm_dev(x, w, eps, lbk.ROUTER_SEQUENTIAL)).reshape(3, n)
    clean_status()
    np.testing.assert_array_equal(bits(seq), bits(want))
    tree = host(norm_dev(x, w, eps, lbk.ROUTER_TREE)).reshape(3, n)
    clean_status()
    assert rel_err(tree, want) <= TOL


def test_rms_norm_reference_vector():
    # tests/norm.rs:11-26
    out = host(norm_dev(np.array([[3.0, 4.0]], np.float32), np.array([1.0, 2.0], np.float32), 1e-5,
                        lbk.ROUTER_SEQUENTIAL))
    clean_status()
    np.testing.assert_array_equal(bits(out), bits(orc.rms_norm(np.array([3.0, 4.0], np.float32),
                                                                np.array([1.0, 2.0], np.float32), 1e-5)))


def test_rms_norm_validation_is_atomic():
    sentinel = np.array([0x7FC000A5, 0x80000000], np.uint32).view(np.float32)
    for mode in (lbk.ROUTER_SEQUENTIAL, lbk.ROUTER_TREE):
        out = dev(sentinel.copy())
        ctx().rms_norm(dev(np.array([1.0, np.nan], np.float32)), dev(np.ones(2, np.float32)), 2, 1, 1e-5, out, mode)
        assert expect_status(12).index == 1  # NonFiniteValue, RMSNorm input index 1
        np.testing.assert_array_equal(bits(host(out)), bits(sentinel))
        mx = np.finfo(np.float32).max
        ctx().rms_norm(dev(np.array([1.0, 0.0], np.float32)), dev(np.array([mx, mx], np.float32)), 2, 1, 1e-5, out,
                       mode)
        expect_status(12)  # the output overflows
        np.testing.assert_array_equal(bits(host(out)), bits(sentinel))
    for n, eps, code in [(0, 1e-5, 15), (2, 0.0, 15), (2, float("inf"), 12)]:
        with pytest.raises(lbk.LbkError) as e:
            ctx().rms_norm(dev(np.ones(2, np.float32)), dev(np.ones(2, np.float32)), n, 1, eps,
                           torch.zeros(2, device="cuda"))
        assert e.value.status == code


def test_residual_add_exact_and_atomic():
    # tests/norm.rs:41-46 and :75-80
    d = dev(np.array([1.0, -2.0, 3.5], np.float32))
    ctx().residual_add(d, dev(np.array([2.0, 1.0, -0.5], np.float32)), 3)
    clean_status()
    np.testing.assert_array_equal(host(d), np.array([3.0, -1.0, 3.0], np.float32))
    mx = np.finfo(np.float32).max
    r = dev(np.array([mx, 1.0], np.float32))
    ctx().residual_add(r, dev(np.array([mx, 2.0], np.float32)), 2)
    expect_status(12)
    np.testing.assert_array_equal(bits(host(r)), bits(np.array([mx, 1.0], np.float32)))
    # the reference checks all of dest, then all of src: a non-finite dest
    # value is reported before an earlier non-finite src value
    rng = np.random.default_rng(3)
    a = rng.standard_normal(10000).astype(np.float32)
    b = rng.standard_normal(10000).astype(np.float32)
    a[7001] = np.inf
    b[5] = np.nan
    want = a.copy()
    assert orc.residual_add_status(want, b) == 12
    ref_index = orc.last_detail().index
    ad = dev(a)
    ctx().residual_add(ad, dev(b), a.size)
    assert expect_status(12).index == ref_index == 7001
    np.testing.assert_array_equal(bits(host(ad)), bits(a))


@pytest.mark.parametrize("mode", [lbk.ROUTER_SEQUENTIAL, lbk.ROUTER_TREE])
@pytest.mark.parametrize("H,F,E,k,T", [(4096, 1536, 24, 8, 1), (2048, 512, 16, 4, 3)])
def test_block_forward_matches_oracle(mode, H, F, E, k, T):
    rng = np.random.default_rng(H + F + E + k + T + mode)
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    hidden = (rng.standard_normal((T, H)) * 3).astype(np.float32)
    norm_w = (rng.random(H) * 2).astype(np.float32)
    eps = 1e-6
    table = orc.ExpertTable(experts, shared, router=router, hidden=H)
    want = hidden.copy()
    want_ids = []
    mag = np.abs(hidden).astype(np.float64)
    for t in range(T):
        xn = orc.rms_norm(hidden[t], norm_w, eps)
        delta, ids, coefs = orc.moe_token(table, np.zeros(E, np.float32), k, 2.826, xn)
        want_ids.append(ids)
        mag[t] += moe_term_magnitude(table, ids, coefs, xn)
        assert orc.residual_add_status(want[t], delta) == 0
    hd = dev(hidden.reshape(-1))
    ws = torch.zeros(layer.block_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    routed = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    layer.block_forward(hd, dev(norm_w), eps, T, ws, routed_out=routed, router_mode=mode)
    clean_status()
    got = host(hd).reshape(T, H)
    ids = host(routed).reshape(T, k, 2)[:, :, 0].astype(np.uint32)
    np.testing.assert_array_equal(ids, np.stack(want_ids))
    assert rel_err(got, want, mag) <= TOL, errs(got, want, mag)
    layer.close()


def test_block_forward_leaves_hidden_untouched_on_error():
    rng = np.random.default_rng(9)
    H, F, E, k = 2048, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    hidden = rng.standard_normal((2, H)).astype(np.float32)
    hidden[1, 17] = np.nan  # the second token's norm input
    hd = dev(hidden.reshape(-1))
    ws = torch.zeros(layer.block_workspace_bytes(2), dtype=torch.uint8, device="cuda")
    layer.block_forward(hd, dev(np.ones(H, np.float32)), 1e-6, 2, ws)
    assert expect_status(12).index == 17
    np.testing.assert_array_equal(bits(host(hd)), bits(hidden.reshape(-1)))
    layer.close()


@pytest.mark.parametrize("mode", [lbk.ROUTER_SEQUENTIAL, lbk.ROUTER_TREE])
@pytest.mark.parametrize("H,F,E,k,T", [(2048, 512, 16, 4, 1), (2048, 512, 16, 4, 3)])
def test_route_then_finish_equals_block_forward(mode, H, F, E, k, T):
    """hy3_moe_route_token then hy3_moe_finish_token with the routing the
    route phase returned: bit for bit the one-call block."""
    rng = np.random.default_rng(H + E + T + 7 * mode)
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    hidden = (rng.standard_normal((T, H)) * 2).astype(np.float32)
    norm_w = (rng.random(H) * 2).astype(np.float32)
    nw = dev(norm_w)
    ws = torch.zeros(layer.block_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    one = dev(hidden.reshape(-1))
    r1 = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    layer.block_forward(one, nw, 1e-6, T, ws, routed_out=r1, router_mode=mode)
    clean_status()
    two = dev(hidden.reshape(-1))
    ws2 = torch.zeros(layer.block_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    r2 = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    layer.block_route(two, nw, 1e-6, T, ws2, routed_out=r2, router_mode=mode)
    clean_status()
    np.testing.assert_array_equal(host(r2), host(r1))
    np.testing.assert_array_equal(bits(host(two)), bits(hidden.reshape(-1)))  # route leaves hidden alone
    layer.block_finish(two, T, r2, ws2)
    clean_status()
    np.testing.assert_array_equal(bits(host(two)), bits(host(one)))
    layer.close()


def test_finish_refuses_routing_that_differs_in_one_bit():
    """layer.rs:631-640: supplied IDs and coefficient bits must equal the
    route phase's routing; otherwise InvalidParameter and hidden untouched."""
    rng = np.random.default_rng(41)
    H, F, E, k, T = 2048, 512, 16, 4, 2
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    hidden = rng.standard_normal((T, H)).astype(np.float32)
    nw = dev(np.ones(H, np.float32))
    ws = torch.zeros(layer.block_workspace_bytes(T), dtype=torch.uint8, device="cuda")
    hd = dev(hidden.reshape(-1))
    r = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    # a finish without a route, and two routes in a row: host errors before any launch
    with pytest.raises(lbk.LbkError) as e:
        layer.block_finish(hd, T, r, ws)
    assert e.value.status == 15
    layer.block_route(hd, nw, 1e-6, T, ws, routed_out=r)
    with pytest.raises(lbk.LbkError) as e:
        layer.block_route(hd, nw, 1e-6, T, ws, routed_out=r)
    assert e.value.status == 15
    with pytest.raises(lbk.LbkError) as e:
        layer.block_finish(hd, T - 1, r, ws)
    assert e.value.status == 10
    clean_status()
    routed = host(r).copy()
    bad = routed.copy()
    bad[2 * (k + 1) + 1] ^= 1  # token 1, slot 1: coefficient's last bit
    layer.block_finish(hd, T, dev(bad), ws)
    d = expect_status(15)
    assert d.index == k + 1
    np.testing.assert_array_equal(bits(host(hd)), bits(hidden.reshape(-1)))
    # the phase ended with that finish: route again, then the matching finish
    layer.block_route(hd, nw, 1e-6, T, ws, routed_out=r)
    clean_status()
    bad = host(r).copy()
    bad[0] = (bad[0] + 1) % E  # token 0, slot 0: another expert ID
    layer.block_finish(hd, T, dev(bad), ws)
    expect_status(15)
    np.testing.assert_array_equal(bits(host(hd)), bits(hidden.reshape(-1)))
    layer.close()
