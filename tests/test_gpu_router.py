"""GPU parity: router logits and Hy3 top-k routing
(bridge-model-hy3/src/routing.rs:25-107, tests/routing.rs:46-235)."""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
from gpu_helpers import bits, clean_status, ctx, dev, expect_status, host

pytestmark = pytest.mark.gpu


def routed_np(t: torch.Tensor, tokens: int, k: int):
    a = host(t.view(torch.int32)).reshape(tokens, k, 2)
    return a[:, :, 0].astype(np.uint32), a[:, :, 1].view(np.float32)


def topk(logits: np.ndarray, bias: np.ndarray, k: int, ws: float):
    T, E = logits.shape
    out = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    ctx().route_topk(dev(logits.reshape(-1)), dev(bias), E, T, k, ws, out)
    clean_status()
    return routed_np(out, T, k)


def test_topk_matches_oracle_on_router_logits():
    rng = np.random.default_rng(2)
    E, H, k = 192, 4096, 8
    w = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    xs = rng.standard_normal((16, H)).astype(np.float32)
    logits = np.stack([orc.gemv_f32(H, E, w, x) for x in xs])
    bias = np.zeros(E, np.float32)
    ids, coefs = topk(logits, bias, k, 2.826)
    for t in range(16):
        wid, wco = orc.route_experts(logits[t], bias, k, 2.826)
        np.testing.assert_array_equal(ids[t], wid)
        np.testing.assert_allclose(coefs[t], wco, rtol=1e-6)


def test_sequential_router_logits_bit_exact_multi_token():
    rng = np.random.default_rng(4)
    E, H, T = 192, 4096, 3
    w = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    xs = rng.standard_normal((T, H)).astype(np.float32)
    wd = dev(w.reshape(-1))
    m = lbk.Matrix(lbk.TYPE_F32, 0, H, E, wd.data_ptr(), wd.numel() * 4)
    logits = torch.zeros(T * E, device="cuda")
    ctx().router_logits(m, dev(xs.reshape(-1)), T, logits, lbk.ROUTER_SEQUENTIAL)
    clean_status()
    got = host(logits).reshape(T, E)
    for t in range(T):
        np.testing.assert_array_equal(bits(got[t]), bits(orc.gemv_f32(H, E, w, xs[t])))


def test_ties_bias_sorting_and_floor():
    ids, coefs = topk(np.zeros((1, 4), np.float32), np.zeros(4, np.float32), 3, 2.826)
    assert list(ids[0]) == [0, 1, 2]
    assert np.allclose(coefs[0], 2.826 / 3, atol=1e-6)
    ids, coefs = topk(np.array([[3, 1, -1, -3]], np.float32), np.array([0, 0, 2, 4], np.float32), 2, 2.0)
    assert list(ids[0]) == [2, 3]
    wid, wco = orc.route_experts(np.array([3, 1, -1, -3], np.float32), np.array([0, 0, 2, 4], np.float32), 2, 2.0)
    np.testing.assert_allclose(coefs[0], wco, rtol=1e-6)
    ids, _ = topk(np.array([[0, 4, -4, 2]], np.float32), np.zeros(4, np.float32), 3, 1.0)
    assert list(ids[0]) == [0, 1, 3]
    fmin = np.finfo(np.float32).min
    ids, coefs = topk(np.array([[fmin, fmin]], np.float32), np.zeros(2, np.float32), 2, 2.826)
    assert (coefs == 0).all()


def test_non_finite_logit_rejected():
    logits = np.zeros((1, 8), np.float32)
    logits[0, 5] = np.nan
    logits[0, 6] = np.inf
    out = torch.full((8,), 77, dtype=torch.int32, device="cuda")
    ctx().route_topk(dev(logits.reshape(-1)), dev(np.zeros(8, np.float32)), 8, 1, 4, 1.0, out)
    d = expect_status(18)
    assert d.index == 5
    assert (host(out) == 77).all()
