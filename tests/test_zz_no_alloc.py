"""lbk_moe_forward_no_alloc: the MoE forward with its workspace in the
library's fixed device array instead of caller memory.

Checked through the C ABI against lbk_moe_forward (caller workspace) on the
same layer and inputs, bit for bit (the same kernels on the same inputs; only
the workspace address differs), for two calls in a row (the second call starts from the
counters the first one left behind), on both the fused and the per-expert
path, and its rejection of a workspace larger than the array. Named to be
collected last, so that it also runs after every other GPU test in one
process; it passes alone as well.
"""

import numpy as np
import pytest
import torch

import lbk
from gpu_helpers import bits, clean_status, dev, host, make_layer_np, upload_layer

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_BYTES = 1 << 20


def forward_workspace(layer, x, T, mode):
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.full((T * layer.hidden,), float("nan"), device="cuda")
    routed = torch.zeros(T * layer.top_k * 2, dtype=torch.int32, device="cuda")
    st = lbk.lib.lbk_moe_forward(layer.ptr, x.data_ptr(), T, out.data_ptr(), routed.data_ptr(), mode,
                                 ws.data_ptr(), ws.numel(), None)
    assert st == 0, (st, lbk.STATUS.get(st))
    clean_status()
    return host(out), host(routed)


def forward_no_alloc(layer, x, T, mode):
    out = torch.full((T * layer.hidden,), float("nan"), device="cuda")
    routed = torch.zeros(T * layer.top_k * 2, dtype=torch.int32, device="cuda")
    st = lbk.lib.lbk_moe_forward_no_alloc(layer.ptr, x.data_ptr(), T, out.data_ptr(), routed.data_ptr(), mode, None)
    assert st == 0, (st, lbk.STATUS.get(st))
    clean_status()
    return host(out), host(routed)


@pytest.mark.parametrize("layout", [lbk.LAYOUT_PLANAR, lbk.LAYOUT_GGUF])
@pytest.mark.parametrize("T", [1, 3])
def test_no_alloc_matches_workspace_forward_twice(layout, T):
    rng = np.random.default_rng(2024 + T)
    H, F, E, k = 1024, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, layout, k)
    assert layer.workspace_bytes(T) <= STATIC_SCRATCH_BYTES
    x = dev(rng.standard_normal(T * H).astype(np.float32))
    for mode in (lbk.ROUTER_TREE, lbk.ROUTER_SEQUENTIAL):
        want, want_routed = forward_workspace(layer, x, T, mode)
        for _ in range(2):  # two calls in a row on the same array
            got, got_routed = forward_no_alloc(layer, x, T, mode)
            np.testing.assert_array_equal(got_routed, want_routed)
            assert np.all(np.isfinite(got))
            np.testing.assert_array_equal(bits(got), bits(want))
    layer.close()
    del keep


def test_no_alloc_rejects_workspace_beyond_the_array():
    rng = np.random.default_rng(9)
    H, F, E, k = 1024, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    T = 1
    while layer.workspace_bytes(T) <= STATIC_SCRATCH_BYTES:
        T *= 2
    need = layer.workspace_bytes(T)
    x = torch.zeros(T * H, device="cuda")
    out = torch.zeros(T * H, device="cuda")
    st = lbk.lib.lbk_moe_forward_no_alloc(layer.ptr, x.data_ptr(), T, out.data_ptr(), None, lbk.ROUTER_TREE, None)
    assert st == 11, lbk.STATUS.get(st)  # SCRATCH_TOO_SMALL
    d = lbk.last_error()
    assert d.expected == need and d.actual == STATIC_SCRATCH_BYTES
    assert b"static MoE scratch" in d.message
    # the rejected call launched nothing: the array still serves a fitting call
    clean_status()
    xs = dev(rng.standard_normal(H).astype(np.float32))
    want, _ = forward_workspace(layer, xs, 1, lbk.ROUTER_TREE)
    got, _ = forward_no_alloc(layer, xs, 1, lbk.ROUTER_TREE)
    np.testing.assert_array_equal(bits(got), bits(want))
    layer.close()
    del keep


def test_no_alloc_checks_arguments_first():
    """Bad arguments are refused before the call touches the device (the
    first call's set-up included)."""
    rng = np.random.default_rng(10)
    H, F, E, k = 1024, 512, 16, 4
    router, experts, shared = make_layer_np(rng, H, F, E)
    layer, keep = upload_layer(router, experts, shared, lbk.LAYOUT_PLANAR, k)
    x = torch.zeros(H, device="cuda")
    out = torch.zeros(H, device="cuda")
    assert lbk.lib.lbk_moe_forward_no_alloc(layer.ptr, x.data_ptr(), 1, out.data_ptr(), None, 7, None) == 15
    assert lbk.lib.lbk_moe_forward_no_alloc(layer.ptr, None, 1, out.data_ptr(), None, lbk.ROUTER_TREE, None) == 15
    assert lbk.lib.lbk_moe_forward_no_alloc(layer.ptr, x.data_ptr() + 4, 1, out.data_ptr(), None, lbk.ROUTER_TREE,
                                            None) == 15
    layer.close()
    del keep
