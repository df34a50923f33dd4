"""GPU parity of a chained stack of config-3 MoE blocks (BASELINE config 5 at
reduced depth): hidden += MoE(RMSNorm(hidden)) per layer, each block's output
fed to the next, against the same chain on the CPU oracle
(weighted_rms_norm_into -> route_experts_into -> moe_routed_by_id_into ->
residual_add_in_place: bridge-kernels-reference/src/norm.rs:5-18, :83-100;
bridge-model-hy3/src/routing.rs:25-107; moe.rs:64-147), mirroring the layer
loop of bridge-runtime/src/hy3_scalar.rs:504-650 with attention omitted.

Two chains. In the benched mode (tree-order F32 sums in the RMSNorm and the
router logits, each within rounding of the reference's sequential chain) every
layer is checked on the stack's own trajectory: the device's normalized input
(the block workspace's first region) against the oracle's RMSNorm of the same
hidden state, then the oracle's MoE step on that normalized input plus the
residual against the device's output. A last-bit difference in a normalized
input can move a Q8_K rounding by one step, which no f32 bar can hold, so the
MoE step is compared on the input it actually saw. With sequential order the
arithmetic is the reference's own, so the two chains run independently over
the whole depth (the oracle's hidden state never takes the device's values).
Layers are generated on the device (seeded torch generator, seed 4 + layer as
in config 5), repacked to the planar layout there, and their GGUF bytes copied
to the host for the oracle. Bars per layer and token: top-8 IDs identical,
hidden state within 1e-5 element-wise relative (tests/gpu_helpers.rel_err).
"""

import numpy as np
import pytest
import torch

import lbk
import oracle as orc
import synth
from gpu_helpers import clean_status, ctx, errs, host, moe_term_magnitude, rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-5
H, F, E, K = 4096, 1536, 192, 8
WEIGHT_SCALE = 2.826
EPS = 1e-6


def device_layer(seed: int):
    """One config-3 layer from a seeded device generator: the lbk layer
    (planar weights) plus the oracle's expert table over host GGUF copies."""
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    keep = []
    router = (torch.randn(E, H, device=dev, generator=gen) * 0.02).contiguous()
    keep.append(router)

    def stacked(ty, k, rows, n):
        g = synth.packed_torch(gen, ty, k, rows * n, dev)
        mb, pb = synth.matrix_bytes(ty, k, rows), synth.planar_bytes(ty, k, rows)
        p = torch.empty(pb * n, dtype=torch.uint8, device=dev)
        for e in range(n):
            ctx().repack(lbk.matrix(ty, k, rows, g[e * mb:(e + 1) * mb]), p[e * pb:(e + 1) * pb])
        keep.append(p)
        return g.cpu().numpy(), p, mb, pb

    gh, gp, mbg, pbg = stacked(orc.TYPE_IQ2_S, H, F, E)
    uh, up, _, _ = stacked(orc.TYPE_IQ2_S, H, F, E)
    dh, dp, mbd, pbd = stacked(orc.TYPE_IQ3_S, F, H, E)
    sg, sgp, _, _ = stacked(orc.TYPE_Q4_K, H, F, 1)
    su, sup, _, _ = stacked(orc.TYPE_Q4_K, H, F, 1)
    sd, sdp, _, _ = stacked(orc.TYPE_Q4_K, F, H, 1)
    norm_w = (torch.rand(H, device=dev, generator=gen) * 2.0).contiguous()
    keep.append(norm_w)
    bias = torch.zeros(E, device=dev)
    keep.append(bias)
    torch.cuda.synchronize()
    experts = [
        lbk.Expert(lbk.matrix(orc.TYPE_IQ2_S, H, F, gp[e * pbg:(e + 1) * pbg], lbk.LAYOUT_PLANAR),
                   lbk.matrix(orc.TYPE_IQ2_S, H, F, up[e * pbg:(e + 1) * pbg], lbk.LAYOUT_PLANAR),
                   lbk.matrix(orc.TYPE_IQ3_S, F, H, dp[e * pbd:(e + 1) * pbd], lbk.LAYOUT_PLANAR))
        for e in range(E)
    ]
    shared = lbk.Expert(lbk.matrix(orc.TYPE_Q4_K, H, F, sgp, lbk.LAYOUT_PLANAR),
                        lbk.matrix(orc.TYPE_Q4_K, H, F, sup, lbk.LAYOUT_PLANAR),
                        lbk.matrix(orc.TYPE_Q4_K, F, H, sdp, lbk.LAYOUT_PLANAR))
    rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, H, E, router.data_ptr(), router.numel() * 4)
    layer = lbk.MoeLayer(ctx(), experts, shared, rm, bias, K, WEIGHT_SCALE)
    assert layer.fused
    host_experts = [(orc.TYPE_IQ2_S, gh[e * mbg:(e + 1) * mbg], orc.TYPE_IQ2_S, uh[e * mbg:(e + 1) * mbg],
                     orc.TYPE_IQ3_S, dh[e * mbd:(e + 1) * mbd], H, F) for e in range(E)]
    host_shared = (orc.TYPE_Q4_K, sg, orc.TYPE_Q4_K, su, orc.TYPE_Q4_K, sd, H, F)
    host_router = router.cpu().numpy()
    table = orc.ExpertTable(host_experts, host_shared, router=host_router, hidden=H)
    return layer, table, norm_w, norm_w.cpu().numpy(), keep, (gh, uh, dh, sg, su, sd, host_router)


@pytest.fixture(scope="module")
def stack():
    layers = [device_layer(4 + l) for l in range(3)]
    yield layers
    for layer, *_ in layers:
        layer.close()


@pytest.mark.parametrize("mode", [lbk.ROUTER_TREE, lbk.ROUTER_SEQUENTIAL])
@pytest.mark.parametrize("batch", [1, 4])
def test_chained_stack_matches_oracle(stack, batch, mode):
    rng = np.random.default_rng(300 + batch)
    hidden0 = rng.standard_normal((batch, H)).astype(np.float32)
    hd = torch.from_numpy(hidden0.reshape(-1).copy()).cuda()
    want = hidden0.copy()
    ws = torch.zeros(stack[0][0].block_workspace_bytes(batch), dtype=torch.uint8, device="cuda")
    zero_bias = np.zeros(E, np.float32)
    for li, (layer, table, norm_w, norm_host, _, _) in enumerate(stack):
        before = host(hd).reshape(batch, H)
        routed = torch.zeros(batch * K * 2, dtype=torch.int32, device="cuda")
        layer.block_forward(hd, norm_w, EPS, batch, ws, routed_out=routed, router_mode=mode)
        clean_status()
        got = host(hd).reshape(batch, H)
        ids = host(routed).reshape(batch, K, 2)[:, :, 0].astype(np.uint32)
        mag = None
        if mode == lbk.ROUTER_TREE:
            want = before.copy()
            xn_dev = host(ws[:batch * H * 4].view(torch.float32)).reshape(batch, H)
            mag = np.abs(before).astype(np.float64)
        for t in range(batch):
            xn = orc.rms_norm(want[t], norm_host, EPS)
            if mode == lbk.ROUTER_TREE:
                assert rel_err(xn_dev[t], xn) <= TOL, f"layer {li} token {t} norm: " + errs(xn_dev[t], xn)
                xn = xn_dev[t]
            delta, wids, wc = orc.moe_token(table, zero_bias, K, WEIGHT_SCALE, xn)
            np.testing.assert_array_equal(ids[t], wids, err_msg=f"layer {li} token {t}")
            if mag is not None:
                mag[t] += moe_term_magnitude(table, wids, wc, xn)
            assert orc.residual_add_status(want[t], delta) == 0
        assert rel_err(got, want, mag) <= TOL, f"layer {li}: " + errs(got, want, mag)
        differ = int(np.count_nonzero(got.view(np.uint32) != want.view(np.uint32)))
        print(f"batch {batch} mode {mode} layer {li}: {errs(got, want, mag)}, {differ} of {got.size} values differ in bits")
