"""GPU: a MoE layer read from a Hy3 GGUF set by lbk_moe_layer_load computes
exactly what the same tensors give when registered through
lbk_moe_layer_create (bit for bit, routing included), and matches the CPU
oracle of the reference's MoE step (moe_token: route_experts_into +
moe_routed_by_id_into, bridge-kernels-reference/src/moe.rs:116-147) within
1e-5 relative. Expert-parallel shares loaded from the file combine to the
full layer's result exactly. The layer owns and frees its device memory.
"""

import numpy as np
import pytest
import torch

import ep
import lbk
import oracle as orc
from gguf_fixture import Hy3Block, write_hy3
from gpu_helpers import clean_status, ctx, dev, errs, moe_term_magnitude, rel_err, upload_layer

pytestmark = pytest.mark.gpu

IQ2, IQ3 = lbk.TYPE_IQ2_S, lbk.TYPE_IQ3_S
SCALE = float(np.float32(2.826))


def checkpoint_block(rng, H, F, E, layer):
    """Types of the Hy3 checkpoint schema (schema.rs:219-258): routed and
    shared gate/up IQ2_S; routed down IQ3_S through layer 5, shared down IQ3_S
    through layer 4, IQ2_S after."""
    return Hy3Block(rng, H, F, E, IQ2, IQ2, IQ3 if layer <= 5 else IQ2, IQ2, IQ2, IQ3 if layer <= 4 else IQ2)


def host_tables(b: Hy3Block, H, F):
    gty, uty, dty, sgty, suty, sdty = b.types
    experts = [(gty, g, uty, u, dty, d, H, F) for g, u, d in b.experts]
    shared = (sgty, b.shared[0], suty, b.shared[1], sdty, b.shared[2], H, F)
    return experts, shared


def forward(layer, x, T):
    H, k = layer.hidden, layer.top_k
    ws = torch.zeros(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.full((T * H,), float("nan"), device="cuda")
    routed = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    layer.forward(x, T, out, ws, routed_out=routed)
    clean_status()
    return out, routed


def same(a, b):
    return torch.equal(a.view(torch.int32).cpu(), b.view(torch.int32).cpu())


@pytest.mark.parametrize("H,F,E,k,T,layer_no", [(2048, 512, 16, 4, 3, 3), (4096, 1536, 24, 8, 2, 7),
                                                  (4096, 1536, 24, 8, 1, 5)])
def test_loaded_layer_equals_registered_layer_and_oracle(tmp_path, H, F, E, k, T, layer_no):
    rng = np.random.default_rng(H + E + layer_no)
    b = checkpoint_block(rng, H, F, E, layer_no)
    entry = write_hy3(tmp_path, H, F, E, k, {layer_no: b})
    with lbk.Gguf(entry) as g:
        loaded = lbk.load_layer(ctx(), g, layer_no)
    assert loaded.fused and isinstance(loaded, lbk.MoeLayer) and not isinstance(loaded, lbk.EpLayer)
    experts, shared = host_tables(b, H, F)
    ref, keep = upload_layer(b.router, experts, shared, lbk.LAYOUT_PLANAR, k, SCALE, bias=b.bias)
    x = (rng.standard_normal((T, H)) * 2).astype(np.float32)
    xd = dev(x.reshape(-1))
    out, routed = forward(loaded, xd, T)
    want, wr = forward(ref, xd, T)
    assert torch.equal(routed.cpu(), wr.cpu())
    assert same(out, want)
    table = orc.ExpertTable(experts, shared, router=b.router, hidden=H)
    got = out.cpu().numpy().reshape(T, H)
    ids = routed.cpu().numpy().reshape(T, k, 2)[:, :, 0].astype(np.uint32)
    for t in range(T):
        o, oid, oc = orc.moe_token(table, b.bias, k, SCALE, x[t])
        np.testing.assert_array_equal(ids[t], oid)
        mag = moe_term_magnitude(table, oid, oc, x[t])
        assert rel_err(got[t], o, mag) <= 1e-5, errs(got[t], o, mag)
    loaded.close()
    ref.close()


def test_blocks_of_a_split_set(tmp_path):
    H, F, E, k, T = 2048, 512, 16, 4, 2
    rng = np.random.default_rng(11)
    blocks = {n: checkpoint_block(rng, H, F, E, n) for n in (4, 5, 6)}
    entry = write_hy3(tmp_path, H, F, E, k, blocks, block_count=8, shards=3)
    x = dev(rng.standard_normal(T * H).astype(np.float32))
    with lbk.Gguf(entry) as g:
        assert g.info().shard_count == 3
        for n, b in blocks.items():
            loaded = lbk.load_layer(ctx(), g, n)
            experts, shared = host_tables(b, H, F)
            ref, keep = upload_layer(b.router, experts, shared, lbk.LAYOUT_PLANAR, k, SCALE, bias=b.bias)
            out, routed = forward(loaded, x, T)
            want, wr = forward(ref, x, T)
            assert torch.equal(routed.cpu(), wr.cpu()) and same(out, want), n
            loaded.close()
            ref.close()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_shares_loaded_from_the_file(tmp_path, world):
    """Each rank loads only its experts; routing on rank 0, the exchange done
    by slicing (as on one GPU), combine: equal to the full layer bit for bit."""
    H, F, E, k, T = 2048, 512, 16, 4, 5
    rng = np.random.default_rng(world)
    entry = write_hy3(tmp_path, H, F, E, k, {0: checkpoint_block(rng, H, F, E, 0)})
    er = E // world
    with lbk.Gguf(entry) as g:
        full = lbk.load_layer(ctx(), g, 0)
        ranks = [lbk.load_layer(ctx(), g, 0, r * er, er) for r in range(world)]
    assert all(isinstance(r, lbk.EpLayer) and r.local_experts == er and r.global_experts == E for r in ranks)
    home = ranks[0]
    x = dev(rng.standard_normal(T * H).astype(np.float32))
    q8b = home.q8_bytes
    ws = torch.zeros(max(home.workspace_bytes(T), home.workspace_bytes(T * k)), dtype=torch.uint8, device="cuda")
    routed = torch.empty((T * k, 2), dtype=torch.int32, device="cuda")
    q8 = torch.empty((T, q8b), dtype=torch.uint8, device="cuda")
    home.route(x, T, routed, q8, ws)
    ids = routed[:, 0]
    plan = ep.local_plan(ids, er, world)
    rows = ep.pack_rows(q8, ids, plan, k, er)
    dots = []
    for r, chunk in enumerate(torch.split(rows, plan.send)):
        n = chunk.shape[0]
        d = torch.empty((n, H), dtype=torch.float32, device="cuda")
        if n:
            imgs, items = ep.unpack_items(chunk, q8b)
            ranks[r].items_forward(imgs, items, n, d, ws)
        dots.append(d)
    routed_dots = ep.place_returned(torch.cat(dots), plan, T * k, H)
    out = torch.full((T * H,), float("nan"), device="cuda")
    home.combine(q8, T, routed, routed_dots, out, ws)
    clean_status()
    want, wr = forward(full, x, T)
    assert torch.equal(routed.view(-1).cpu(), wr.cpu()) and same(out, want)
    full.close()
    for r in ranks:
        r.close()


def test_layer_frees_its_device_memory(tmp_path):
    H, F, E, k = 4096, 1536, 24, 8
    rng = np.random.default_rng(5)
    entry = write_hy3(tmp_path, H, F, E, k, {0: checkpoint_block(rng, H, F, E, 0)})
    torch.cuda.synchronize()
    with lbk.Gguf(entry) as g:
        layer = lbk.load_layer(ctx(), g, 0)
        free_loaded = torch.cuda.mem_get_info()[0]
        layer.close()
        free_after = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            lbk.load_layer(ctx(), g, 0).close()
        free_end = torch.cuda.mem_get_info()[0]
    layer_bytes = E * (2 * H * F // 256 * 82 + F * H // 256 * 110)
    assert free_after - free_loaded >= layer_bytes  # the experts' planar copies were released
    assert abs(free_end - free_after) < 64 << 20
