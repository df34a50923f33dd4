"""Expert parallelism: the dispatch / return plumbing of ep.ExpertParallelMoe
(host logic on gloo ranks, world size 2) and, on a GPU, lbk_ep_* against
lbk_moe_forward bit for bit -- one rank, two ranks simulated on one GPU, and
real nccl ranks when the box has two GPUs.

The reference runs every expert of a layer on one host
(bridge-runtime/src/hy3_scalar.rs:561-628); the expert-parallel result must
equal that single-host combine (bridge-kernels-reference/src/moe.rs:116-147)
exactly, so every GPU check here is bit-exact, not a tolerance.
"""

import os
import pathlib
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

import ep

REPO = pathlib.Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(nproc: int, mode: str, timeout: int) -> subprocess.CompletedProcess:
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(REPO / "tests" / "ep_worker.py"),
           "--mode", mode]
    env = dict(os.environ, OMP_NUM_THREADS="1", NCCL_NVLS_ENABLE="0")
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)


# ----------------------------------------------------------------- host logic


def test_plan_orders_pairs_by_owner_stably():
    ids = torch.tensor([5, 1, 7, 0, 2, 6, 3, 4], dtype=torch.int32)
    plan = ep.local_plan(ids, experts_per_rank=2, world=4)
    assert plan.send == [2, 2, 2, 2] and plan.recv == plan.send
    assert plan.order.tolist() == [1, 3, 4, 6, 0, 7, 2, 5]
    assert plan.owner.tolist() == [2, 0, 3, 0, 1, 3, 1, 2]


def test_plan_rejects_expert_beyond_the_ranks():
    with pytest.raises(ValueError):
        ep.local_plan(torch.tensor([0, 9], dtype=torch.int32), experts_per_rank=2, world=4)


def test_rows_round_trip_and_returned_dots_land_in_pair_order():
    k, q8b, H = 3, 32, 5
    q8 = torch.arange(4 * q8b, dtype=torch.int64).remainder(251).to(torch.uint8).view(4, q8b)
    ids = torch.tensor([0, 3, 5, 1, 2, 4, 0, 1, 5, 2, 3, 4], dtype=torch.int32)  # 4 tokens x 3
    plan = ep.local_plan(ids, experts_per_rank=2, world=3)
    rows = ep.pack_rows(q8, ids, plan, k, 2)
    assert rows.shape == (12, q8b + ep.ROW_HEADER_BYTES) and (q8b + ep.ROW_HEADER_BYTES) % 16 == 0
    imgs, items = ep.unpack_items(rows, q8b)
    for i, p in enumerate(plan.order.tolist()):
        assert torch.equal(imgs[i], q8[p // k])
        assert items[i, 0].item() == ids[p].item() % 2 and items[i, 1].item() == 0
    back = torch.arange(12 * H, dtype=torch.float32).view(12, H)
    got = ep.place_returned(back, plan, 12, H)
    for i, p in enumerate(plan.order.tolist()):
        assert torch.equal(got[p], back[i])


def test_empty_dispatch():
    plan = ep.local_plan(torch.zeros(0, dtype=torch.int32), experts_per_rank=4, world=2)
    assert plan.send == [0, 0]
    rows = ep.pack_rows(torch.zeros((0, 32), dtype=torch.uint8), torch.zeros(0, dtype=torch.int32), plan, 8, 4)
    imgs, items = ep.unpack_items(rows, 32)
    assert imgs.shape == (0, 32) and items.shape == (0, 2)
    assert ep.place_returned(torch.zeros((0, 7)), plan, 0, 7).shape == (0, 7)


def test_layer_must_hold_its_rank_share():
    class L:
        global_experts, local_experts, first_expert = 8, 4, 0

    with pytest.raises(ValueError):
        ep.ExpertParallelMoe(L())  # one rank must hold all 8


def test_gloo_two_ranks_match_one_rank_bit_for_bit():
    """Two gloo ranks on the host with exact stand-in compute stages:
    ragged token counts, a rank without tokens, pairs all on one rank."""
    r = _torchrun(2, "cpu", timeout=240)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ok" in r.stdout


# ------------------------------------------------------------------------ GPU


def _gpu_layers(H, F, E, k, seed, world):
    import lbk
    from gpu_helpers import ctx, dev, make_layer_np, matrix, planar_dev

    rng = np.random.default_rng(seed)
    router, experts, shared = make_layer_np(rng, H, F, E)
    keep = []

    def up(ty, b, in_w):
        t = planar_dev(ty, b, in_w)
        keep.append(t)
        return t

    def ex(e):
        gty, gb, uty, ub, dty, db, h, f = e
        return lbk.Expert(matrix(gty, h, f, up(gty, gb, h), lbk.LAYOUT_PLANAR),
                          matrix(uty, h, f, up(uty, ub, h), lbk.LAYOUT_PLANAR),
                          matrix(dty, f, h, up(dty, db, f), lbk.LAYOUT_PLANAR))

    dex = [ex(e) for e in experts]
    sh = ex(shared)
    rt = dev(router)
    keep.append(rt)
    rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, H, E, rt.data_ptr(), rt.numel() * 4)
    bias = dev(np.zeros(E, np.float32))
    keep.append(bias)
    full = lbk.MoeLayer(ctx(), dex, sh, rm, bias, k, 2.826)
    er = E // world
    ranks = [lbk.EpLayer(ctx(), dex[r * er:(r + 1) * er], sh, rm, bias, k, 2.826, E, r * er) for r in range(world)]
    return full, ranks, keep, rng


def _full_forward(full, x, T):
    from gpu_helpers import clean_status

    H = full.hidden
    ws = torch.zeros(full.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.full((T * H,), float("nan"), device="cuda")
    routed = torch.zeros(T * full.top_k * 2, dtype=torch.int32, device="cuda")
    full.forward(x, T, out, ws, routed_out=routed)
    clean_status()
    return out, routed


@pytest.mark.gpu
@pytest.mark.parametrize("H,F,E,k,T", [(4096, 1536, 24, 8, 1), (2048, 512, 16, 4, 3), (4096, 256, 32, 8, 5)])
def test_single_rank_ep_equals_moe_forward(H, F, E, k, T):
    from gpu_helpers import clean_status, dev

    full, ranks, keep, rng = _gpu_layers(H, F, E, k, H + F + E + T, 1)
    moe = ep.ExpertParallelMoe(ranks[0])
    x = dev(rng.standard_normal(T * H).astype(np.float32))
    out = torch.full((T * H,), float("nan"), device="cuda")
    routed = torch.zeros(T * k * 2, dtype=torch.int32, device="cuda")
    moe.forward(x, T, out, routed_out=routed)
    clean_status()
    want, wr = _full_forward(full, x, T)
    assert torch.equal(routed.cpu(), wr.cpu())
    assert torch.equal(out.view(torch.int32).cpu(), want.view(torch.int32).cpu())
    full.close()
    ranks[0].close()


@pytest.mark.gpu
@pytest.mark.parametrize("world,H,F,E,k,T", [(2, 4096, 1536, 48, 8, 1), (4, 2048, 512, 16, 4, 6), (8, 4096, 256, 64, 8, 2)])
def test_ranks_simulated_on_one_gpu_equal_moe_forward(world, H, F, E, k, T):
    """`world` rank layers on one GPU: route on rank 0, hand each rank its rows
    (the exchange done by slicing), items_forward per rank, place, combine."""
    from gpu_helpers import clean_status, dev

    full, ranks, keep, rng = _gpu_layers(H, F, E, k, 7 * H + F + E + T, world)
    home = ranks[0]
    x = dev(rng.standard_normal(T * H).astype(np.float32))
    er = E // world
    q8b = home.q8_bytes
    ws = torch.zeros(max(home.workspace_bytes(T), home.workspace_bytes(T * k)), dtype=torch.uint8, device="cuda")
    routed = torch.empty((T * k, 2), dtype=torch.int32, device="cuda")
    q8 = torch.empty((T, q8b), dtype=torch.uint8, device="cuda")
    home.route(x, T, routed, q8, ws)
    ids = routed[:, 0]
    plan = ep.local_plan(ids, er, world)
    send = plan.send
    rows = ep.pack_rows(q8, ids, plan, k, er)
    dots = []
    for r, chunk in enumerate(torch.split(rows, send)):
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
    want, wr = _full_forward(full, x, T)
    assert torch.equal(routed.view(-1).cpu(), wr.cpu())
    assert torch.equal(out.view(torch.int32).cpu(), want.view(torch.int32).cpu())
    full.close()
    for r in ranks:
        r.close()


@pytest.mark.gpu
def test_items_forward_reports_out_of_range_local_expert():
    """A local expert ID beyond the rank's share is reported through the
    status word (INVALID_PARAMETER, index = the ID); the kernels stay in bounds."""
    import lbk
    from gpu_helpers import expect_status

    full, ranks, keep, rng = _gpu_layers(2048, 512, 16, 4, 5, 2)
    r1 = ranks[1]
    n = 2
    imgs = torch.zeros((n, r1.q8_bytes), dtype=torch.uint8, device="cuda")
    items = torch.tensor([[3, 0], [8, 0]], dtype=torch.int32, device="cuda")
    ws = torch.zeros(r1.workspace_bytes(n), dtype=torch.uint8, device="cuda")
    dots = torch.zeros((n, 2048), device="cuda")
    r1.items_forward(imgs, items, n, dots, ws)
    d = expect_status(15)
    assert d.index == 8
    full.close()
    for r in ranks:
        r.close()


@pytest.mark.gpu
def test_nccl_ranks_equal_moe_forward():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    r = _torchrun(2, "gpu", timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ok" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("world,T", [(2, 12), (4, 16)])
def test_grouped_expert_parallel_equals_ungrouped_forward(world, T):
    """Grouped kernels on every rank (items grouped by local expert; the home
    rank's shared-expert pass grouped by token) against the ungrouped
    single-GPU forward: bit for bit."""
    from gpu_helpers import clean_status, dev

    H, F, E, k = 2048, 512, 16, 4
    full, ranks, keep, rng = _gpu_layers(H, F, E, k, 31 * T + world, world)
    full.set_grouping(0)
    for r in ranks:
        r.set_grouping(2)
    home = ranks[0]
    x = dev(rng.standard_normal(T * H).astype(np.float32))
    er = E // world
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
    want, wr = _full_forward(full, x, T)
    assert torch.equal(routed.view(-1).cpu(), wr.cpu())
    assert torch.equal(out.view(torch.int32).cpu(), want.view(torch.int32).cpu())
    full.close()
    for r in ranks:
        r.close()


def _peer_ranks(ranks, world, cap):
    """`world` simulated ranks on one GPU: exchange buffers in this process,
    every rank's scratch as PeerExpertParallelMoe holds it."""
    xl = ranks[0].exchange_layout(cap)
    bufs = [torch.zeros(xl.total, dtype=torch.uint8, device="cuda") for _ in range(world)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    cap_items = world * cap * ranks[0].top_k
    q8b, H = ranks[0].q8_bytes, ranks[0].hidden
    st = []
    for r in range(world):
        st.append(dict(
            q8_items=torch.empty((cap_items, q8b), dtype=torch.uint8, device="cuda"),
            items=torch.zeros((cap_items, 2), dtype=torch.int32, device="cuda"),
            returns=torch.zeros(cap_items, dtype=torch.int64, device="cuda"),
            count=torch.zeros(1, dtype=torch.int32, device="cuda"),
            dots=torch.empty((cap_items, H), dtype=torch.float32, device="cuda"),
            ws=torch.zeros(ranks[r].workspace_bytes(max(cap_items, cap)), dtype=torch.uint8, device="cuda")))
    return xl, bufs, peers, st


@pytest.mark.gpu
@pytest.mark.parametrize("world,H,F,E,k,tokens,grouping,tc", [
    (1, 4096, 1536, 24, 8, (3,), 0, 0), (2, 4096, 1536, 48, 8, (1, 2), 0, 0), (4, 2048, 512, 16, 4, (6, 0, 3, 5), 0, 0),
    (8, 4096, 256, 64, 8, (2, 1, 0, 2, 2, 1, 2, 2), 0, 0),
    # items on the grouped kernels (grouped on the device by local expert, counted there)
    (2, 4096, 512, 16, 8, (16, 11), 2, 0), (4, 2048, 256, 32, 4, (9, 0, 16, 3), 2, 0),
    # ... with the gate/up on the tensor cores (groups of up to 32 pairs, partial row tiles)
    (2, 4096, 512, 16, 8, (16, 11), 2, 1), (4, 2048, 768, 32, 4, (9, 0, 16, 3), 2, 1),
    (2, 4096, 1536, 8, 8, (40, 33), 2, 1)])
def test_peer_exchange_ranks_simulated_on_one_gpu(world, H, F, E, k, tokens, grouping, tc):
    """The peer-memory exchange (lbk_ep_publish / gather / items_forward_counted
    / scatter / combine_exchange) with `world` ranks on one GPU: each rank's
    exchange buffer is device memory of this process, addressed by every rank
    as its peers would address it, each rank with its own tokens (one with
    none). Every call of a step is issued after the calls whose flags it waits
    for, so no kernel waits on another. Two steps on the same buffers (the
    second with the shared expert from lbk_ep_shared and the items' rows
    returned in place by lbk_ep_items_return): every rank's output equals
    lbk_moe_forward on its tokens bit for bit."""
    from gpu_helpers import clean_status, dev

    full, ranks, keep, rng = _gpu_layers(H, F, E, k, 13 * H + F + E + world, world)
    for r in ranks:
        r.set_grouping(grouping)
        r.set_tensor_cores(tc)
    cap = max(tokens)
    xl, bufs, peers, st = _peer_ranks(ranks, world, cap)
    for step in range(2):
        xs = [dev(rng.standard_normal(max(T, 1) * H).astype(np.float32)) for T in tokens]
        for r in range(world):
            ranks[r].publish(xs[r], tokens[r], bufs[r].data_ptr(), cap, st[r]["ws"])
        for r in range(world):
            s = st[r]
            ranks[r].gather(peers, world, r, cap, s["q8_items"], s["items"], s["returns"], s["count"])
            if step == 0:  # items, then their dots sent home
                ranks[r].items_forward_counted(s["q8_items"], s["items"], s["count"], s["dots"], s["ws"])
                ranks[r].scatter(peers, world, r, cap, s["dots"], s["returns"], s["count"])
            else:  # the down rows stored in the home buffers directly
                ranks[r].items_return(peers, world, r, cap, s["q8_items"], s["items"], s["returns"], s["count"],
                                      s["ws"])
        outs = [torch.full((max(T, 1) * H,), float("nan"), device="cuda") for T in tokens]
        for r in range(world):
            sd = None
            if step == 1 and tokens[r]:  # the shared expert by lbk_ep_shared, its own workspace
                sd = torch.full((cap * H,), float("nan"), device="cuda")
                ws2 = torch.zeros(ranks[r].workspace_bytes(cap), dtype=torch.uint8, device="cuda")
                ranks[r].shared(bufs[r].data_ptr(), cap, tokens[r], sd, ws2)
            ranks[r].combine_exchange(bufs[r].data_ptr(), world, cap, tokens[r], outs[r] if tokens[r] else None,
                                      st[r]["ws"], shared_dots=sd)
        clean_status()
        for r in range(world):
            T = tokens[r]
            ctl = bufs[r][xl.control:xl.control + 16].view(torch.int32).cpu().tolist()
            assert ctl[0] == T and ctl[1] == step + 1 and ctl[2] == step + 1, f"rank {r} control {ctl}"
            assert bufs[r][xl.control + 64:xl.control + 64 + 4 * world].view(torch.int32).cpu().tolist() == \
                [step + 1] * world, f"rank {r} done flags"
            if T == 0:
                continue
            want, wr = _full_forward(full, xs[r][:T * H], T)
            got_routing = bufs[r][xl.routing:xl.routing + T * k * 8].view(torch.int32)
            assert torch.equal(got_routing.cpu(), wr.cpu()), f"rank {r} routing"
            assert torch.equal(outs[r].view(torch.int32).cpu(), want.view(torch.int32).cpu()), f"rank {r} output"
    full.close()
    for r in ranks:
        r.close()


@pytest.mark.gpu
def test_peer_exchange_wait_that_runs_out_reports_timeout():
    """Rank 1 of 2 never publishes: rank 0's gather waits its limit out and
    reports LBK_TIMEOUT (index 8, bits = the step); its combine, with no dots
    from rank 1, reports LBK_TIMEOUT (index 9). Both return, the context stays
    usable, and a full step afterwards (rank 1 catching up) is exact."""
    from gpu_helpers import clean_status, dev, expect_status

    H, F, E, k, world, cap = 2048, 256, 16, 4, 2, 2
    full, ranks, keep, rng = _gpu_layers(H, F, E, k, 99, world)
    xl, bufs, peers, st = _peer_ranks(ranks, world, cap)
    for r in ranks:
        r.set_wait_limit(2000)
    x = dev(rng.standard_normal(cap * H).astype(np.float32))
    s0 = st[0]
    ranks[0].publish(x, cap, bufs[0].data_ptr(), cap, s0["ws"])
    ranks[0].gather(peers, world, 0, cap, s0["q8_items"], s0["items"], s0["returns"], s0["count"])
    d = expect_status(31)
    assert d.index == 8 and d.bits == 1
    ranks[0].combine_exchange(bufs[0].data_ptr(), world, cap, cap, torch.zeros(cap * H, device="cuda"), s0["ws"])
    d = expect_status(31)
    assert d.index == 9 and d.bits == 1
    # rank 1 catches up on step 1 (rank 0's own step-1 flags are set; its scatter of step 1 ran short)
    ranks[1].publish(x, cap, bufs[1].data_ptr(), cap, st[1]["ws"])
    for r in range(world):
        s = st[r]
        ranks[r].gather(peers, world, r, cap, s["q8_items"], s["items"], s["returns"], s["count"])
        ranks[r].items_forward_counted(s["q8_items"], s["items"], s["count"], s["dots"], s["ws"])
        ranks[r].scatter(peers, world, r, cap, s["dots"], s["returns"], s["count"])
    out = torch.full((cap * H,), float("nan"), device="cuda")
    ranks[1].combine_exchange(bufs[1].data_ptr(), world, cap, cap, out, st[1]["ws"])
    clean_status()
    want, _ = _full_forward(full, x, cap)
    assert torch.equal(out.view(torch.int32).cpu(), want.view(torch.int32).cpu())
    full.close()
    for r in ranks:
        r.close()


@pytest.mark.gpu
@pytest.mark.parametrize("world,B", [(4, 1), (2, 4)])
def test_peer_exchange_stack_chain_equals_block_forward(world, B):
    """Config 5's expert-parallel chain at reduced depth: three layers of
    hidden += MoE(RMSNorm(hidden)) with the MoE step through the peer exchange
    (ranks simulated on one GPU, one set of exchange buffers for all layers,
    each rank with its own B tokens), against lbk_moe_block_forward of the
    whole layers fed back into itself: every rank's hidden state equals the
    one-GPU chain bit for bit after every layer."""
    import lbk
    from gpu_helpers import clean_status, ctx, dev

    H, F, E, k, depth = 4096, 512, 32, 8, 3
    stack = [_gpu_layers(H, F, E, k, 500 + l, world) for l in range(depth)]
    ranks0 = stack[0][1]
    xl, bufs, peers, st = _peer_ranks(ranks0, world, B)
    rng = np.random.default_rng(7)
    norm_w = dev((1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    hid = [dev(rng.standard_normal(B * H).astype(np.float32)) for _ in range(world)]
    ref = [h.clone() for h in hid]
    normed = [torch.empty(B * H, device="cuda") for _ in range(world)]
    delta = [torch.empty(B * H, device="cuda") for _ in range(world)]
    bws = torch.zeros(stack[0][0].block_workspace_bytes(B), dtype=torch.uint8, device="cuda")
    for l, (full, ranks, keep, _) in enumerate(stack):
        for r in range(world):
            ctx().rms_norm(hid[r], norm_w, H, B, 1e-6, normed[r], mode=lbk.ROUTER_TREE)
            ranks[r].publish(normed[r], B, bufs[r].data_ptr(), B, st[r]["ws"])
        for r in range(world):
            s = st[r]
            ranks[r].gather(peers, world, r, B, s["q8_items"], s["items"], s["returns"], s["count"])
            ranks[r].items_return(peers, world, r, B, s["q8_items"], s["items"], s["returns"], s["count"], s["ws"])
        for r in range(world):
            ranks[r].combine_exchange(bufs[r].data_ptr(), world, B, B, delta[r], st[r]["ws"])
            ctx().residual_add(hid[r], delta[r], B * H)
            full.block_forward(ref[r], norm_w, 1e-6, B, bws)
        clean_status()
        for r in range(world):
            assert torch.equal(hid[r].view(torch.int32).cpu(), ref[r].view(torch.int32).cpu()), f"layer {l} rank {r}"
    for full, ranks, keep, _ in stack:
        full.close()
        for r in ranks:
            r.close()
