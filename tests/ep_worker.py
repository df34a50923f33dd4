"""One rank of the expert-parallel tests, launched by torch.distributed.run.

--mode cpu: gloo ranks on the host; the compute stages are FakeEpLayer
(exact small-integer f32 arithmetic), so the test checks the dispatch, return
and placement plumbing of ep.ExpertParallelMoe bit for bit against the same
stages run on one rank holding every expert.

--mode gpu: nccl ranks, one GPU each; the compute stages are lbk.EpLayer, and
each rank's output must equal lbk_moe_forward of the whole layer on its own
GPU bit for bit (routing identical), both with the exchange over collectives
(ep.ExpertParallelMoe) and over IPC-mapped peer memory
(ep.PeerExpertParallelMoe).

Exits non-zero on any mismatch; rank 0 prints "ok" when every rank passed.
"""

import argparse
import datetime
import os
import pathlib
import sys

import numpy as np
import torch
import torch.distributed as dist

REPO = pathlib.Path(__file__).resolve().parents[1]
for sub in ("oracle", "lightbridge-engine_b200", "tests"):
    sys.path.insert(0, str(REPO / sub))

import ep  # noqa: E402


class FakeEpLayer:
    """Stand-in for lbk.EpLayer on the host. route: top-k of x @ W^T in
    ascending ID order with coefficients 1 / (j + 2), Q8 image = round(8x)
    clipped to int8; items_forward: dots = image * (e + 1) + e / 2 for global
    expert e; combine: sum_j c_j * dots_j then + shared (image / 4), in order.
    Every value is exact in f32, so any misplaced row shows."""

    def __init__(self, W: torch.Tensor, k: int, first: int, local: int):
        self.W = W
        self.global_experts, self.hidden = W.shape
        self.top_k = k
        self.first_expert = first
        self.local_experts = local
        self.q8_bytes = self.hidden

    def workspace_bytes(self, count):
        return 16

    def route(self, x, tokens, routed, q8, ws):
        xs = x.view(tokens, self.hidden)
        logits = xs.double() @ self.W.double().T
        ids = torch.sort(torch.topk(logits, self.top_k, dim=1).indices, dim=1).values.to(torch.int32)
        coef = (1.0 / (torch.arange(self.top_k, dtype=torch.float32) + 2.0)).expand(tokens, -1)
        r = routed.view(tokens, self.top_k, 2)
        r[:, :, 0] = ids
        r[:, :, 1] = coef.contiguous().view(torch.int32)
        q8.copy_(torch.clamp(torch.round(xs * 8.0), -127, 127).to(torch.int8).view(torch.uint8))

    def items_forward(self, q8_items, items, n, dots, ws):
        e = (items[:, 0].to(torch.int64) + self.first_expert)
        assert int(items[:, 0].min()) >= 0 and int(items[:, 0].max()) < self.local_experts
        img = q8_items.view(torch.int8).to(torch.float32)
        dots.copy_(img * (e + 1).to(torch.float32)[:, None] + (e.to(torch.float32) * 0.5)[:, None])

    def combine(self, q8, tokens, routed, routed_dots, out, ws):
        k, H = self.top_k, self.hidden
        c = routed.view(tokens, k, 2)[:, :, 1].contiguous().view(torch.float32)
        d = routed_dots.view(tokens, k, H)
        acc = torch.zeros((tokens, H), dtype=torch.float32)
        for j in range(k):
            acc = acc + c[:, j:j + 1] * d[:, j]
        shared = q8.view(torch.int8).to(torch.float32) / 4.0
        out.view(tokens, H).copy_(acc + shared)


def cpu_case(rank, world, E, H, k, tokens_per_rank, seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn((E, H), generator=g)
    xs = [torch.randn((t * H,), generator=g) for t in tokens_per_rank]
    er = E // world
    moe = ep.ExpertParallelMoe(FakeEpLayer(W, k, rank * er, er))
    T = tokens_per_rank[rank]
    out = torch.full((T * H,), float("nan"))
    routed = torch.zeros((T * k * 2,), dtype=torch.int32)
    moe.forward(xs[rank], T, out, routed_out=routed)
    # the same stages with every expert on one rank, no exchange
    one = FakeEpLayer(W, k, 0, E)
    want = torch.full((T * H,), float("nan"))
    if T:
        r1 = torch.empty((T * k, 2), dtype=torch.int32)
        q1 = torch.empty((T, H), dtype=torch.uint8)
        one.route(xs[rank], T, r1, q1, None)
        d1 = torch.empty((T * k, H))
        it = torch.zeros((T * k, 2), dtype=torch.int32)
        it[:, 0] = r1[:, 0]
        one.items_forward(q1.index_select(0, torch.arange(T * k) // k), it, T * k, d1, None)
        one.combine(q1, T, r1, d1, want, None)
        assert torch.equal(routed.view(-1), r1.view(-1)), "routing differs"
    assert torch.equal(out.view(torch.int32), want.view(torch.int32)), f"rank {rank}: output differs"


def gpu_case(rank, world, E, H, F, k, tokens_per_rank, seed):
    import lbk
    import synth

    dev = torch.device("cuda", rank)
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    TY_G, TY_D, TY_S = lbk.TYPE_IQ2_S, lbk.TYPE_IQ3_S, lbk.TYPE_Q4_K

    def mat(ty, in_w, out_w):
        t = torch.from_numpy(synth.planar_np(ty, synth.packed_np(rng, ty, in_w, out_w), in_w)).to(dev)
        return lbk.matrix(ty, in_w, out_w, t, lbk.LAYOUT_PLANAR), t

    keep = []

    def expert(gty, dty):
        g, tg = mat(gty, H, F)
        u, tu = mat(gty, H, F)
        d, td = mat(dty, F, H)
        keep.extend([tg, tu, td])
        return lbk.Expert(g, u, d)

    experts = [expert(TY_G, TY_D) for _ in range(E)]  # every rank draws the same tables
    shared = expert(TY_S, TY_S)
    rt = torch.from_numpy(router).to(dev)
    rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, H, E, rt.data_ptr(), rt.numel() * 4)
    bias = torch.zeros(E, dtype=torch.float32, device=dev)
    xs = [rng.standard_normal(t * H).astype(np.float32) for t in tokens_per_rank]
    ctx = lbk.Context(rank)
    er = E // world
    epl = lbk.EpLayer(ctx, experts[rank * er:(rank + 1) * er], shared, rm, bias, k, 2.826, E, rank * er)
    full = lbk.MoeLayer(ctx, experts, shared, rm, bias, k, 2.826)
    moe = ep.ExpertParallelMoe(epl)
    T = tokens_per_rank[rank]
    x = torch.from_numpy(xs[rank]).to(dev)
    out = torch.full((max(T, 1) * H,), float("nan"), device=dev)
    routed = torch.zeros((max(T, 1) * k * 2,), dtype=torch.int32, device=dev)
    for _ in range(2):  # the second step reuses the grown workspace
        moe.forward(x, T, out, routed_out=routed)
    torch.cuda.synchronize(dev)
    ctx.raise_status()
    if T:
        ws = torch.zeros(full.workspace_bytes(T), dtype=torch.uint8, device=dev)
        want = torch.full((T * H,), float("nan"), device=dev)
        wr = torch.zeros((T * k * 2,), dtype=torch.int32, device=dev)
        full.forward(x, T, want, ws, routed_out=wr)
        torch.cuda.synchronize(dev)
        ctx.raise_status()
        assert torch.equal(routed[: T * k * 2].cpu(), wr.cpu()), f"rank {rank}: routing differs"
        assert torch.equal(out[: T * H].view(torch.int32).cpu(), want.view(torch.int32).cpu()), f"rank {rank}: output differs"
    # the same layer step with the exchange over peer memory (IPC-mapped buffers)
    peer = ep.PeerExpertParallelMoe(epl, max(tokens_per_rank))
    for step in range(3):  # later steps reuse the buffers
        out.fill_(float("nan"))
        peer.forward(x, T, out)
        torch.cuda.synchronize(dev)
        ctx.raise_status()
        if T:
            assert torch.equal(out[: T * H].view(torch.int32).cpu(), want.view(torch.int32).cpu()), \
                f"rank {rank}: peer exchange output differs (step {step})"
    peer.close()
    epl.close()
    full.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=("cpu", "gpu"), required=True)
    args = ap.parse_args()
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    if args.mode == "gpu":
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    else:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        if args.mode == "cpu":
            # ragged token counts, a rank with no tokens, E = 2k (a token's pairs can all land on one rank)
            for E, H, k, tpr, seed in [(16, 64, 4, [3, 5], 1), (16, 32, 4, [0, 4], 2), (8, 32, 4, [2, 0], 3),
                                       (32, 48, 8, [1, 1], 4), (12, 16, 3, [7, 2], 5)]:
                cpu_case(rank, world, E, H, k, tpr[:world] + [1] * (world - len(tpr)), seed)
        else:
            for E, H, F, k, tpr, seed in [(16, 2048, 512, 4, [2, 3], 11), (24, 4096, 256, 8, [1, 0], 12),
                                          (32, 2048, 256, 8, [4, 1], 13)]:
                gpu_case(rank, world, E, H, F, k, tpr[:world] + [1] * (world - len(tpr)), seed)
        dist.barrier()
    finally:
        dist.destroy_process_group()
    if rank == 0:
        print("ok")


if __name__ == "__main__":
    main()
