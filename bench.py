"""Benchmark: routed-MoE single-token decode through HBM-resident expert tables.

Workload: one routed-MoE FFN layer per decode token --
hidden 4096, 192 experts (gate/up IQ2_S 4096->1536, down IQ3_S 1536->4096),
one shared expert (all Q4_K), F32 router 4096x192 ~ N(0, 0.02), top-8 with
the reference's renormalisation (weight_scale 2.826, zero selection bias),
token ~ N(0, 1). Weights are synthetic (seeded; see synth.py) because the
reference measures only a real checkpoint that is not available.

A step is one batch of TOKENS_PER_STEP independent single-token layer passes.
Consecutive tokens rotate over LAYERS distinct resident layer tables (10.4 GB
in total), so every pass streams its weights from HBM, not from the 126 MB
L2 ("inputs larger than L2").

value   : tokens/s with inputs already resident (CUDA graph of one step,
          CUDA events, max over ranks).
e2e     : tokens/s through the C ABI call per token (lbk_moe_forward), with
          each step's tokens copied from pinned host memory and its outputs
          read back inside the timed region.
roofline: the dominant kernel's algorithmic bytes / its CUDA-event time.
cpu_baseline: the CPU restatement of the reference's AVX2 path (oracle/),
          moe_routed_by_id_into as the reference runs it (preflight + accept).

--impl reference times that CPU path on the host cores on the same config.
With N>1 GPUs every rank runs its own resident copy of the layers on its own
tokens (replicas; weak scaling).

ep      : at every N, config 4's layer step with the experts sharded over the
          N GPUs (192 / N each), 64 tokens per GPU, dispatch and return over
          peer memory (lightbridge-engine_b200/ep.py, PeerExpertParallelMoe):
          tokens/s, per-stage times (dispatch, return), gpus_active. `value`
          stays the config-3 line, so the scaling run's efficiency reflects
          replicas of config 3; the `ep` record's tokens/s is the expert-
          parallel curve.

--config 4 measures that batched layer as the line itself (--exchange nccl:
the NCCL all-to-all exchange instead); weak scaling.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "lightbridge-engine_b200"))

H, F, E, K_TOP = 4096, 1536, 192, 8
WEIGHT_SCALE = 2.826
TOKENS_PER_STEP = 256
LAYERS = 8
BATCH_TOKENS = 64  # config 4, per GPU
TYPE_IQ2_S, TYPE_IQ3_S, TYPE_Q4_K, TYPE_Q5_K = 22, 21, 12, 13
METRIC = "routed-MoE decode tokens/s (single-token MoE FFN layer, config 3)"


def row_bytes(ty: int, k: int) -> int:
    return k // 256 * {TYPE_IQ2_S: 82, TYPE_IQ3_S: 110, TYPE_Q4_K: 144, TYPE_Q5_K: 176}[ty]


# algorithmic bytes per token: router + 8 routed experts + shared (weights read once) + x + out
ROUTER_B = E * H * 4
GATE_UP_B = K_TOP * 2 * F * row_bytes(TYPE_IQ2_S, H) + 2 * F * row_bytes(TYPE_Q4_K, H)
DOWN_B = K_TOP * H * row_bytes(TYPE_IQ3_S, F) + H * row_bytes(TYPE_Q4_K, F)
X_B, OUT_B = H * 4, H * 4
LAYER_B = ROUTER_B + GATE_UP_B + DOWN_B + X_B + OUT_B


def peaks() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profiled_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` from a committed ncu summary, if any:
    (bytes, the summary's path). Not measured in this run: ncu captures come
    from a separate profiling command (named in the summary)."""
    for f in sorted((REPO / "profiles").glob("*.md")) + sorted((REPO / "profiles").glob("*.txt")):
        for line in f.read_text().splitlines():
            if line.startswith(f"traffic_bytes_per_launch[{kernel}]:"):
                try:
                    return int(float(line.split(":", 1)[1].split()[0])), str(f.relative_to(REPO))
                except ValueError:
                    pass
    return None, None


def cpu_model() -> str:
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index: int):
        self.proc = None
        self.index = index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[2:]):
                if v.lower() == "active":
                    reasons.add(n)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---------------------------------------------------------------- reference

def reference_arm(args, rank: int) -> None:
    """The reference's CPU path (its AVX2 restatement in oracle/) on the host cores."""
    if rank != 0:
        return
    sys.path.insert(0, str(REPO / "oracle"))
    import numpy as np

    import oracle as orc
    import synth

    threads = orc.hw_threads()
    rng = np.random.default_rng(2)
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    experts = []
    for _ in range(E):
        experts.append((TYPE_IQ2_S, synth.packed_np(rng, TYPE_IQ2_S, H, F), TYPE_IQ2_S,
                        synth.packed_np(rng, TYPE_IQ2_S, H, F), TYPE_IQ3_S, synth.packed_np(rng, TYPE_IQ3_S, F, H), H, F))
    shared = (TYPE_Q4_K, synth.packed_np(rng, TYPE_Q4_K, H, F), TYPE_Q4_K, synth.packed_np(rng, TYPE_Q4_K, H, F),
              TYPE_Q4_K, synth.packed_np(rng, TYPE_Q4_K, F, H), H, F)
    table = orc.ExpertTable(experts, shared, router=router, hidden=H)
    bias = np.zeros(E, np.float32)
    xs = rng.standard_normal((args.warmup + args.steps, H)).astype(np.float32)
    for i in range(args.warmup):
        orc.moe_token(table, bias, K_TOP, WEIGHT_SCALE, xs[i], preflight=True, simd=True, threads=threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        orc.moe_token(table, bias, K_TOP, WEIGHT_SCALE, xs[args.warmup + i], preflight=True, simd=True, threads=threads)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q8_k x packed (int8 dots, f32 tails)",
        "data": "synthetic (seeded, config shapes)",
        "config": {"workload": "config3: routed-MoE FFN layer, single-token decode", "hidden": H, "experts": E,
                   "expert_ffn": F, "top_k": K_TOP, "gate_up": "IQ2_S", "down": "IQ3_S", "shared": "Q4_K",
                   "step": "1 token (bounded sample of the GPU arm's 256-token step)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} tokens through one layer, moe_routed_by_id_into as-is (preflight + accept), AVX2 restatement"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm

def build_layers(ctx, lbk, torch, dev, layers: int, seed0: int, keep_gguf_layer0: bool):
    import synth

    gen = torch.Generator(device=dev)
    tables = []
    host0 = None
    for l in range(layers):
        gen.manual_seed(seed0 + l)
        keep = []
        router = (torch.randn(E, H, device=dev, generator=gen) * 0.02).contiguous()
        keep.append(router)

        def stacked(ty, k, rows):
            g = synth.packed_torch(gen, ty, k, rows * E, dev)
            mb, pb = synth.matrix_bytes(ty, k, rows), synth.planar_bytes(ty, k, rows)
            p = torch.empty(pb * E, dtype=torch.uint8, device=dev)
            for e in range(E):
                ctx.repack(lbk.matrix(ty, k, rows, g[e * mb:(e + 1) * mb]), p[e * pb:(e + 1) * pb])
            return g, p

        gg, gp = stacked(TYPE_IQ2_S, H, F)
        ug, up = stacked(TYPE_IQ2_S, H, F)
        dg, dp = stacked(TYPE_IQ3_S, F, H)
        keep += [gp, up, dp]
        sh = []
        for ty, k, rows in [(TYPE_Q4_K, H, F), (TYPE_Q4_K, H, F), (TYPE_Q4_K, F, H)]:
            g = synth.packed_torch(gen, ty, k, rows, dev)
            p = torch.empty(synth.planar_bytes(ty, k, rows), dtype=torch.uint8, device=dev)
            ctx.repack(lbk.matrix(ty, k, rows, g), p)
            sh.append((ty, k, rows, g, p))
            keep.append(p)
        torch.cuda.synchronize()
        if l == 0 and keep_gguf_layer0:
            host0 = {
                "router": router.cpu().numpy(),
                "gate": gg.cpu().numpy(), "up": ug.cpu().numpy(), "down": dg.cpu().numpy(),
                "shared": [s[3].cpu().numpy() for s in sh],
            }
        del gg, ug, dg
        mbg, mbd = synth.planar_bytes(TYPE_IQ2_S, H, F), synth.planar_bytes(TYPE_IQ3_S, F, H)
        experts = [
            lbk.Expert(lbk.matrix(TYPE_IQ2_S, H, F, gp[e * mbg:(e + 1) * mbg], lbk.LAYOUT_PLANAR),
                       lbk.matrix(TYPE_IQ2_S, H, F, up[e * mbg:(e + 1) * mbg], lbk.LAYOUT_PLANAR),
                       lbk.matrix(TYPE_IQ3_S, F, H, dp[e * mbd:(e + 1) * mbd], lbk.LAYOUT_PLANAR))
            for e in range(E)
        ]
        shared = lbk.Expert(*[lbk.matrix(ty, k, rows, p, lbk.LAYOUT_PLANAR) for ty, k, rows, _, p in sh])
        bias = torch.zeros(E, device=dev)
        keep.append(bias)
        rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, H, E, router.data_ptr(), router.numel() * 4)
        layer = lbk.MoeLayer(ctx, experts, shared, rm, bias, K_TOP, WEIGHT_SCALE)
        assert layer.fused
        tables.append((layer, keep))
    return tables, host0


def cpu_baseline(host0, xs_host, budget_s: float = 8.0) -> dict:
    """The reference's CPU path (the oracle's AVX2 restatement) on the host
    cores, on layer 0 of the bench's tables: moe_routed_by_id_into as the
    reference runs it (a preflight pass of every expert, then the accepting
    pass; moe.rs:29-60) on all host threads -- the reported value -- plus the
    same at the reference's default pool of ceil(threads / 2)
    (bridge-kernels-cpu/src/lib.rs:121-139) and a single-pass run (no
    preflight: half the expert work, the same result)."""
    sys.path.insert(0, str(REPO / "oracle"))
    import numpy as np

    import oracle as orc

    mbg = H // 256 * 82 * F
    mbd = F // 256 * 110 * H
    experts = [(TYPE_IQ2_S, host0["gate"][e * mbg:(e + 1) * mbg], TYPE_IQ2_S, host0["up"][e * mbg:(e + 1) * mbg],
                TYPE_IQ3_S, host0["down"][e * mbd:(e + 1) * mbd], H, F) for e in range(E)]
    s = host0["shared"]
    shared = (TYPE_Q4_K, s[0], TYPE_Q4_K, s[1], TYPE_Q4_K, s[2], H, F)
    table = orc.ExpertTable(experts, shared, router=host0["router"], hidden=H)
    bias = np.zeros(E, np.float32)
    threads = orc.hw_threads()

    def run(nthreads: int, preflight: bool, budget: float):
        orc.moe_token(table, bias, K_TOP, WEIGHT_SCALE, xs_host[0], preflight=preflight, simd=True, threads=nthreads)
        n, t0 = 0, time.perf_counter()
        while True:
            orc.moe_token(table, bias, K_TOP, WEIGHT_SCALE, xs_host[(n + 1) % len(xs_host)], preflight=preflight,
                          simd=True, threads=nthreads)
            n += 1
            dt = time.perf_counter() - t0
            if dt >= budget or n >= 2000:
                return n, n / dt

    n, v = run(threads, True, budget_s)
    half = (threads + 1) // 2
    nh, vh = run(half, True, budget_s * 0.5)
    ns, vs = run(threads, False, budget_s * 0.5)
    return {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "cpu_model": cpu_model(),
            "sample": f"{n} tokens through layer 0, moe_routed_by_id_into as-is (preflight + accept), AVX2 restatement",
            "variants": {
                f"as-is, {half} threads (the reference's default ceil(threads/2))": {"value": vh, "tokens": nh},
                f"single pass (no preflight), {threads} threads": {"value": vs, "tokens": ns}},
            "gb_per_s_as_is": v * LAYER_B / 1e9}


def our_arm(args, rank: int, world: int, local_rank: int) -> None:
    import numpy as np
    import torch

    import lbk

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist_mod

        dist = dist_mod
    ctx = lbk.Context(local_rank)
    tables, host0 = build_layers(ctx, lbk, torch, dev, LAYERS, 4 + 97 * rank, keep_gguf_layer0=(rank == 0 and world == 1))
    ws_bytes = tables[0][0].workspace_bytes(1)
    wss = [torch.zeros(ws_bytes, dtype=torch.uint8, device=dev) for _ in tables]
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + rank)
    xs = torch.randn(TOKENS_PER_STEP, H, device=dev, generator=gen)
    outs = torch.zeros(TOKENS_PER_STEP, H, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step_calls(s):
        for t in range(TOKENS_PER_STEP):
            layer = tables[t % LAYERS][0]
            layer.forward(xs[t], 1, outs[t], wss[t % LAYERS], stream=s.cuda_stream)

    stream.wait_stream(torch.cuda.current_stream())  # weights and inputs come from the default stream
    with torch.cuda.stream(stream):
        step_calls(stream)  # warm: sets kernel attributes outside capture
    torch.cuda.synchronize()
    ctx.raise_status(stream.cuda_stream)

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step_calls(stream)
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ctx.raise_status(stream.cuda_stream)

    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if dist:
        dist.barrier()
    clk = clocks.stop()
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ctx.raise_status(stream.cuda_stream)
    tokens_total = args.steps * TOKENS_PER_STEP * world
    value = tokens_total / (ms / 1000.0)

    # per-kernel times: a traced copy of one step, replayed with a sync each time
    for layer, _ in tables:
        layer.trace(True)
    tgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(tgraph, stream=stream):
        for t in range(LAYERS):
            tables[t][0].forward(xs[t], 1, outs[t], wss[t], stream=stream.cuda_stream)
    sums = [0.0, 0.0, 0.0]
    reps = 64
    for _ in range(reps):
        tgraph.replay()
        torch.cuda.synchronize()
        for layer, _ in tables:
            r = layer.trace_read()
            for i in range(3):
                sums[i] += r[i]
    n_traced = reps * LAYERS
    avg = [s / n_traced for s in sums]  # ms: router, gate/up, down
    for layer, _ in tables:
        layer.trace(False)
    del tgraph
    kernels = [("router_fused", ROUTER_B + X_B, avg[0]), ("moe_gate_up", GATE_UP_B, avg[1]),
               ("moe_down", DOWN_B + OUT_B, avg[2])]
    dom = max(kernels, key=lambda k: k[2])
    peak, peak_kind = peaks()
    achieved = dom[1] / (dom[2] / 1000.0) / 1e9
    traffic, traffic_src = profiled_traffic(dom[0])

    # the bit-exact router order (one f32 chain per expert, as dot_f32_row):
    # the same calls with router_mode sequential, timed the same way
    seq_tokens = 64
    sgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(sgraph, stream=stream):
        for t in range(seq_tokens):
            tables[t % LAYERS][0].forward(xs[t], 1, outs[t], wss[t % LAYERS], router_mode=lbk.ROUTER_SEQUENTIAL,
                                          stream=stream.cuda_stream)
    for _ in range(3):
        sgraph.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s0.record(stream)
        for _ in range(5):
            sgraph.replay()
        s1.record(stream)
    torch.cuda.synchronize()
    seq_ms = s0.elapsed_time(s1) / (5 * seq_tokens)
    del sgraph
    ctx.raise_status(stream.cuda_stream)

    # e2e: per-token C-ABI calls, step inputs from pinned host, outputs read back
    x_host = torch.randn(TOKENS_PER_STEP, H, generator=torch.Generator().manual_seed(5 + rank)).pin_memory()
    o_host = torch.zeros(TOKENS_PER_STEP, H).pin_memory()
    e2e_steps = max(1, min(args.steps, 20))
    with torch.cuda.stream(stream):
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            xs.copy_(x_host, non_blocking=True)
            step_calls(stream)
            o_host.copy_(outs, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    e2e_ms = max(e0.elapsed_time(e1), wall * 1000.0)
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = e2e_steps * TOKENS_PER_STEP * world / (e2e_ms / 1000.0)
    ctx.raise_status(stream.cuda_stream)

    # expert parallelism at this N: config 4's layer step over the peer exchange
    ep_rec = None
    if not args.no_ep:
        ep_rec = ep_peer_measure(ctx, lbk, torch, dev, rank, world, min(args.steps, 50), 3)

    cpu = None
    if rank == 0 and world == 1 and host0 is not None and not args.no_cpu_baseline:
        cpu = cpu_baseline(host0, x_host.numpy()[:16])

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q8_k x packed (int8 dots, f32 tails)",
            "data": "synthetic (seeded, config shapes)",
            "config": {
                "workload": "config3: routed-MoE FFN layer, single-token decode",
                "hidden": H, "experts": E, "expert_ffn": F, "top_k": K_TOP,
                "gate_up": "IQ2_S", "down": "IQ3_S", "shared": "Q4_K",
                "router": "F32, tree order (the headline; logits within 1e-5 of the reference's sequential sum)",
                "tokens_per_step": TOKENS_PER_STEP, "resident_layers": LAYERS,
                "l2": f"inputs larger than L2: tokens rotate over {LAYERS} resident layers ({LAYERS * 1.3:.1f} GB)",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "algorithmic_bytes_per_token": LAYER_B,
            },
            "hbm_gbs_achieved": LAYER_B * tokens_total / (ms / 1000.0) / 1e9 / world,
            "kernel_ms": {"router_fused": avg[0], "moe_gate_up": avg[1], "moe_down": avg[2]},
            "roofline": {"bound": "hbm", "kernel": dom[0], "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic,
                         "traffic_source": f"stored ncu capture ({traffic_src}), not measured in this run"
                         if traffic_src else None,
                         "algorithmic_bytes_per_launch": dom[1]},
            "router_sequential": {"value": 1000.0 / seq_ms, "unit": "tokens/s", "us_per_token": seq_ms * 1000.0,
                                  "what": "the same layer calls with the bit-exact sequential router "
                                          "(one f32 chain per expert, dot_f32_row order)"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": TOKENS_PER_STEP * H * 4,
                    "d2h_bytes_per_step": TOKENS_PER_STEP * H * 4},
            "gpu_launches": args.steps * TOKENS_PER_STEP * 3,
            "clocks": clk,
            "cpu_baseline": cpu,
            "ep": ep_rec,
        }
        print(json.dumps(line), flush=True)
    del graph
    for layer, _ in tables:
        layer.close()
    ctx.close()


def profile_forwards(n: int) -> None:
    """A small case for ncu captures: one config-3 layer (1.3 GB) resident and
    n single-token forwards through the C ABI, tokens rotating over 8."""
    import torch

    import lbk

    ctx = lbk.Context(0)
    dev = torch.device("cuda", 0)
    tables, _ = build_layers(ctx, lbk, torch, dev, 1, 4, keep_gguf_layer0=False)
    layer = tables[0][0]
    ws = torch.zeros(layer.workspace_bytes(1), dtype=torch.uint8, device=dev)
    xs = torch.randn(8, H, device=dev, generator=torch.Generator(device=dev).manual_seed(5))
    out = torch.zeros(8, H, device=dev)
    for i in range(n):
        layer.forward(xs[i % 8], 1, out[i % 8], ws)
    torch.cuda.synchronize()
    ctx.raise_status()
    layer.close()
    ctx.close()
    print(f"profile_forwards: {n} forwards ok", flush=True)


def build_ep_layer(ctx, lbk, torch, dev, seed: int, first: int, count: int):
    """This rank's share of one config-3 layer (experts [first, first + count)),
    the whole router and shared expert, as an lbk.EpLayer."""
    import synth

    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    keep = []
    router = (torch.randn(E, H, device=dev, generator=gen) * 0.02).contiguous()
    keep.append(router)

    def planar(ty, k, rows, n):
        g = synth.packed_torch(gen, ty, k, rows * n, dev)
        mb, pb = synth.matrix_bytes(ty, k, rows), synth.planar_bytes(ty, k, rows)
        p = torch.empty(pb * n, dtype=torch.uint8, device=dev)
        for e in range(n):
            ctx.repack(lbk.matrix(ty, k, rows, g[e * mb:(e + 1) * mb]), p[e * pb:(e + 1) * pb])
        keep.append(p)
        return p, pb

    gp, mbg = planar(TYPE_IQ2_S, H, F, count)
    up, _ = planar(TYPE_IQ2_S, H, F, count)
    dp, mbd = planar(TYPE_IQ3_S, F, H, count)
    sh = [planar(ty, k, rows, 1)[0] for ty, k, rows in [(TYPE_Q4_K, H, F), (TYPE_Q4_K, H, F), (TYPE_Q4_K, F, H)]]
    torch.cuda.synchronize()
    experts = [
        lbk.Expert(lbk.matrix(TYPE_IQ2_S, H, F, gp[e * mbg:(e + 1) * mbg], lbk.LAYOUT_PLANAR),
                   lbk.matrix(TYPE_IQ2_S, H, F, up[e * mbg:(e + 1) * mbg], lbk.LAYOUT_PLANAR),
                   lbk.matrix(TYPE_IQ3_S, F, H, dp[e * mbd:(e + 1) * mbd], lbk.LAYOUT_PLANAR))
        for e in range(count)
    ]
    shared = lbk.Expert(*[lbk.matrix(ty, k, rows, p, lbk.LAYOUT_PLANAR)
                          for (ty, k, rows), p in zip([(TYPE_Q4_K, H, F), (TYPE_Q4_K, H, F), (TYPE_Q4_K, F, H)], sh)])
    bias = torch.zeros(E, device=dev)
    keep.append(bias)
    rm = lbk.Matrix(lbk.TYPE_F32, lbk.LAYOUT_GGUF, H, E, router.data_ptr(), router.numel() * 4)
    return lbk.EpLayer(ctx, experts, shared, rm, bias, K_TOP, WEIGHT_SCALE, E, first), keep


EP_LAYERS = 4  # config 4 through the peer exchange: resident EP layers a step rotates over


def ep_peer_measure(ctx, lbk, torch, dev, rank: int, world: int, steps: int, warmup: int, grouping=None,
                    tokens: int = BATCH_TOKENS) -> dict:
    """Config 4 through the peer-memory exchange (ep.PeerExpertParallelMoe):
    BATCH_TOKENS tokens per rank per layer step, experts sharded E / world per
    GPU, EP_LAYERS resident layers per rank so that a step's weights exceed
    L2 at every N (at N = 8, 24 experts are 160 MB per layer). One CUDA graph
    holds EP_LAYERS layer steps (no host work, no collective inside); timed
    with CUDA events, max over ranks. Then one pass with events between the
    stages of every layer step gives each stage's time (a stage's time on a
    rank includes its wait for the other ranks)."""
    import torch.distributed as dist

    import ep

    T = tokens
    er = E // world
    layers = [build_ep_layer(ctx, lbk, torch, dev, 4 + 1000 * rank + 17 * i, rank * er, er) for i in range(EP_LAYERS)]
    if grouping is not None:
        for L, _ in layers:
            L.set_grouping(grouping)
    stream = torch.cuda.Stream(device=dev)
    moe = ep.PeerExpertParallelMoe(layers[0][0], T, stream=stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + rank)
    xs = torch.randn(EP_LAYERS, T * H, device=dev, generator=gen)
    out = torch.empty(EP_LAYERS, T * H, device=dev)

    def step():
        for i, (L, _) in enumerate(layers):
            moe.forward(xs[i], T, out[i], layer=L)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[dev.index])

    stream.wait_stream(torch.cuda.current_stream())  # weights and inputs come from the default stream
    with torch.cuda.stream(stream):
        step()  # sets kernel attributes outside capture
    barrier()
    ctx.raise_status()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    barrier()
    for _ in range(warmup):
        graph.replay()
    barrier()
    ctx.raise_status()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
    barrier()
    ctx.raise_status()
    ms_layer = e0.elapsed_time(e1) / (steps * EP_LAYERS)

    # stage times: a second graph of one step with events recorded between the
    # stages (graph event nodes), replayed `passes` times
    names = ["route", "shared", "dispatch", "experts", "return", "combine"]
    acc = [0.0] * len(names)
    passes = 8
    evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(names) + 1)]
           for _ in range(EP_LAYERS)]
    items_seen = torch.zeros(EP_LAYERS, dtype=torch.int32, device=dev)  # the gathered count (the scatter resets it)
    sgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(sgraph, stream=stream):
        for i, (L, _) in enumerate(layers):
            ev = evs[i]
            ev[0].record(stream)
            moe.publish(xs[i], T, L)
            ev[1].record(stream)
            moe.shared(T, L)
            ev[2].record(stream)
            moe.dispatch(L)
            items_seen[i:i + 1].copy_(moe.count)
            ev[3].record(stream)
            moe.compute(L)
            ev[4].record(stream)
            moe.send_back(L)
            ev[5].record(stream)
            moe.combine(T, out[i], L, shared_done=True)
            ev[6].record(stream)
    barrier()
    for _ in range(passes):
        with torch.cuda.stream(stream):
            sgraph.replay()
        stream.synchronize()
        for ev in evs:
            for j in range(len(names)):
                acc[j] += ev[j].elapsed_time(ev[j + 1])
    del sgraph
    barrier()
    ctx.raise_status()
    stage_ms = [a / (passes * EP_LAYERS) for a in acc]
    items = int(items_seen[-1].item())
    t = torch.tensor([ms_layer] + stage_ms + [float(items > 0), float(items)], device=dev)
    if world > 1:
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = t.clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
    else:
        tmax = tsum = t
    ms_layer = float(tmax[0])
    stage_max = {n: float(tmax[1 + j]) for j, n in enumerate(names)}
    del graph
    moe.close()
    for L, _ in layers:
        L.close()
    return {
        "tokens_per_s": T * world / (ms_layer / 1000.0),
        "unit": f"tokens/s (layer steps of {T} tokens per GPU)",
        "ms_per_layer_step": ms_layer,
        "n_gpus": world,
        "gpus_active": int(tsum[1 + len(names)]),
        "experts_per_gpu": er,
        "pairs_per_gpu_mean": float(tsum[2 + len(names)]) / world,
        "stage_ms_max_over_ranks": stage_max,
        "dispatch_ms": stage_max["dispatch"],
        "return_ms": stage_max["return"],
        "limiter": max(stage_max, key=stage_max.get),
        "exchange": "peer memory over NVLink (CUDA IPC; plain peer loads and stores; step flags in the buffers, "
                    "no collective, no host read; one CUDA graph per step)",
        "stage_timing": "a second graph with event nodes between the stages, run one after another, with the "
                        "return as its own call (lbk_ep_scatter); the timed graph runs the shared expert on a "
                        "second stream, concurrent with dispatch and experts, and stores the experts' down rows "
                        "straight into the home buffers (lbk_ep_items_return); a stage's time includes its wait "
                        "for other ranks",
        "l2": f"{EP_LAYERS} resident layers per rank rotate within a step",
        "steps": steps,
    }


def batched_ep_arm(args, rank: int, world: int, local_rank: int) -> None:
    """Config 4: the routed-MoE layer on BATCH_TOKENS tokens per step per rank,
    experts sharded in contiguous ranges over the ranks (E / world each), the
    router and shared expert whole on every rank; dispatch and return of the
    routed pairs by NCCL all-to-all (ep.ExpertParallelMoe). Weak scaling: every
    rank is home to its own BATCH_TOKENS tokens."""
    import torch
    import torch.distributed as dist

    import ep
    import lbk

    T = BATCH_TOKENS
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = lbk.Context(local_rank)
    er = E // world
    if args.exchange == "peer":
        clocks = Clocks(local_rank)
        clocks.start()
        r = ep_peer_measure(ctx, lbk, torch, dev, rank, world, args.steps, args.warmup, args.grouping)
        clk = clocks.stop()
        if rank == 0:
            print(json.dumps({
                "metric": "routed-MoE batched tokens/s (config 4: 64 tokens per step per GPU, expert-parallel)",
                "value": r["tokens_per_s"],
                "unit": "tokens/s",
                "n_gpus": world,
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": r["ms_per_layer_step"],
                "higher_is_better": True,
                "scaling": "weak",
                "vs_baseline": None,
                "dtype": "q8_k x packed (int8 dots, f32 tails)",
                "data": "synthetic (seeded, config shapes)",
                "config": {"workload": "config4: routed-MoE FFN layer, 64 tokens per step per GPU", "hidden": H,
                           "experts": E, "experts_per_gpu": er, "expert_ffn": F, "top_k": K_TOP,
                           "tokens_per_step_per_gpu": T, "parallelism": f"expert-parallel x{world}",
                           "l2": r["l2"], "exchange": r["exchange"]},
                "ep": r,
                "gpu_launches": None,
                "clocks": clk,
            }), flush=True)
        ctx.close()
        return
    layer, keep = build_ep_layer(ctx, lbk, torch, dev, 4 + 1000 * rank, rank * er, er)
    if args.grouping is not None:
        layer.set_grouping(args.grouping)
    moe = ep.ExpertParallelMoe(layer)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + rank)
    xs = torch.randn(T * H, device=dev, generator=gen)
    out = torch.empty(T * H, device=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        moe.forward(xs, T, out)
    ctx.raise_status()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        moe.forward(xs, T, out)
    end.record()
    barrier()
    ctx.raise_status()
    ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        line = {
            "metric": "routed-MoE batched tokens/s (config 4: 64 tokens per step per GPU, expert-parallel)",
            "value": T * world / (ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q8_k x packed (int8 dots, f32 tails)",
            "data": "synthetic (seeded, config shapes)",
            "config": {"workload": "config4: routed-MoE FFN layer, 64 tokens per step per GPU", "hidden": H,
                       "experts": E, "experts_per_gpu": er, "expert_ffn": F, "top_k": K_TOP,
                       "tokens_per_step_per_gpu": T, "parallelism": f"expert-parallel x{world}",
                       "grouped_kernels": args.grouping is not None and args.grouping != 0,  # off by default for EP layers
                       "exchange": "NCCL all_to_all_single (counts, Q8_K rows, row dots)"},
        }
        print(json.dumps(line), flush=True)
    layer.close()
    ctx.close()


def batched_direct_arm(args, rank: int, world: int, local_rank: int) -> None:
    """Config 4's layer without expert parallelism: one lbk_moe_forward call of
    BATCH_TOKENS tokens per resident layer (all 192 experts on this GPU),
    rotating over LAYERS layers (larger than L2), one CUDA graph per step.
    With N > 1, N independent replicas (weak scaling)."""
    import torch

    import lbk

    T = BATCH_TOKENS
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = lbk.Context(local_rank)
    tables, _ = build_layers(ctx, lbk, torch, dev, LAYERS, 4 + 97 * rank, keep_gguf_layer0=False)
    if args.grouping is not None:
        for layer, _ in tables:
            layer.set_grouping(args.grouping)
    ws = torch.zeros(tables[0][0].workspace_bytes(T), dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + rank)
    xs = torch.randn(LAYERS, T * H, device=dev, generator=gen)
    outs = torch.zeros(LAYERS, T * H, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(s):
        for l, (layer, _) in enumerate(tables):
            layer.forward(xs[l], T, outs[l], ws, stream=s.cuda_stream)

    stream.wait_stream(torch.cuda.current_stream())  # weights and inputs come from the default stream
    with torch.cuda.stream(stream):
        step(stream)
        stream.synchronize()
        ctx.raise_status(stream.cuda_stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step(stream)
        for _ in range(args.warmup):
            graph.replay()
        stream.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        stream.synchronize()
    ctx.raise_status(stream.cuda_stream)
    ms = ev0.elapsed_time(ev1) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    if rank == 0:
        print(json.dumps({
            "metric": "routed-MoE batched tokens/s (config 4 layer, 64 tokens per call, all experts on one GPU)",
            "value": T * LAYERS * world / (ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q8_k x packed (int8 dots, f32 tails)",
            "data": "synthetic (seeded, config shapes)",
            "config": {"workload": f"config4 layer: {LAYERS} calls of {T} tokens per step, one per resident layer",
                       "hidden": H, "experts": E, "expert_ffn": F, "top_k": K_TOP, "tokens_per_call": T,
                       "us_per_call": ms * 1000.0 / LAYERS, "grouped_kernels": args.grouping != 0,
                       "parallelism": "single GPU" if world == 1 else f"replicas x{world}"},
        }), flush=True)
    del graph
    ctx.close()


def gemv_arm(args, cfg: int, rank: int, world: int, local_rank: int) -> None:
    """Configs 1-2: one quantized matvec y = W Q8_K(x) per call through
    lbk_gemv (planar layout). Config 1: Q4_K 4096 x 4096; config 2: IQ2_S and
    IQ3_S 6144 x 4096. Calls rotate over enough distinct weight copies that
    every call streams its matrix from HBM; a step is one call per copy,
    replayed as a CUDA graph. value = algorithmic bytes (W + x + y) / time."""
    import torch

    import lbk
    import synth

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = lbk.Context(local_rank)
    # config 1 adds the checkpoint's output projection (Q5_K, 120832 vocabulary rows)
    # config 2 adds a Hy3 block's attention projections (q, k: IQ2_S; v: Q4_K; output: IQ3_S over 8192)
    cases = [(TYPE_Q4_K, 4096, 4096), (TYPE_Q5_K, 4096, 120832)] if cfg == 1 else \
        [(TYPE_IQ2_S, 4096, 6144), (TYPE_IQ3_S, 4096, 6144), (TYPE_IQ2_S, 4096, 8192), (TYPE_IQ2_S, 4096, 1024),
         (TYPE_Q4_K, 4096, 1024), (TYPE_IQ3_S, 8192, 4096)]
    results = []
    for ty, k, rows in cases:
        gen = torch.Generator(device=dev)
        gen.manual_seed(cfg + 97 * rank)
        pb = synth.planar_bytes(ty, k, rows)
        copies = max(8, (320 << 20) // pb + 1)  # > 2.5 x L2 in total
        ws = []
        for _ in range(copies):
            g = synth.packed_torch(gen, ty, k, rows, dev)
            p = torch.empty(pb, dtype=torch.uint8, device=dev)
            ctx.repack(lbk.matrix(ty, k, rows, g), p)
            ws.append(p)
        mats = [lbk.matrix(ty, k, rows, p, lbk.LAYOUT_PLANAR) for p in ws]
        x = torch.randn(k, device=dev, generator=gen)
        y = torch.empty(rows, device=dev)
        q8 = torch.empty(k // 256 * 292, dtype=torch.uint8, device=dev)
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream())  # weights and inputs come from the default stream
        with torch.cuda.stream(stream):
            for m in mats:
                ctx.gemv(m, x, y, q8, stream=stream.cuda_stream)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for m in mats:
                    ctx.gemv(m, x, y, q8, stream=stream.cuda_stream)
            for _ in range(args.warmup):
                graph.replay()
            stream.synchronize()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record(stream)
            for _ in range(args.steps):
                graph.replay()
            en.record(stream)
            stream.synchronize()
        ctx.raise_status()
        us = st.elapsed_time(en) * 1000.0 / (args.steps * copies)
        alg = rows * row_bytes(ty, k) + k * 4 + rows * 4
        results.append({"type": {TYPE_Q4_K: "Q4_K", TYPE_Q5_K: "Q5_K", TYPE_IQ2_S: "IQ2_S", TYPE_IQ3_S: "IQ3_S"}[ty],
                        "rows": rows,
                        "input_width": k, "us_per_call": us, "gbs": alg / us / 1e3, "algorithmic_bytes": alg,
                        "copies": copies})
        del graph
    peak, kind = peaks()
    if rank == 0:
        head = results[0]
        line = {
            "metric": f"quantized GEMV HBM GB/s (config {cfg}: {head['type']} {head['rows']}x{head['input_width']})",
            "value": head["gbs"] * world,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": head["us_per_call"] * head["copies"] / 1000.0,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q8_k x packed (int8 dots, f32 tails)",
            "data": "synthetic (seeded, config shapes)",
            "config": {"workload": f"config{cfg}: single quantized matvec", "l2": "rotating over distinct weight copies (> L2)"},
            "roofline": {"bound": "hbm", "achieved": head["gbs"], "peak": peak, "unit": "GB/s", "frac": head["gbs"] / peak,
                         "peak_kind": kind},
            "cases": results,
        }
        print(json.dumps(line), flush=True)
    ctx.close()


def stack_ep_arm(args, rank: int, world: int, local_rank: int) -> None:
    """Config 5 over N GPUs: the STACK_LAYERS-layer stack with every layer's
    experts sharded E / N per GPU (24 on 8 GPUs), router and shared expert on
    every GPU. Every rank decodes its own args.batch tokens through all
    layers: hidden += MoE(RMSNorm(hidden)), the MoE step through the peer
    exchange (ep.PeerExpertParallelMoe: route, dispatch, experts, return,
    combine; one set of exchange buffers for all layers); one CUDA graph per
    step, no host work or collective inside. Weak scaling: N * batch tokens
    per step."""
    import torch
    import torch.distributed as dist

    import ep
    import lbk

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = lbk.Context(local_rank)
    B = args.batch
    er = E // world
    layers = [build_ep_layer(ctx, lbk, torch, dev, 4 + l + 1000 * rank, rank * er, er) for l in range(args.stack_layers)]
    if args.grouping is not None:
        for L, _ in layers:
            L.set_grouping(args.grouping)
    stream = torch.cuda.Stream(device=dev)
    moe = ep.PeerExpertParallelMoe(layers[0][0], B, stream=stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + rank)
    hidden = torch.randn(B * H, device=dev, generator=gen)
    normed = torch.empty(B * H, device=dev)
    delta = torch.empty(B * H, device=dev)
    norm_w = torch.ones(H, device=dev)

    def step():
        for L, _ in layers:
            ctx.rms_norm(hidden, norm_w, H, B, 1e-6, normed, mode=lbk.ROUTER_TREE, stream=stream.cuda_stream)
            moe.forward(normed, B, delta, layer=L)
            ctx.residual_add(hidden, delta, B * H, stream=stream.cuda_stream)

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    stream.wait_stream(torch.cuda.current_stream())  # weights and inputs come from the default stream
    with torch.cuda.stream(stream):
        step()
    barrier()
    ctx.raise_status()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    barrier()
    for _ in range(args.warmup):
        graph.replay()
    barrier()
    ctx.raise_status()
    clocks = Clocks(local_rank)
    clocks.start()
    time.sleep(0.3)
    barrier()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        st.record(stream)
        for _ in range(args.steps):
            graph.replay()
        en.record(stream)
    barrier()
    clk = clocks.stop()
    ctx.raise_status()
    ms = st.elapsed_time(en) / args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # weights a GPU streams per step: its experts touched by the step's pairs (at most all of its
    # E / N), the shared expert and the router, per layer
    per_expert = 2 * row_bytes(TYPE_IQ2_S, H) * F + row_bytes(TYPE_IQ3_S, F) * H
    shared_b = 2 * row_bytes(TYPE_Q4_K, H) * F + row_bytes(TYPE_Q4_K, F) * H
    touched = er * (1.0 - (1.0 - K_TOP / E) ** (B * world))
    bytes_step = args.stack_layers * (touched * per_expert + shared_b + E * H * 4)
    if rank == 0:
        print(json.dumps({
            "metric": f"routed-MoE stack decode tokens/s (config 5: {args.stack_layers} layers, batch {B} per GPU)",
            "value": B * world / (ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q8_k x packed (int8 dots, f32 tails)",
            "data": "synthetic (seeded, config shapes)",
            "config": {"workload": f"config5: {args.stack_layers}-layer stack, batch {B} per GPU, expert-parallel",
                       "layers": args.stack_layers, "batch_per_gpu": B, "experts_per_gpu": er,
                       "resident_gb_per_gpu": round(args.stack_layers * (er * per_expert + shared_b + E * H * 4) / 1e9, 1),
                       "us_per_layer_step": ms * 1000.0 / args.stack_layers,
                       "parallelism": f"expert-parallel x{world}",
                       "exchange": "peer memory over NVLink (ep.PeerExpertParallelMoe), one CUDA graph per step"},
            "hbm_gbs_per_gpu_expected_touched": bytes_step / (ms / 1000.0) / 1e9,
            "clocks": clk,
        }), flush=True)
    del graph
    moe.close()
    for L, _ in layers:
        L.close()
    ctx.close()


def stack_arm(args, rank: int, world: int, local_rank: int) -> None:
    """Config 5: a stack of STACK_LAYERS config-3 MoE blocks (attention
    omitted), per-layer random weights from seed 4 + layer, all HBM-resident
    (about 104 GB planar on one GPU). A step decodes args.batch tokens through
    every layer: hidden += MoE(RMSNorm(hidden)) per layer
    (lbk_moe_block_forward, the FFN half of a Hy3 block: the residual stream
    feeds the next layer), one CUDA graph per step. Token counts above one run
    the single-token kernels per (token, expert) pair."""
    import torch

    import lbk

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = lbk.Context(local_rank)
    B = args.batch
    layers = []
    for l in range(args.stack_layers):
        t, _ = build_layers(ctx, lbk, torch, dev, 1, 4 + l + 1000 * rank, keep_gguf_layer0=False)
        if args.grouping is not None:
            t[0][0].set_grouping(args.grouping)
        layers.append(t[0])
    ws = torch.zeros(layers[0][0].block_workspace_bytes(B), dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 + rank)
    hidden = torch.randn(B * H, device=dev, generator=gen)
    norm_w = torch.ones(H, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step(s):
        for layer, _ in layers:
            layer.block_forward(hidden, norm_w, 1e-6, B, ws, stream=s.cuda_stream)

    stream.wait_stream(torch.cuda.current_stream())  # weights and inputs come from the default stream
    with torch.cuda.stream(stream):
        step(stream)
        stream.synchronize()
        ctx.raise_status()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step(stream)
        for _ in range(args.warmup):
            graph.replay()
        stream.synchronize()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record(stream)
        for _ in range(args.steps):
            graph.replay()
        en.record(stream)
        stream.synchronize()
    ctx.raise_status()
    ms = st.elapsed_time(en) / args.steps
    if rank == 0:
        print(json.dumps({
            "metric": f"routed-MoE stack decode tokens/s (config 5: {args.stack_layers} layers, batch {B})",
            "value": B * world / (ms / 1000.0),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q8_k x packed (int8 dots, f32 tails)",
            "data": "synthetic (seeded, config shapes)",
            "config": {"workload": f"config5: {args.stack_layers}-layer stack, batch {B}", "layers": args.stack_layers,
                       "batch": B, "resident_gb": round(args.stack_layers * 1.3066, 1),
                       "grouped_kernels": B >= 2 and args.grouping != 0,
                       "us_per_layer_step": ms * 1000.0 / args.stack_layers,
                       "parallelism": "single GPU" if world == 1 else f"replicas x{world}"},
        }), flush=True)
    del graph
    ctx.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=1, help="config 5: tokens decoded per step")
    ap.add_argument("--stack-layers", type=int, default=80, help="config 5: layers in the stack")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5], default=3,
                    help="3: single-token decode (the headline); 4: 64 tokens per step per GPU, expert-parallel; "
                         "1, 2: single quantized matvec; 5: 80-layer stack")
    ap.add_argument("--direct", action="store_true",
                    help="config 4: all experts on every GPU, one lbk_moe_forward call per layer (no expert parallelism)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="config 4: expert-parallel exchange over peer memory (default) or NCCL all-to-all")
    ap.add_argument("--no-ep", action="store_true", help="config 3: skip the expert-parallel sub-record")
    ap.add_argument("--grouping", type=int, default=None,
                    help="configs 4, 5: token count from which the grouped kernels run (0: never; default: the library's)")
    ap.add_argument("--profile-forwards", type=int, default=0,
                    help="profiling driver: one resident layer, this many single-token forwards, no timing")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.profile_forwards > 0:
        profile_forwards(args.profile_forwards)
        return
    if args.impl == "reference":
        reference_arm(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if args.config == 4 and args.direct:
            batched_direct_arm(args, rank, world, local_rank)
        elif args.config == 4:
            batched_ep_arm(args, rank, world, local_rank)
        elif args.config in (1, 2):
            gemv_arm(args, args.config, rank, world, local_rank)
        elif args.config == 5 and world > 1:
            stack_ep_arm(args, rank, world, local_rank)
        elif args.config == 5:
            stack_arm(args, rank, world, local_rank)
        else:
            our_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
