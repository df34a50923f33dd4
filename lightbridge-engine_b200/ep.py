"""Expert-parallel routed-MoE layer over torch.distributed, one process per GPU.

Experts are sharded in contiguous ranges: with E global experts over `world`
ranks, rank r holds global experts [r * E_r, (r + 1) * E_r), E_r = E / world
(24 per GPU for 192 experts on 8 GPUs). The router and the shared expert are
whole on every rank. Each rank owns its own tokens (their home rank). One
layer step for a home rank's T tokens:

1. route (lbk_ep_route): the top-k routing in ascending expert-ID order and
   the tokens' Q8_K images, on the home rank;
2. dispatch: every (token, slot) pair travels to the rank owning its expert as
   one row [Q8_K image | local expert ID]; the per-peer counts go first (an
   all-to-all of `world` integers), then the rows (all_to_all_single with those
   splits);
3. items_forward (lbk_ep_items_forward) on every rank over the rows it
   received: the raw row dots down(SwiGLU(gate, up)) of each item;
4. return: the dots travel back with the splits reversed and land at
   routed_dots[t * k + j];
5. combine (lbk_ep_combine) on the home rank: the coefficient-weighted sum in
   ascending expert-ID order, then the shared expert, the one-GPU order of
   moe_routed_by_id_into's accept pass (bridge-kernels-reference/src/moe.rs:116-147),
   so the output is bit-identical to lbk_moe_forward on one GPU.

Partial sums are never all-reduced across ranks: that would change the f32
summation order. The reference runs every expert of a layer on one host
(bridge-runtime/src/hy3_scalar.rs:561-628); this module has no counterpart
there.

The compute stages are the methods of `layer` (lbk.EpLayer on a GPU: route,
items_forward, combine, q8_bytes, workspace_bytes). Every rank takes the same
collective steps in the same order, also with no tokens of its own or no items
to compute.

Two exchanges implement steps 2 and 4:
- ExpertParallelMoe: NCCL all-to-all; the per-peer counts are read on the
  host to size the row exchange (one device-to-host read per layer step).
  Works wherever torch.distributed does.
- PeerExpertParallelMoe: the ranks of one node map each other's exchange
  buffers (CUDA IPC) and move only the pairs' bytes with plain peer loads and
  stores; the counts stay on the device and the ranks order a step through
  flags in the buffers, so a step has no collective and no host read and can
  be captured in a CUDA graph. This is the exchange the benchmark uses.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

# bytes after the Q8_K image in a dispatch row: the local expert ID (int32),
# padded so that rows keep the image's 16-byte alignment
ROW_HEADER_BYTES = 16


@dataclass
class DispatchPlan:
    """Where the (token, slot) pairs of one home rank go.

    order: pair indices (t * k + j) sorted by owning rank, stable, so each
    peer's rows keep ascending pair order; send / recv: rows per peer."""

    order: torch.Tensor
    owner: torch.Tensor
    send: list[int]
    recv: list[int]


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _owners(ids: torch.Tensor, experts_per_rank: int, world: int):
    owner = ids.to(torch.int64) // experts_per_rank
    order = torch.argsort(owner, stable=True)
    send = torch.bincount(owner, minlength=world)
    if send.numel() != world:
        raise ValueError(f"routed expert ID beyond {world} ranks x {experts_per_rank} experts")
    return owner, order, send


def local_plan(ids: torch.Tensor, experts_per_rank: int, world: int) -> DispatchPlan:
    """The plan without a count exchange (recv = send): for one process that
    hands every rank's rows out itself."""
    owner, order, send = _owners(ids, experts_per_rank, world)
    s = send.cpu().tolist()
    return DispatchPlan(order, owner, s, list(s))


def plan_dispatch(ids: torch.Tensor, experts_per_rank: int, world: int, group=None) -> DispatchPlan:
    """Owner rank of every routed pair and the per-peer row counts (one
    all-to-all of `world` counts, then one device-to-host read of 2 * world
    integers for the split sizes of the row exchanges)."""
    owner, order, send = _owners(ids, experts_per_rank, world)
    recv = torch.empty_like(send)
    if world > 1:
        dist.all_to_all_single(recv, send, group=group)
    else:
        recv.copy_(send)
    counts = torch.cat([send, recv]).cpu().tolist()
    return DispatchPlan(order, owner, counts[:world], counts[world:])


def pack_rows(q8: torch.Tensor, ids: torch.Tensor, plan: DispatchPlan, k: int, experts_per_rank: int) -> torch.Tensor:
    """Dispatch rows in plan order: [Q8_K image of the pair's token | local
    expert ID (int32) | zero pad]."""
    n = plan.order.numel()
    q8b = q8.shape[1]
    rows = torch.zeros((n, q8b + ROW_HEADER_BYTES), dtype=torch.uint8, device=q8.device)
    if n == 0:
        return rows
    rows[:, :q8b] = q8.index_select(0, plan.order // k)
    local = (ids.to(torch.int64).index_select(0, plan.order) - plan.owner.index_select(0, plan.order) * experts_per_rank)
    rows[:, q8b:q8b + 4] = local.to(torch.int32).unsqueeze(1).view(torch.uint8)
    return rows


def unpack_items(rows: torch.Tensor, q8_bytes: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Received rows -> (contiguous Q8_K images [n][q8_bytes], lbk_routed items
    [n][2] int32 with the local expert ID and a zero coefficient)."""
    n = rows.shape[0]
    q8_items = rows[:, :q8_bytes].contiguous()
    items = torch.zeros((n, 2), dtype=torch.int32, device=rows.device)
    if n:
        items[:, 0] = rows[:, q8_bytes:q8_bytes + 4].contiguous().view(torch.int32).view(-1)
    return q8_items, items


def exchange(rows: torch.Tensor, send: list[int], recv: list[int], world: int, group=None) -> torch.Tensor:
    """all_to_all_single of `rows` (first dimension split by `send`) into a new
    tensor split by `recv`; a copy on one rank."""
    out = rows.new_empty((sum(recv),) + tuple(rows.shape[1:]))
    if world > 1:
        dist.all_to_all_single(out, rows, output_split_sizes=recv, input_split_sizes=send, group=group)
    else:
        out.copy_(rows)
    return out


def place_returned(back: torch.Tensor, plan: DispatchPlan, pairs: int, hidden: int) -> torch.Tensor:
    """Returned dots (plan order) -> routed_dots [pairs][hidden] in pair order."""
    routed_dots = back.new_empty((pairs, hidden))
    if pairs:
        routed_dots.index_copy_(0, plan.order, back)
    return routed_dots


class ExpertParallelMoe:
    """One rank of an expert-parallel MoE layer.

    layer: this rank's compute stages (lbk.EpLayer), holding the global
    experts [rank * E_r, (rank + 1) * E_r). group: the process group of the
    expert-parallel ranks (None: the default group; one rank without
    torch.distributed)."""

    def __init__(self, layer, group=None):
        self.layer = layer
        self.group = group
        self.world, self.rank = _world(group)
        E = layer.global_experts
        if E % self.world:
            raise ValueError(f"{E} experts do not shard evenly over {self.world} ranks")
        self.experts_per_rank = E // self.world
        if layer.local_experts != self.experts_per_rank or layer.first_expert != self.rank * self.experts_per_rank:
            raise ValueError(
                f"rank {self.rank} must hold experts [{self.rank * self.experts_per_rank}, "
                f"{(self.rank + 1) * self.experts_per_rank}), has [{layer.first_expert}, "
                f"{layer.first_expert + layer.local_experts})"
            )
        self._ws = None

    def workspace(self, count: int, device) -> torch.Tensor:
        """A zero-filled workspace for `count` tokens or items, grown on demand
        and reused (one zero fill at creation keeps it valid for every count)."""
        need = self.layer.workspace_bytes(max(count, 1))
        if self._ws is None or self._ws.numel() < need or self._ws.device != torch.device(device):
            self._ws = torch.zeros(need, dtype=torch.uint8, device=device)
        return self._ws

    def forward(self, x: torch.Tensor, tokens: int, out: torch.Tensor, routed_out: torch.Tensor | None = None) -> None:
        """out[tokens * hidden] = the MoE layer on this rank's tokens x[tokens *
        hidden]. Collective: every rank of the group calls it once per layer
        step, with tokens >= 0."""
        L = self.layer
        k, H, q8b = L.top_k, L.hidden, L.q8_bytes
        dev = x.device
        routed = torch.empty((tokens * k, 2), dtype=torch.int32, device=dev)
        q8 = torch.empty((tokens, q8b), dtype=torch.uint8, device=dev)
        if tokens:
            L.route(x, tokens, routed, q8, self.workspace(tokens, dev))
        ids = routed[:, 0]
        plan = plan_dispatch(ids, self.experts_per_rank, self.world, self.group)
        rows = exchange(pack_rows(q8, ids, plan, k, self.experts_per_rank), plan.send, plan.recv, self.world, self.group)
        n = rows.shape[0]
        dots = torch.empty((n, H), dtype=torch.float32, device=dev)
        if n:
            q8_items, items = unpack_items(rows, q8b)
            L.items_forward(q8_items, items, n, dots, self.workspace(n, dev))
        back = exchange(dots, plan.recv, plan.send, self.world, self.group)
        routed_dots = place_returned(back, plan, tokens * k, H)
        if tokens:
            L.combine(q8, tokens, routed, routed_dots, out, self.workspace(tokens, dev))
        if routed_out is not None and tokens:
            routed_out.view(torch.int32).view(-1)[: tokens * k * 2].copy_(routed.view(-1))


class PeerExpertParallelMoe:
    """One rank of an expert-parallel MoE layer whose exchange runs over peer
    memory (NVLink) instead of collectives: every rank's exchange buffer is
    mapped into every other rank (lbk.PeerBuffer, plain peer loads and stores),
    the home rank publishes its routing and Q8_K images there, every rank
    gathers the pairs of its experts and scatters their row dots back into the
    home buffers, and the home rank combines (lbk_ep_publish / gather /
    items_forward_counted / scatter / combine_exchange). The ranks order a
    step among themselves through flags in the buffers, so a layer step has no
    collective, no size exchange and no device-to-host read, and can be
    captured in a CUDA graph. Results equal lbk_moe_forward on one GPU bit for
    bit (the combine order is the one-GPU order).

    cap: the most tokens any rank brings to a step. Every rank of the group
    calls forward once per layer step (a rank without tokens too). The
    constructor and close() are collective over the process group."""

    def __init__(self, layer, cap: int, group=None, stream=None, overlap_shared: bool = True):
        import lbk

        self.layer = layer
        self.group = group
        self.stream = stream  # a raw CUDA stream handle, or None for torch's current stream
        self.overlap_shared = overlap_shared
        self.world, self.rank = _world(group)
        E = layer.global_experts
        if E % self.world:
            raise ValueError(f"{E} experts do not shard evenly over {self.world} ranks")
        self.experts_per_rank = E // self.world
        if layer.local_experts != self.experts_per_rank or layer.first_expert != self.rank * self.experts_per_rank:
            raise ValueError(f"rank {self.rank} holds the wrong share of the experts")
        self.cap = cap
        self.x = layer.exchange_layout(cap)
        self.buf = lbk.PeerBuffer(layer.ctx, self.x.total)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.buf.handle, group=group)
            ptrs = [self.buf.ptr if r == self.rank else self.buf.open(handles[r]) for r in range(self.world)]
        else:
            ptrs = [self.buf.ptr]
        dev = torch.device("cuda", torch.cuda.current_device())
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        k, H, q8b = layer.top_k, layer.hidden, layer.q8_bytes
        self.cap_items = self.world * cap * k
        self.q8_items = torch.empty((self.cap_items, q8b), dtype=torch.uint8, device=dev)
        self.items = torch.zeros((self.cap_items, 2), dtype=torch.int32, device=dev)
        self.returns = torch.zeros(self.cap_items, dtype=torch.int64, device=dev)
        self.count = torch.zeros(1, dtype=torch.int32, device=dev)
        self.dots = torch.empty((self.cap_items, H), dtype=torch.float32, device=dev)
        self.ws = torch.zeros(layer.workspace_bytes(max(self.cap_items, cap)), dtype=torch.uint8, device=dev)
        # the shared expert on a second stream, concurrent with the exchange
        self.shared_dots = torch.empty((cap, H), dtype=torch.float32, device=dev)
        self.ws_shared = torch.zeros(layer.workspace_bytes(cap), dtype=torch.uint8, device=dev)
        self.side = torch.cuda.Stream(device=dev)
        self._ev_pub = torch.cuda.Event()
        self._ev_shared = torch.cuda.Event()
        self._ext = torch.cuda.ExternalStream(stream, device=dev) if stream is not None else None
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=group)  # every buffer mapped and zeroed before any rank's first step

    # The stages of one layer step; `layer` (default: the constructor's) may be
    # any EpLayer of the same shapes and expert share, so that one set of
    # buffers serves every layer of a stack. Each stage runs on the main stream.
    def _main(self):
        s = self._ext if self._ext is not None else torch.cuda.current_stream()
        return s.cuda_stream, s

    def publish(self, x: torch.Tensor, tokens: int, layer=None) -> None:
        (layer or self.layer).publish(x, tokens, self.buf.ptr, self.cap, self.ws, stream=self._main()[0])

    def dispatch(self, layer=None) -> None:
        """Gather this rank's pairs from every buffer (waits for every publication)."""
        (layer or self.layer).gather(self.peers, self.world, self.rank, self.cap, self.q8_items, self.items,
                                     self.returns, self.count, stream=self._main()[0])

    def compute(self, layer=None) -> None:
        (layer or self.layer).items_forward_counted(self.q8_items, self.items, self.count, self.dots, self.ws,
                                                    stream=self._main()[0])

    def send_back(self, layer=None) -> None:
        (layer or self.layer).scatter(self.peers, self.world, self.rank, self.cap, self.dots, self.returns,
                                      self.count, stream=self._main()[0])

    def compute_return(self, layer=None) -> None:
        """compute and send_back in one: the down rows stored in the home buffers."""
        (layer or self.layer).items_return(self.peers, self.world, self.rank, self.cap, self.q8_items, self.items,
                                           self.returns, self.count, self.ws, stream=self._main()[0])

    def shared(self, tokens: int, layer=None) -> None:
        """The shared expert of the published tokens into shared_dots."""
        (layer or self.layer).shared(self.buf.ptr, self.cap, tokens, self.shared_dots, self.ws_shared,
                                     stream=self._main()[0])

    def combine(self, tokens: int, out: torch.Tensor | None, layer=None, shared_done: bool = False) -> None:
        """Waits for every rank's dots, then combines this rank's tokens into
        out (the shared expert computed here unless shared_done)."""
        (layer or self.layer).combine_exchange(self.buf.ptr, self.world, self.cap, tokens, out, self.ws,
                                               shared_dots=self.shared_dots if shared_done and tokens else None,
                                               stream=self._main()[0])

    def forward(self, x: torch.Tensor, tokens: int, out: torch.Tensor | None, layer=None) -> None:
        """out[tokens * hidden] = the MoE layer on this rank's tokens (tokens <= cap).
        With overlap_shared the shared expert runs on a second stream between
        the publication and the combine (a fork and a join, also under CUDA
        graph capture)."""
        if tokens > self.cap:
            raise ValueError(f"{tokens} tokens beyond the exchange capacity {self.cap}")
        L = layer or self.layer
        self.publish(x, tokens, L)
        side = self.overlap_shared and tokens > 0
        if side:
            main = self._main()[1]
            self._ev_pub.record(main)
            self.side.wait_event(self._ev_pub)
            L.shared(self.buf.ptr, self.cap, tokens, self.shared_dots, self.ws_shared, stream=self.side.cuda_stream)
            self._ev_shared.record(self.side)
        self.dispatch(L)
        self.compute_return(L)
        if side:
            main.wait_event(self._ev_shared)
        self.combine(tokens, out, L, shared_done=side)

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers before any buffer is freed."""
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
            self.buf.close_opened()
            dist.barrier(group=self.group)
        self.buf.close()
