"""Expert-parallel MoE layer across the GPUs of one node.

The reference has no multi-GPU code; this is the expert-parallel form the task asks for.
- Tokens are sharded over ranks. Each rank routes its own tokens (router replicated) and runs
  the shared expert on them (shared expert replicated).
- The routed experts are sharded: rank r holds the experts whose `placement[e] == r`, stacked
  in ascending expert order (their local slots).

Token-level exchange, one forward per rank in three phases:
1. route -> `vfmoe_ep_plan_tokens`: one send entry per (token, destination rank) that owns
   at least one of the token's experts, carrying the token's k lanes as (owner-local slot
   or -1, weight) -> `vfmoe_ep_pack` gathers the send rows.
2. exchange counts, then rows and lane metadata (all-to-all-v). While the rows are in
   flight, `vfmoe_forward_routed` runs the shared expert on this rank's own tokens; then on
   the received rows, summing each row's local lanes with their weights: one fp16 partial
   row per entry.
3. all-to-all-v the partial rows back; `vfmoe_combine` adds, per token, the partials from
   each rank (rank order) and the shared expert's row.
A token whose experts live on m ranks crosses the links m times each way, instead of k times
(once per (token, expert) pair), and the return rows are fp16 partial sums.

The GPU compute is libvfmoe. The all-to-all is a `Transport`:
- `DistTransport`: torch.distributed over NCCL (NVLink/NVSwitch), or gloo on CPU.
- `VirtualTransport`: N virtual ranks held by one process. The whole multi-rank data path
  (plans, packing, per-rank expert sets, exchange order) then runs on one GPU.

Hot experts can be replicated (`replicated_placement`, `split_replicas`): a copy on a second
rank takes the odd tokens' lanes, so no rank carries a whole hottest expert.
"""

from __future__ import annotations

import numpy as np
import torch


# ----------------------------------------------------------------------------- placement
def contiguous_placement(n_experts: int, n_ranks: int) -> np.ndarray:
    """Expert e -> rank e // (E / n_ranks)."""
    if n_experts % n_ranks:
        raise ValueError("n_experts must be divisible by n_ranks")
    return (np.arange(n_experts) // (n_experts // n_ranks)).astype(np.int32)


def balanced_placement(load, n_ranks: int, tile_rows: int = 128, tile_cost: float = 1.4) -> np.ndarray:
    """Load-aware placement with exactly E/n_ranks experts per rank: experts in descending
    cost order go to the least-loaded rank that still has room (greedy bin packing).

    cost(e) = rows(e) + tile_cost * tile_rows * ceil(rows(e) / tile_rows): an expert's prefill
    GEMM pays per token tile for streaming and dequantizing its weights, whatever the tile's
    row count, so many cold experts cost more than their rows suggest.  tile_cost = 0 is a
    balance of rows alone."""
    load = np.asarray(load, dtype=np.float64)
    E = load.shape[0]
    if E % n_ranks:
        raise ValueError("n_experts must be divisible by n_ranks")
    cost = load + tile_cost * tile_rows * np.ceil(load / tile_rows)
    cap = E // n_ranks
    owner = np.empty(E, dtype=np.int32)
    tot = np.zeros(n_ranks)
    room = np.full(n_ranks, cap)
    for e in np.argsort(-cost, kind="stable"):
        r = min((r for r in range(n_ranks) if room[r] > 0), key=lambda r: (tot[r], r))
        owner[e] = r
        tot[r] += cost[e]
        room[r] -= 1
    return owner


def replicated_placement(load, n_ranks: int, n_replicas: int | None = None, tile_rows: int = 128,
                         tile_cost: float = 1.4):
    """Placement of E + R virtual experts in which the R most expensive experts have a copy.

    Virtual expert E + j is a copy of expert hot[j]; `split_replicas` sends the lanes of hot[j]
    from odd-numbered tokens to the copy, so each copy carries about half of the expert's rows.
    A prefill work item costs about the same whatever its row count, so an expert's cost grows
    with its token tiles, and the rank holding the hottest expert caps an 8-GPU step however
    the rest is packed; splitting that expert removes the cap.  Copies go to the least-loaded
    rank other than their sibling's (greedy bin packing as balanced_placement, each rank
    holding exactly (E + R) / n_ranks virtual experts).
    Returns (placement int32 [E + R], replica_of int32 [R]).  R defaults to n_ranks."""
    load = np.asarray(load, dtype=np.float64)
    E = load.shape[0]
    R = n_ranks if n_replicas is None else int(n_replicas)
    if R < 0 or R > E or (E + R) % n_ranks:
        raise ValueError("n_experts + n_replicas must be divisible by n_ranks")
    cost = load + tile_cost * tile_rows * np.ceil(load / tile_rows)
    hot = np.argsort(-cost, kind="stable")[:R].astype(np.int32)
    vload = np.concatenate([load, np.zeros(R)])
    sibling = np.full(E + R, -1, dtype=np.int64)
    for j, h in enumerate(hot):
        vload[h] = vload[E + j] = load[h] / 2
        sibling[h], sibling[E + j] = E + j, h
    vcost = vload + tile_cost * tile_rows * np.ceil(vload / tile_rows)
    cap = (E + R) // n_ranks
    owner = np.full(E + R, -1, dtype=np.int32)
    tot = np.zeros(n_ranks)
    room = np.full(n_ranks, cap)
    for v in np.argsort(-vcost, kind="stable"):
        avoid = owner[sibling[v]] if sibling[v] >= 0 else -1
        cands = [r for r in range(n_ranks) if room[r] > 0 and r != avoid]
        if not cands:  # only the sibling's rank has room left: both halves on one rank
            cands = [r for r in range(n_ranks) if room[r] > 0]
        r = min(cands, key=lambda r: (tot[r], r))
        owner[v] = r
        tot[r] += vcost[v]
        room[r] -= 1
    return owner, hot


def split_replicas(idx: torch.Tensor, replica_of, n_experts: int) -> torch.Tensor:
    """Routing ids over the virtual experts of replicated_placement: lane (t, l) of expert
    replica_of[j] goes to its copy n_experts + j when the token index t is odd.  idx int32
    [T, k] (any device).  The weights are unchanged: the combined output is the same sum, its
    partials possibly added in another rank order."""
    R = len(replica_of)
    if R == 0:
        return idx
    dev = idx.device
    copy_of = torch.full((n_experts,), -1, dtype=torch.int32, device=dev)
    copy_of[torch.as_tensor(np.asarray(replica_of), dtype=torch.long, device=dev)] = torch.arange(
        n_experts, n_experts + R, dtype=torch.int32, device=dev)
    cand = copy_of[idx.long()]
    odd = (torch.arange(idx.shape[0], device=dev) % 2 == 1)[:, None]
    return torch.where((cand >= 0) & odd, cand, idx)


def local_slots(placement: np.ndarray) -> np.ndarray:
    """local_slot[e] = index of expert e among its owner's experts (ascending expert id)."""
    placement = np.asarray(placement)
    slot = np.empty_like(placement)
    for r in np.unique(placement):
        ids = np.nonzero(placement == r)[0]
        slot[ids] = np.arange(len(ids))
    return slot.astype(np.int32)


# ----------------------------------------------------------------------------- transports
class DistTransport:
    """All-to-all(v) through torch.distributed (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def counts(self, send_counts):
        """send_counts: int tensor [world] -> recv_counts python list (host sync)."""
        out = torch.empty_like(send_counts)
        self.dist.all_to_all_single(out, send_counts, group=self.group)
        return out.tolist(), send_counts.tolist()

    def rows(self, send, send_splits, recv_splits):
        recv, work = self.rows_async(send, send_splits, recv_splits)
        work.wait()
        return recv

    def rows_async(self, send, send_splits, recv_splits):
        """Start the exchange on the collective stream; work.wait() orders later work on the
        current stream after it.  Work enqueued meanwhile overlaps the transfer."""
        recv = torch.empty((sum(recv_splits),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        work = self.dist.all_to_all_single(recv, send, output_split_sizes=recv_splits, input_split_sizes=send_splits,
                                           group=self.group, async_op=True)
        return recv, work


class VirtualTransport:
    """N ranks held by one process: a collective is a gather over the per-rank inputs."""

    def __init__(self, world: int):
        self.world = world

    def counts_all(self, send_counts_per_rank):
        sc = [c.tolist() for c in send_counts_per_rank]
        recv = [[sc[src][dst] for src in range(self.world)] for dst in range(self.world)]
        return recv, sc

    def rows_all(self, sends, send_splits, recv_splits):
        parts = [list(torch.split(s, sp)) for s, sp in zip(sends, send_splits)]
        return [torch.cat([parts[src][dst] for src in range(self.world)]) for dst in range(self.world)]


# ----------------------------------------------------------------------------- one rank
class EpRank:
    """One rank's share of an expert-parallel MoE layer.

    `backend` provides:
      route(x) -> (idx, w)
      plan(idx, w) -> (send_counts, send_tok, send_slot, send_w, pos_of)   (token-level plan)
      pack(x, send_tok, n) -> rows
      experts(rows, slots, w) -> partial rows (fp16): sum of the weighted local lanes
      (also the shared expert: one lane with slot shared_slot, weight 1)
      combine(y_back, pos_of, T, y_shared) -> out
      shared_slot, k
    `GpuBackend` is the libvfmoe one.  With replica_of (replicated_placement), the backend's
    placement covers the E + R virtual experts and its layer holds the local ones.
    """

    def __init__(self, rank: int, world: int, backend, replica_of=None, n_experts: int = 0):
        self.rank, self.world, self.b = rank, world, backend
        # replicated experts (replicated_placement): the routing ids are split over the copies
        self.replica_of = np.asarray(replica_of if replica_of is not None else [], dtype=np.int32)
        self.n_experts = n_experts

    def phase1(self, x):
        idx, w = self.b.route(x)
        if len(self.replica_of):
            idx = split_replicas(idx, self.replica_of, self.n_experts)
        counts, tok, slot, sw, pos = self.b.plan(idx, w)
        return dict(x=x, counts=counts, tok=tok, slot=slot, sw=sw, pos=pos)

    def pack(self, st, n: int):
        """Send rows and lane metadata of the n valid entries (n = sum of the send counts)."""
        st["rows"] = self.b.pack(st["x"], st["tok"], n)
        # lane metadata as one int32 tensor [n, 2k]: slots, then the weights' bits
        st["meta"] = torch.cat([st["slot"][:n], st["sw"][:n].view(torch.int32)], dim=1)

    def shared(self, st):
        """The shared expert on this rank's own tokens (weight 1, one lane)."""
        x = st["x"]
        T = x.shape[0]
        own_s = torch.full((T, 1), self.b.shared_slot, dtype=torch.int32, device=x.device)
        own_w = torch.ones((T, 1), dtype=torch.float32, device=x.device)
        st["y_shared"] = self.b.experts(x, own_s, own_w)

    def phase2(self, st, recv_rows, recv_meta):
        k = self.b.k
        if recv_rows.shape[0] == 0:
            return torch.empty((0, st["x"].shape[1]), dtype=self.b.partial_dtype, device=st["x"].device)
        slots, wts = recv_meta[:, :k], recv_meta[:, k:].view(torch.float32)
        return self.b.experts(recv_rows, slots.contiguous(), wts.contiguous())

    def phase3(self, st, y_back):
        T = st["x"].shape[0]
        return self.b.combine(y_back, st["pos"], T, st["y_shared"])


def ep_forward_dist(rank_state: EpRank, x, transport: DistTransport, mark=None):
    """Expert-parallel forward of this process's tokens (one rank per process).
    mark(name), if given, is called after each phase (e.g. to record CUDA events)."""
    mark = mark or (lambda name: None)
    st = rank_state.phase1(x)
    mark("route_plan")
    recv_splits, send_splits = transport.counts(st["counts"])
    mark("counts")
    rank_state.pack(st, sum(send_splits))
    mark("pack")
    # the shared expert on this rank's tokens runs while the rows are in flight
    recv_rows, w_rows = transport.rows_async(st["rows"], send_splits, recv_splits)
    recv_meta, w_meta = transport.rows_async(st["meta"], send_splits, recv_splits)
    rank_state.shared(st)
    mark("shared")
    w_rows.wait()
    w_meta.wait()
    mark("dispatch")
    y_recv = rank_state.phase2(st, recv_rows, recv_meta)
    mark("experts")
    y_back = transport.rows(y_recv, recv_splits, send_splits)
    mark("return")
    out = rank_state.phase3(st, y_back)
    mark("combine")
    return out


def ep_forward_virtual(ranks, xs, transport: VirtualTransport):
    """Expert-parallel forward of N virtual ranks held by this process."""
    sts = [r.phase1(x) for r, x in zip(ranks, xs)]
    recv_splits, send_splits = transport.counts_all([s["counts"] for s in sts])
    for r, s, sp in zip(ranks, sts, send_splits):
        r.pack(s, sum(sp))
    recv_rows = transport.rows_all([s["rows"] for s in sts], send_splits, recv_splits)
    recv_meta = transport.rows_all([s["meta"] for s in sts], send_splits, recv_splits)
    for r, s in zip(ranks, sts):
        r.shared(s)
    y_recv = [r.phase2(s, rr, rm) for r, s, rr, rm in zip(ranks, sts, recv_rows, recv_meta)]
    y_back = transport.rows_all(y_recv, recv_splits, send_splits)
    return [r.phase3(s, yb) for r, s, yb in zip(ranks, sts, y_back)]


# ----------------------------------------------------------------------------- GPU backend
class GpuBackend:
    """libvfmoe kernels for one rank: a MoELayer holding the router (all E experts), the
    shared expert and this rank's routed experts (n_local_experts)."""

    def __init__(self, layer, placement, n_ranks: int, out_dtype=torch.bfloat16, partial_dtype=torch.float16):
        from . import moe
        self.moe = moe
        self.layer = layer
        self.E, self.k = len(placement), layer.k  # routed ids, copies of replicated experts included
        self.n_ranks = n_ranks
        self.placement = torch.as_tensor(np.asarray(placement, np.int32)).cuda()
        self.local_slot = torch.as_tensor(local_slots(placement)).cuda()
        self.shared_slot = layer.n_local
        self.out_dtype = out_dtype
        self.partial_dtype = partial_dtype

    def route(self, x):
        return self.layer.route(x)

    def plan(self, idx, w):
        return self.moe.ep_plan_tokens(idx, w, self.E, self.placement, self.local_slot, self.n_ranks)

    def pack(self, x, tok, n):
        return self.moe.gather_rows(x, tok, n)

    def experts(self, rows, slots, w):
        return self.layer.forward_routed(rows, slots, w, y_dtype=self.partial_dtype)

    def combine(self, y_back, pos, T, y_shared):
        return self.moe.combine(y_back, pos.reshape(-1), None, T, self.n_ranks, y_shared=y_shared,
                                out_dtype=self.out_dtype)


def rank_experts(dev, placement, rank: int, replica_of=None):
    """Stacked Q8_0 matrices of the experts `rank` owns (ascending expert id) from full
    [E+1, rows, bytes] stacks (last = shared).  With replica_of, placement covers E + R
    virtual experts and copy E + j holds expert replica_of[j]'s weights.
    Returns (gate, up, down, shared tuple)."""
    P = np.asarray(placement)
    R = 0 if replica_of is None else len(replica_of)
    E = len(P) - R
    v = np.nonzero(P == rank)[0]
    real = v.copy()
    if R:
        real[v >= E] = np.asarray(replica_of)[v[v >= E] - E]
    ids = torch.as_tensor(real, device=dev[0].device)
    return (dev[0][ids].contiguous(), dev[1][ids].contiguous(), dev[2][ids].contiguous(),
            (dev[0][E], dev[1][E], dev[2][E]))
