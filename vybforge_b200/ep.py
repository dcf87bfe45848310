"""Expert-parallel MoE layer across the GPUs of one node.

The reference has no multi-GPU code; this is the expert-parallel form the task asks for.
- Tokens are sharded over ranks. Each rank routes its own tokens (router replicated) and runs
  the shared expert on them (shared expert replicated).
- The routed experts are sharded: rank r holds the experts whose `placement[e] == r`, stacked
  in ascending expert order (their local slots).

One forward per rank, in three phases:
1. route -> `vfmoe_ep_plan` (stable sort of the (token, lane) pairs by owner rank) ->
   `vfmoe_ep_pack` (send rows + the owner's local slot ids).
2. exchange counts, then rows and slots (all-to-all-v). Then run `vfmoe_forward_rows` on the
   received rows plus this rank's own tokens for the shared expert.
3. all-to-all-v the expert outputs back, then `vfmoe_combine`.

The GPU compute is libvfmoe. The all-to-all is a `Transport`:
- `DistTransport`: torch.distributed over NCCL (NVLink/NVSwitch), or gloo on CPU.
- `VirtualTransport`: N virtual ranks held by one process. The whole multi-rank data path
  (plans, packing, per-rank expert sets, exchange order) then runs on one GPU.
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


def balanced_placement(load, n_ranks: int) -> np.ndarray:
    """Load-aware placement with exactly E/n_ranks experts per rank: experts in descending
    load order go to the least-loaded rank that still has room (greedy bin packing)."""
    load = np.asarray(load, dtype=np.float64)
    E = load.shape[0]
    if E % n_ranks:
        raise ValueError("n_experts must be divisible by n_ranks")
    cap = E // n_ranks
    owner = np.empty(E, dtype=np.int32)
    tot = np.zeros(n_ranks)
    room = np.full(n_ranks, cap)
    for e in np.argsort(-load, kind="stable"):
        r = min((r for r in range(n_ranks) if room[r] > 0), key=lambda r: (tot[r], r))
        owner[e] = r
        tot[r] += load[e]
        room[r] -= 1
    return owner


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
        recv = torch.empty((sum(recv_splits),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        self.dist.all_to_all_single(recv, send, output_split_sizes=recv_splits, input_split_sizes=send_splits,
                                    group=self.group)
        return recv


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

    `backend` provides: route(x) -> (idx, w); plan(idx) -> (send_counts, send_perm, inv_perm);
    pack(x, idx, send_perm) -> (rows, slots); rows(rows, slots) -> y fp32;
    combine(y_back, inv_perm, w, T, y_shared) -> out.  `GpuBackend` is the libvfmoe one.
    """

    def __init__(self, rank: int, world: int, backend):
        self.rank, self.world, self.b = rank, world, backend

    def phase1(self, x):
        idx, w = self.b.route(x)
        counts, perm, inv = self.b.plan(idx)
        rows, slots = self.b.pack(x, idx, perm)
        return dict(x=x, idx=idx, w=w, counts=counts, perm=perm, inv=inv, rows=rows, slots=slots)

    def phase2(self, st, recv_rows, recv_slots):
        x = st["x"]
        T = x.shape[0]
        n_recv = recv_rows.shape[0]
        rows_all = torch.cat([recv_rows, x.to(recv_rows.dtype)]) if T else recv_rows
        shared = torch.full((T,), self.b.shared_slot, dtype=recv_slots.dtype, device=recv_slots.device)
        y_all = self.b.rows(rows_all, torch.cat([recv_slots, shared]))
        st["y_shared"] = y_all[n_recv:]
        return y_all[:n_recv]

    def phase3(self, st, y_back):
        T = st["x"].shape[0]
        return self.b.combine(y_back, st["inv"], st["w"], T, st["y_shared"])


def ep_forward_dist(rank_state: EpRank, x, transport: DistTransport):
    """Expert-parallel forward of this process's tokens (one rank per process)."""
    st = rank_state.phase1(x)
    recv_splits, send_splits = transport.counts(st["counts"])
    recv_rows = transport.rows(st["rows"], send_splits, recv_splits)
    recv_slots = transport.rows(st["slots"], send_splits, recv_splits)
    y_recv = rank_state.phase2(st, recv_rows, recv_slots)
    y_back = transport.rows(y_recv, recv_splits, send_splits)
    return rank_state.phase3(st, y_back)


def ep_forward_virtual(ranks, xs, transport: VirtualTransport):
    """Expert-parallel forward of N virtual ranks held by this process."""
    sts = [r.phase1(x) for r, x in zip(ranks, xs)]
    recv_splits, send_splits = transport.counts_all([s["counts"] for s in sts])
    recv_rows = transport.rows_all([s["rows"] for s in sts], send_splits, recv_splits)
    recv_slots = transport.rows_all([s["slots"] for s in sts], send_splits, recv_splits)
    y_recv = [r.phase2(s, rr, rs) for r, s, rr, rs in zip(ranks, sts, recv_rows, recv_slots)]
    y_back = transport.rows_all(y_recv, recv_splits, send_splits)
    return [r.phase3(s, yb) for r, s, yb in zip(ranks, sts, y_back)]


# ----------------------------------------------------------------------------- GPU backend
class GpuBackend:
    """libvfmoe kernels for one rank: a MoELayer holding the router (all E experts), the
    shared expert and this rank's routed experts (n_local_experts)."""

    def __init__(self, layer, placement, n_ranks: int, out_dtype=torch.bfloat16):
        from . import moe
        self.moe = moe
        self.layer = layer
        self.E = layer.E
        self.n_ranks = n_ranks
        self.placement = torch.as_tensor(np.asarray(placement, np.int32)).cuda()
        self.local_slot = torch.as_tensor(local_slots(placement)).cuda()
        self.shared_slot = layer.n_local
        self.out_dtype = out_dtype

    def route(self, x):
        return self.layer.route(x)

    def plan(self, idx):
        return self.moe.ep_plan(idx, self.E, self.placement, self.n_ranks)

    def pack(self, x, idx, perm):
        return self.moe.ep_pack(x, idx, perm, self.local_slot)

    def rows(self, rows, slots):
        return self.layer.forward_rows(rows, slots)

    def combine(self, y_back, inv, w, T, y_shared):
        return self.moe.combine(y_back, inv, w, T, self.layer.k, y_shared=y_shared, out_dtype=self.out_dtype)


def rank_experts(dev, placement, rank: int):
    """Stacked Q8_0 matrices of the experts `rank` owns (ascending expert id) from full
    [E+1, rows, bytes] stacks (last = shared).  Returns (gate, up, down, shared tuple)."""
    E = len(placement)
    ids = torch.as_tensor(np.nonzero(np.asarray(placement) == rank)[0], device=dev[0].device)
    return (dev[0][ids].contiguous(), dev[1][ids].contiguous(), dev[2][ids].contiguous(),
            (dev[0][E], dev[1][E], dev[2][E]))
