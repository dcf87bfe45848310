"""Expert-parallel MoE layer across the GPUs of one node: a thin caller of libvfmoe.

The reference has no multi-GPU code; this is the expert-parallel form the task asks for.
- Tokens are sharded over ranks. Each rank routes its own tokens (router replicated) and runs
  the shared expert on them (shared expert replicated).
- The routed experts are sharded: rank r holds the (virtual) experts whose `placement[v] == r`,
  stacked in ascending id order (their local slots).  Hot experts may have copies
  (`replicated_placement`): virtual expert E + j holds expert hot[j]'s weights on another rank
  and takes that expert's lanes (t, l) with t + l odd.

The whole forward lives in the library (include/vfmoe.h, "expert parallelism inside the
library"): plan, pack, a fixed-capacity exchange (every peer block is t_cap entries, so no count
crosses to the host), the shared expert overlapping the exchange, the rank's experts on the
received rows (one fp16 partial row per entry), the exchange back and the combine.
- `EpComm`: the library's NCCL communicator (`vfmoe_ep_init`), bootstrapped by sharing the
  unique id over torch.distributed (or any other host channel).
- `EpLayer`: one rank's layer (`vfmoe_ep_set_placement`, workspace), `forward(comm, x)` =
  `vfmoe_ep_forward`, and the phase entry points for a caller's own transport.
- `ep_forward_virtual`: N virtual ranks in one process on one GPU, the blocks moved between their
  workspaces by device copies (tests the whole multi-rank data path on a single GPU).

Placement helpers (`balanced_placement`, `replicated_placement`, `local_slots`) are host logic
with no GPU work.
"""

from __future__ import annotations

import ctypes as C

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
    replica_of[j] goes to its copy n_experts + j when t + l is odd (the rule the library's plan
    kernel applies; lane parity splits an expert's lanes even at one token per rank).  idx int32
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
    T, k = idx.shape
    odd = ((torch.arange(T, device=dev)[:, None] + torch.arange(k, device=dev)[None, :]) % 2) == 1
    return torch.where((cand >= 0) & odd, cand, idx)


def local_slots(placement: np.ndarray) -> np.ndarray:
    """local_slot[e] = index of expert e among its owner's experts (ascending expert id)."""
    placement = np.asarray(placement)
    slot = np.empty_like(placement)
    for r in np.unique(placement):
        ids = np.nonzero(placement == r)[0]
        slot[ids] = np.arange(len(ids))
    return slot.astype(np.int32)


# ----------------------------------------------------------------------------- library EP
class EpComm:
    """NCCL communicator inside libvfmoe (one per process / GPU)."""

    def __init__(self, rank: int, world: int, unique_id: bytes, timeout_ms: int = 120000):
        from . import _lib
        self.lib = _lib.load()
        self.rank, self.world = rank, world
        buf = C.create_string_buffer(bytes(unique_id), 128)
        self.handle = _lib.check(self.lib.vfmoe_ep_init(world, rank, buf, timeout_ms))

    @staticmethod
    def unique_id() -> bytes:
        from . import _lib
        buf = C.create_string_buffer(128)
        _lib.check(_lib.load().vfmoe_ep_unique_id(buf, 128))
        return buf.raw

    @classmethod
    def from_torch_dist(cls, group=None, timeout_ms: int = 120000):
        """Rank 0 makes the unique id; torch.distributed carries it to the other ranks (the only
        use of torch.distributed here: the exchange itself is the library's NCCL)."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(rank, world, obj[0], timeout_ms)

    def close(self):
        if getattr(self, "handle", 0) > 0:
            self.lib.vfmoe_ep_destroy(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_BUF_NAMES = ["send_rows", "recv_rows", "rows_block", "send_slots", "recv_slots", "send_weights", "recv_weights",
              "lanes_block", "send_partials", "recv_partials", "partials_block", "send_counts"]


class EpLayer:
    """One rank's share of an expert-parallel MoE layer over libvfmoe.

    layer: a MoELayer holding the router (all E experts), the shared expert and this rank's
    (virtual) experts (n_local_experts); placement int32 [E + R] (owner rank per virtual
    expert); replica_of int32 [R] (copies); t_cap: capacity per rank, >= every rank's token
    count and equal on all ranks."""

    def __init__(self, layer, placement, rank: int, world: int, t_cap: int, replica_of=None):
        from . import _lib
        self._lib = _lib
        self.layer, self.rank, self.world, self.t_cap = layer, rank, world, t_cap
        pl = np.ascontiguousarray(np.asarray(placement, dtype=np.int32))
        rep = np.ascontiguousarray(np.asarray(replica_of if replica_of is not None else [], dtype=np.int32))
        self.placement, self.replica_of = pl, rep
        i32p = C.POINTER(C.c_int32)
        _lib.check(layer.lib.vfmoe_ep_set_placement(layer.handle, world, rank, pl.ctypes.data_as(i32p), len(pl),
                                                     rep.ctypes.data_as(i32p) if len(rep) else None, len(rep)))
        need = _lib.check(layer.lib.vfmoe_ep_workspace_bytes(layer.handle, t_cap))
        self.ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        offs = (C.c_int64 * 12)()
        _lib.check(layer.lib.vfmoe_ep_buffers(layer.handle, t_cap, offs, 12))
        self.buf = dict(zip(_BUF_NAMES, list(offs)))

    def _args(self):
        return int(self.ws.data_ptr()), self.ws.numel(), int(torch.cuda.current_stream().cuda_stream)

    def forward(self, comm: EpComm, x: torch.Tensor, out=None, idx=None, w=None):
        """This rank's tokens x [T, H] through the layer (vfmoe_ep_forward)."""
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.layer.H), dtype=self.layer.out_dtype, device=x.device)
        ws, nb, st = self._args()
        p = lambda t: 0 if t is None else int(t.data_ptr())  # noqa: E731
        self._lib.check(self.layer.lib.vfmoe_ep_forward(comm.handle, self.layer.handle, p(x), T, self.t_cap, p(out),
                                                        p(idx), p(w), ws, nb, st))
        return out

    # ---- phases (a caller's own transport moves the blocks between them)
    def prepare(self, x, idx=None, w=None):
        ws, nb, st = self._args()
        p = lambda t: 0 if t is None else int(t.data_ptr())  # noqa: E731
        self._lib.check(self.layer.lib.vfmoe_ep_prepare(self.layer.handle, p(x), x.shape[0], self.t_cap, p(idx), p(w),
                                                        ws, nb, st))

    def shared(self, x):
        ws, nb, st = self._args()
        self._lib.check(self.layer.lib.vfmoe_ep_shared(self.layer.handle, int(x.data_ptr()), x.shape[0], self.t_cap,
                                                       ws, nb, st))

    def experts(self):
        ws, nb, st = self._args()
        self._lib.check(self.layer.lib.vfmoe_ep_experts(self.layer.handle, self.t_cap, ws, nb, st))

    def combine(self, T: int, out=None):
        if out is None:
            out = torch.empty((T, self.layer.H), dtype=self.layer.out_dtype, device="cuda")
        ws, nb, st = self._args()
        self._lib.check(self.layer.lib.vfmoe_ep_combine(self.layer.handle, T, self.t_cap, int(out.data_ptr()), ws,
                                                        nb, st))
        return out

    def block(self, name: str, d: int) -> torch.Tensor:
        """Byte view of peer block d of an exchange buffer ("send_rows", "recv_slots", ...)."""
        size = self.buf[{"rows": "rows_block", "slots": "lanes_block", "weights": "lanes_block",
                         "partials": "partials_block"}[name.split("_", 1)[1]]]
        at = self.buf[name] + d * size
        return self.ws[at:at + size]

    def send_counts(self) -> torch.Tensor:
        at = self.buf["send_counts"]
        return self.ws[at:at + 4 * self.world].view(torch.int32)


def ep_forward_virtual(ranks, xs, outs=None):
    """N virtual ranks (EpLayer, one per rank, same t_cap) in one process on one GPU: the phases,
    with every peer block moved by a device copy where the NCCL exchange would move it."""
    N = len(ranks)
    for r, x in zip(ranks, xs):
        r.prepare(x)
    for kind in ("rows", "slots", "weights"):
        for s in range(N):
            for d in range(N):
                if s != d:
                    ranks[d].block("recv_" + kind, s).copy_(ranks[s].block("send_" + kind, d))
    for r, x in zip(ranks, xs):
        r.shared(x)
        r.experts()
    for s in range(N):
        for d in range(N):
            if s != d:
                ranks[d].block("recv_partials", s).copy_(ranks[s].block("send_partials", d))
    return [r.combine(x.shape[0], None if outs is None else outs[i]) for i, (r, x) in enumerate(zip(ranks, xs))]


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
