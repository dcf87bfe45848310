"""Expert-parallel protocol on CPU: the library's fixed-capacity exchange (include/vfmoe.h,
vfmoe_ep_*) restated in numpy (tests/ep_protocol.py) and run on 2 gloo ranks and on N virtual
ranks, end to end against the single-device oracle; plus the host-side placement logic of
vybforge_b200/ep.py and the C ABI's argument checks of the expert-parallel entry points (no GPU
work).  The CUDA kernels of the same steps are compared with this restatement, bit for bit, in
tests/test_gpu_ep.py."""

import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import ep, synth

from helpers import run_ranks, guarded

import ep_protocol as proto


def _setup(world):
    cfg = synth.config("c0", tokens=24)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    experts = synth.expert_q8_numpy(cfg, rng)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    load = np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts)
    placement = ep.balanced_placement(load, world)
    return cfg, x, w_r, bias, experts, placement


def _reference(cfg, x, w_r, bias, experts):
    H, I, E = cfg.hidden, cfg.inter, cfg.n_experts

    def mats(e):
        return (orc.q8_0_expert_inout(experts[0][e], I, H), orc.q8_0_expert_inout(experts[1][e], I, H),
                orc.q8_0_expert_inout(experts[2][e], H, I))
    out, _, _ = orc.moe_block_grouped(x, w_r, bias, mats, lambda: mats(E), E, cfg.topk)
    return out


def test_placements():
    load = np.array([100, 1, 50, 2, 30, 3, 20, 4])
    p = ep.balanced_placement(load, 2)
    assert np.bincount(p).tolist() == [4, 4]
    tot = [load[p == r].sum() for r in range(2)]
    assert max(tot) - min(tot) <= 40
    assert ep.contiguous_placement(8, 4).tolist() == [0, 0, 1, 1, 2, 2, 3, 3]
    assert ep.local_slots(np.array([1, 0, 1, 0])).tolist() == [0, 0, 1, 1]


def test_replicated_placement_and_split():
    cfg = synth.config("c4p")
    E, W = cfg.n_experts, 8
    # expected selection counts of a C4-prefill layer (Zipf(1.1), T = 8192, top-8)
    load = np.round(synth.zipf_targets(E, cfg.tokens, cfg.topk, cfg.zipf_s, np.random.default_rng(3)))
    pv, hot = ep.replicated_placement(load, W)
    assert pv.shape == (E + W,) and np.bincount(pv).tolist() == [(E + W) // W] * W
    cost = load + 1.4 * 128 * np.ceil(load / 128)
    assert sorted(hot.tolist()) == sorted(np.argsort(-cost, kind="stable")[:W].tolist())
    assert all(pv[h] != pv[E + j] for j, h in enumerate(hot))      # each copy on another rank

    def tile_cost(ld):                                              # prefill work per expert
        return np.ceil(ld / 128) * 752 + np.ceil(ld / 256) * 562

    def spread(placement, ld):
        per = np.array([tile_cost(ld)[placement == r].sum() for r in range(W)])
        return per.max() / per.mean()
    vload = np.concatenate([load, np.zeros(W)])
    vload[hot] = load[hot] / 2
    vload[E:] = load[hot] / 2
    assert spread(pv, vload) < spread(ep.balanced_placement(load, W), load) - 0.05
    # split: lanes (t, l) of a replicated expert with t + l odd move to its copy, nothing else changes
    idx = torch.tensor([[int(hot[0]), 5], [int(hot[0]), 6], [7, int(hot[1])], [8, int(hot[1])]], dtype=torch.int32)
    got = ep.split_replicas(idx, hot, E)
    want = idx.clone()
    want[1, 0] = E + 0
    want[2, 1] = E + 1
    assert torch.equal(got, want)
    assert torch.equal(ep.split_replicas(idx, np.zeros(0, np.int32), E), idx)


class NumpyRank:
    """One rank of the protocol with the oracle's f64 arithmetic (test infrastructure)."""

    def __init__(self, cfg, w_r, bias, experts, owner, replica_of, rank, world, cap):
        self.cfg, self.w_r, self.bias = cfg, w_r, bias
        self.owner, self.replica_of = np.asarray(owner), np.asarray(replica_of, dtype=np.int64)
        self.rank, self.world, self.cap = rank, world, cap
        E, H, I = cfg.n_experts, cfg.hidden, cfg.inter
        self.mine = np.nonzero(self.owner == rank)[0]             # virtual ids of the local slots

        def mats(e):
            return (orc.q8_0_expert_inout(experts[0][e], I, H), orc.q8_0_expert_inout(experts[1][e], I, H),
                    orc.q8_0_expert_inout(experts[2][e], H, I))

        def real(v):
            return int(v) if v < E else int(self.replica_of[v - E])
        self.mats = [mats(real(v)) for v in self.mine]
        self.shared = mats(E)

    def prepare(self, x):
        idx, w = orc.route(x, self.w_r, self.bias, self.cfg.topk)
        counts, tok, slot, wt, pos = proto.plan(idx, w.astype(np.float32), self.owner, self.replica_of,
                                                self.cfg.n_experts, self.world, self.cap)
        rows = np.zeros((self.world, self.cap, x.shape[1]), dtype=np.float64)
        for d in range(self.world):
            rows[d, :counts[d]] = x[tok[d, :counts[d]]]
        self.x, self.pos = x, pos
        return rows, slot, wt

    def experts(self, rows, slot, wt):
        H = rows.shape[-1]
        y = proto.expert_partials(rows.reshape(-1, H), slot.reshape(-1, slot.shape[-1]),
                                  wt.reshape(-1, wt.shape[-1]), lambda s, r: orc.ffn(r, *self.mats[s]))
        return y.reshape(self.world, self.cap, H)

    def combine(self, y_back):
        y_shared = orc.ffn(self.x, *self.shared)
        return proto.combine(y_back.reshape(-1, y_back.shape[-1]), self.pos, y_shared)


def _virtual_forward(ranks, xs):
    """N ranks in one process: block d of rank s's send buffers becomes block s of rank d's."""
    N = len(ranks)
    sent = [r.prepare(x) for r, x in zip(ranks, xs)]
    recv = [tuple(np.stack([sent[s][b][d] for s in range(N)]) for b in range(3)) for d in range(N)]
    ys = [r.experts(*rv) for r, rv in zip(ranks, recv)]
    back = [np.stack([ys[s][d] for s in range(N)]) for d in range(N)]
    return [r.combine(b) for r, b in zip(ranks, back)]


def test_plan_restatement_small_case():
    """Two ranks, expert 1 copied (virtual 4 on rank 0): lanes (t, l) with t + l odd of expert 1
    go to the copy; entries per destination in token order; padding carries no lanes."""
    idx = np.array([[1, 0], [1, 2], [3, 1]], dtype=np.int32)
    w = np.array([[0.5, 0.25], [1.0, 2.0], [3.0, 4.0]], dtype=np.float32)
    owner = np.array([0, 1, 1, 0, 0])              # experts 0..3, virtual 4 = copy of expert 1
    counts, tok, slot, wt, pos = proto.plan(idx, w, owner, [1], 4, 2, 4)
    # virtual ids: t0 [1, 0]; t1 [4 (t+l = 1), 2]; t2 [3, 4 (t+l = 3)]
    # owners:      t0 [1, 0]; t1 [0, 1];            t2 [0, 0]
    assert counts.tolist() == [3, 2]
    assert tok[0].tolist() == [0, 1, 2, -1] and tok[1].tolist() == [0, 1, -1, -1]
    # local slots: rank 0 owns virtual 0, 3, 4 -> slots 0, 1, 2; rank 1 owns 1, 2 -> 0, 1
    assert slot[0, 0].tolist() == [-1, 0] and slot[1, 0].tolist() == [0, -1]
    assert slot[0, 1].tolist() == [2, -1] and slot[1, 1].tolist() == [-1, 1]
    assert slot[0, 2].tolist() == [1, 2]
    assert (slot[0, 3] == -1).all() and (slot[1, 2:] == -1).all()
    assert pos.tolist() == [[0, 4], [1, 5], [2, -1]]
    assert wt[0, 2].tolist() == [3.0, 4.0] and wt[1, 1].tolist() == [0.0, 2.0]


@pytest.mark.parametrize("world,replicas", [(2, False), (4, False), (2, True), (4, True)])
def test_virtual_ranks_match_single_device_oracle(world, replicas):
    cfg, x, w_r, bias, experts, placement = _setup(world)
    hot = np.zeros(0, np.int32)
    if replicas:
        idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
        placement, hot = ep.replicated_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    shards = np.array_split(np.arange(cfg.tokens), world)
    cap = max(len(s) for s in shards)
    ranks = [NumpyRank(cfg, w_r, bias, experts, placement, hot, r, world, cap) for r in range(world)]
    outs = _virtual_forward(ranks, [x[s] for s in shards])
    got = np.concatenate(outs)
    np.testing.assert_allclose(got, _reference(cfg, x, w_r, bias, experts), rtol=0, atol=1e-6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_body(rank, world, port):
    """One rank per process; the fixed-size blocks cross with gloo all-to-alls of equal splits,
    exactly the transfers vfmoe_ep_forward makes with NCCL send/recv."""
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, x, w_r, bias, experts, placement = _setup(world)
        shards = np.array_split(np.arange(cfg.tokens), world)
        cap = max(len(s) for s in shards)
        r = NumpyRank(cfg, w_r, bias, experts, placement, np.zeros(0, np.int32), rank, world, cap)

        def a2a(blocks):
            t = torch.from_numpy(np.ascontiguousarray(blocks))
            out = torch.empty_like(t)
            dist.all_to_all_single(out, t)
            return out.numpy()
        rows, slot, wt = r.prepare(x[shards[rank]])
        y = r.experts(a2a(rows), a2a(slot), a2a(wt))
        return r.combine(a2a(y))
    finally:
        dist.destroy_process_group()


_gloo_worker = guarded(_gloo_body)


def test_two_gloo_ranks_match_single_device_oracle():
    world = 2
    res = run_ranks(_gloo_worker, world, timeout=300)
    cfg, x, w_r, bias, experts, placement = _setup(world)
    got = np.concatenate([res[r] for r in range(world)])
    np.testing.assert_allclose(got, _reference(cfg, x, w_r, bias, experts), rtol=0, atol=1e-6)


def _abi_body(rank, world, port):
    """The expert-parallel entry points through ctypes on a CPU-only rank: argument checks answer
    before any device work, and a communicator cannot be made without a GPU (a status, no abort)."""
    from vybforge_b200 import _lib
    lib = _lib.load()
    bad = lib.vfmoe_ep_init(0, 0, None, 0)
    none = lib.vfmoe_ep_forward(12345, 67890, 0, 0, 1, 0, 0, 0, 0, 0, 0)
    buf = (C.c_char * 128)()
    rc = lib.vfmoe_ep_init(world, rank, buf, 1000)
    return bad, none, rc


_abi_worker = guarded(_abi_body)


def test_ep_abi_status_codes_on_cpu_ranks():
    from vybforge_b200 import _lib
    res = run_ranks(_abi_worker, 2, timeout=120)
    for rank in range(2):
        bad, none, rc = res[rank]
        assert bad == _lib.ERR_INVALID
        assert none == _lib.ERR_HANDLE
        assert rc in (_lib.ERR_CUDA, _lib.ERR_NCCL)   # no device here: a status, not a crash
