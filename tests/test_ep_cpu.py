"""Expert-parallel orchestration on CPU: 2 gloo ranks (and N virtual ranks) whose per-rank
compute is the numpy oracle, checked end to end against the single-device oracle.  This
covers the host logic of vybforge_b200/ep.py (placement, send plan, pack order, all-to-all
splits, combine) without a GPU; the CUDA kernels of the same steps are covered by
tests/test_gpu_ep.py."""

import os
import socket

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import ep, synth

from helpers import run_ranks, guarded


class NumpyBackend:
    """Oracle compute for one rank (test infrastructure only), in the token-level exchange
    protocol of ep.EpRank: plan / pack / experts / combine restated in numpy."""

    def __init__(self, cfg, w_r, bias, experts, placement, rank, replica_of=()):
        self.cfg, self.w_r, self.bias = cfg, w_r, bias
        self.placement = np.asarray(placement)
        self.n_ranks = len(np.unique(self.placement))
        self.local = ep.local_slots(placement)
        self.my = np.nonzero(self.placement == rank)[0]          # (virtual) ids of local slots
        self.shared_slot = len(self.my)
        self.k = cfg.topk
        self.partial_dtype = torch.float64
        H, I, E = cfg.hidden, cfg.inter, cfg.n_experts

        def mats(e):
            return (orc.q8_0_expert_inout(experts[0][e], I, H), orc.q8_0_expert_inout(experts[1][e], I, H),
                    orc.q8_0_expert_inout(experts[2][e], H, I))
        def real(e):                                             # copy E + j holds replica_of[j]
            return int(e) if e < E else int(replica_of[e - E])
        self.mats = {int(e): mats(real(e)) for e in self.my}
        self.mats[-1] = mats(E)                                  # shared

    def route(self, x):
        idx, w = orc.route(x.numpy().astype(np.float64), self.w_r, self.bias, self.k)
        return torch.from_numpy(idx.astype(np.int32)), torch.from_numpy(w.astype(np.float32))

    def plan(self, idx, w):
        idx, w = idx.numpy(), w.numpy()
        T, k, R = idx.shape[0], self.k, self.n_ranks
        owner = self.placement[idx]
        tok, slot, sw = [], [], []
        pos = np.full((T, R), -1, dtype=np.int32)
        counts = np.zeros(R, dtype=np.int32)
        for r in range(R):
            for t in range(T):
                mine = owner[t] == r
                if mine.any():
                    pos[t, r] = len(tok)
                    tok.append(t)
                    slot.append(np.where(mine, self.local[idx[t]], -1))
                    sw.append(np.where(mine, w[t], 0.0))
                    counts[r] += 1
        n = len(tok)
        return (torch.from_numpy(counts), torch.tensor(tok, dtype=torch.int32),
                torch.from_numpy(np.array(slot, dtype=np.int32).reshape(n, k)),
                torch.from_numpy(np.array(sw, dtype=np.float32).reshape(n, k)), torch.from_numpy(pos))

    def pack(self, x, tok, n):
        return x[tok[:n].long()]

    def experts(self, rows, slots, w):
        r = rows.numpy().astype(np.float64)
        s, wv = slots.numpy(), w.numpy().astype(np.float64)
        y = np.zeros_like(r)
        for l in range(s.shape[1]):
            for sl in np.unique(s[:, l]):
                if sl < 0:
                    continue
                sel = s[:, l] == sl
                key = -1 if sl == self.shared_slot else int(self.my[sl])
                y[sel] += wv[sel, l:l + 1] * orc.ffn(r[sel], *self.mats[key])
        return torch.from_numpy(y)

    def combine(self, y_back, pos, T, y_shared):
        yb, p = y_back.numpy(), pos.numpy()
        out = y_shared.numpy().copy()
        for t in range(T):
            for r in range(p.shape[1]):
                if p[t, r] >= 0:
                    out[t] += yb[p[t, r]]
        return torch.from_numpy(out)


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
    # split: the odd tokens' lanes of a replicated expert move to its copy, nothing else changes
    idx = torch.tensor([[int(hot[0]), 5], [int(hot[0]), 6], [7, int(hot[1])], [8, int(hot[1])]], dtype=torch.int32)
    got = ep.split_replicas(idx, hot, E)
    want = idx.clone()
    want[1, 0] = E + 0
    want[3, 1] = E + 1
    assert torch.equal(got, want)
    assert torch.equal(ep.split_replicas(idx, np.zeros(0, np.int32), E), idx)


@pytest.mark.parametrize("world", [2, 4])
def test_virtual_ranks_with_replicas_match_single_device_oracle(world):
    cfg, x, w_r, bias, experts, _ = _setup(world)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    pv, hot = ep.replicated_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    shards = np.array_split(np.arange(cfg.tokens), world)
    ranks = [ep.EpRank(r, world, NumpyBackend(cfg, w_r, bias, experts, pv, r, replica_of=hot), replica_of=hot,
                       n_experts=cfg.n_experts) for r in range(world)]
    outs = ep.ep_forward_virtual(ranks, [torch.from_numpy(x[s]) for s in shards], ep.VirtualTransport(world))
    got = np.concatenate([o.numpy() for o in outs])
    np.testing.assert_allclose(got, _reference(cfg, x, w_r, bias, experts), rtol=0, atol=1e-6)


@pytest.mark.parametrize("world", [2, 4])
def test_virtual_ranks_match_single_device_oracle(world):
    cfg, x, w_r, bias, experts, placement = _setup(world)
    shards = np.array_split(np.arange(cfg.tokens), world)
    ranks = [ep.EpRank(r, world, NumpyBackend(cfg, w_r, bias, experts, placement, r)) for r in range(world)]
    outs = ep.ep_forward_virtual(ranks, [torch.from_numpy(x[s]) for s in shards], ep.VirtualTransport(world))
    got = np.concatenate([o.numpy() for o in outs])
    ref = _reference(cfg, x, w_r, bias, experts)
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-6)  # routing weights are fp32, as on the GPU


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_body(rank, world, port):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, x, w_r, bias, experts, placement = _setup(world)
        shard = np.array_split(np.arange(cfg.tokens), world)[rank]
        r = ep.EpRank(rank, world, NumpyBackend(cfg, w_r, bias, experts, placement, rank))
        out = ep.ep_forward_dist(r, torch.from_numpy(x[shard]), ep.DistTransport())
        return out.numpy()
    finally:
        dist.destroy_process_group()


_gloo_worker = guarded(_gloo_body)


def test_two_gloo_ranks_match_single_device_oracle():
    world = 2
    res = run_ranks(_gloo_worker, world, timeout=300)
    cfg, x, w_r, bias, experts, placement = _setup(world)
    got = np.concatenate([res[r] for r in range(world)])
    np.testing.assert_allclose(got, _reference(cfg, x, w_r, bias, experts), rtol=0, atol=1e-6)
