"""Expert parallelism on the GPU through the library's entry points (include/vfmoe.h, vfmoe_ep_*).

* The plan and pack kernels against the numpy restatement of the protocol (tests/ep_protocol.py),
  bit for bit: counts, lane slots and weights of every block, packed rows.
* N virtual ranks in one process on one GPU: the library's phases with the blocks moved by
  device copies; against the fused single-GPU forward.
* vfmoe_ep_forward over a 1-rank NCCL communicator (the full NCCL path without peers), eager
  and recorded in a CUDA graph.
* A communicator whose second rank never joins: vfmoe_ep_init gives up after its limit with
  VFMOE_ERR_NCCL (host-side failure; no kernel runs).
* 2 processes x 2 GPUs over NCCL, when two GPUs are visible.
"""

import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import _lib, ep, moe, synth
from vybforge_b200.moe import MoELayer, quantizer

import ep_protocol as proto
from helpers import rel_l2, run_ranks, guarded

pytestmark = pytest.mark.gpu


def _weights(cfg, rng):
    if cfg.name == "c0":
        ex = synth.expert_q8_numpy(cfg, rng)
        return {p: torch.from_numpy(ex[p]).cuda() for p in range(3)}
    return synth.expert_q8_cuda(cfg, quantizer)


def _kw(cfg, w_r, bias, out_dtype):
    return dict(hidden=cfg.hidden, inter=cfg.inter, n_experts=cfg.n_experts, topk=cfg.topk,
                router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                x_dtype=torch.bfloat16 if cfg.x_dtype == "bf16" else torch.float32, out_dtype=out_dtype)


def _full(cfg, dev, w_r, bias, out_dtype):
    E = cfg.n_experts
    return MoELayer(gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E], shared=(dev[0][E], dev[1][E], dev[2][E]),
                    **_kw(cfg, w_r, bias, out_dtype))


def _ep_layers(cfg, dev, w_r, bias, placement, world, cap, out_dtype, replica_of=None):
    out = []
    for r in range(world):
        g, u, d, sh = ep.rank_experts(dev, placement, r, replica_of)
        L = MoELayer(gate=g, up=u, down=d, shared=sh, n_local_experts=len(placement) // world,
                     **_kw(cfg, w_r, bias, out_dtype))
        out.append(ep.EpLayer(L, placement, r, world, cap, replica_of))
    return out


def _xdev(cfg, x):
    return (torch.from_numpy(x).to(torch.bfloat16) if cfg.x_dtype == "bf16" else torch.from_numpy(x)).cuda()


# fp32 output: fp32 partial rows, only the lane sums reassociate (1e-4); bf16 output: fp16 partial
# rows and bf16 rounding of the sum, against the single-GPU bf16 output (a few ulp flips).
@pytest.mark.parametrize("cfg_name,world,T,out", [("c0", 4, 48, "f32"), ("c1", 2, 16, "f32"), ("c1", 8, 64, "f32"),
                                                  ("c1", 8, 64, "bf16")])
def test_virtual_ranks_match_single_gpu(cfg_name, world, T, out):
    moe.init(0)
    cfg = synth.config(cfg_name, tokens=T)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    dev = _weights(cfg, rng)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    placement = ep.balanced_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    odt = torch.float32 if out == "f32" else torch.bfloat16
    xd = _xdev(cfg, x)
    ref = _full(cfg, dev, w_r, bias, odt).forward(xd).float().cpu().numpy()
    shards = np.array_split(np.arange(T), world)
    cap = max(len(s) for s in shards)
    ranks = _ep_layers(cfg, dev, w_r, bias, placement, world, cap, odt)
    outs = ep.ep_forward_virtual(ranks, [xd[s[0]:s[-1] + 1].contiguous() for s in shards])
    got = torch.cat(outs).float().cpu().numpy()
    for r in ranks:
        r.layer.check_device_error()
    d = rel_l2(got, ref)
    print(f"[ep virtual {cfg_name} N={world} T={T} out {out}] rel-L2 vs single GPU {d:.3e}")
    assert d < (1e-4 if out == "f32" else 2e-3)


@pytest.mark.parametrize("world", [2, 8])
def test_virtual_ranks_with_replicated_experts_match_single_gpu(world):
    """The hottest experts copied to a second rank; lanes (t, l) with t + l odd go to the copy."""
    moe.init(0)
    cfg = synth.config("c1", tokens=64)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    dev = synth.expert_q8_cuda(cfg, quantizer)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    pv, hot = ep.replicated_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    xd = _xdev(cfg, x)
    ref = _full(cfg, dev, w_r, bias, torch.float32).forward(xd).cpu().numpy()
    shards = np.array_split(np.arange(cfg.tokens), world)
    cap = max(len(s) for s in shards)
    ranks = _ep_layers(cfg, dev, w_r, bias, pv, world, cap, torch.float32, replica_of=hot)
    outs = ep.ep_forward_virtual(ranks, [xd[s[0]:s[-1] + 1].contiguous() for s in shards])
    got = torch.cat(outs).cpu().numpy()
    for r in ranks:
        r.layer.check_device_error()
    print(f"[ep virtual replicas N={world}] rel-L2 vs single GPU {rel_l2(got, ref):.3e}")
    assert rel_l2(got, ref) < 1e-4


def test_plan_and_pack_match_the_protocol_restatement():
    """vfmoe_ep_prepare on one rank of 4 (with copies of hot experts): the send counts, every
    block's lane slots and weights (the own block in the receive buffers) and the packed rows
    equal tests/ep_protocol.py bit for bit, padding included."""
    moe.init(0)
    world, rank, T, cap = 4, 1, 24, 32
    cfg = synth.config("c0", tokens=T)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    dev = _weights(cfg, rng)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    pv, hot = ep.replicated_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    lay = _ep_layers(cfg, dev, w_r, bias, pv, world, cap, torch.float32, replica_of=hot)[rank]
    xd = _xdev(cfg, x)
    idx = torch.empty((T, cfg.topk), dtype=torch.int32, device="cuda")
    w = torch.empty((T, cfg.topk), dtype=torch.float32, device="cuda")
    lay.prepare(xd, idx, w)
    torch.cuda.synchronize()
    lay.layer.check_device_error()
    np.testing.assert_array_equal(idx.cpu().numpy(), idx_all)
    counts, tok, slot, wt, pos = proto.plan(idx.cpu().numpy(), w.cpu().numpy(), pv, hot, cfg.n_experts, world, cap)
    np.testing.assert_array_equal(lay.send_counts().cpu().numpy(), counts)
    k, H = cfg.topk, cfg.hidden
    for d in range(world):
        side = "recv" if d == rank else "send"
        got_s = lay.block(side + "_slots", d).view(torch.int32).cpu().numpy().reshape(cap, k)
        got_w = lay.block(side + "_weights", d).view(torch.float32).cpu().numpy().reshape(cap, k)
        np.testing.assert_array_equal(got_s, slot[d])
        np.testing.assert_array_equal(got_w, wt[d])
        rows = lay.block(side + "_rows", d).view(torch.float32).cpu().numpy().reshape(cap, H)
        n = counts[d]
        np.testing.assert_array_equal(rows[:n], x[tok[d, :n]])
    print(f"[ep plan] counts {counts.tolist()} bit-exact")


# ----------------------------------------------------------------------------- NCCL, one rank
def _one_rank_body(rank, world, port):
    """vfmoe_ep_forward through a 1-rank NCCL communicator equals vfmoe_forward; then the same
    call recorded in a CUDA graph and replayed."""
    moe.init(0)
    cfg = synth.config("c1", tokens=32)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    dev = synth.expert_q8_cuda(cfg, quantizer)
    full = _full(cfg, dev, w_r, bias, torch.bfloat16)
    xd = _xdev(cfg, x)
    ref = full.forward(xd)
    comm = ep.EpComm(0, 1, ep.EpComm.unique_id(), timeout_ms=60000)
    lay = ep.EpLayer(full, np.zeros(cfg.n_experts, np.int32), 0, 1, 32)
    out = torch.empty_like(ref)
    lay.forward(comm, xd, out=out)
    torch.cuda.synchronize()
    full.check_device_error()
    eager = out.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lay.forward(comm, xd, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    replay = out.clone()
    del g
    comm.close()
    d = rel_l2(eager.float().cpu().numpy(), ref.float().cpu().numpy())
    return d, bool(torch.equal(eager, replay))


_one_rank_worker = guarded(_one_rank_body)


def test_nccl_one_rank_forward_and_graph_capture():
    res = run_ranks(_one_rank_worker, 1, timeout=300)
    d, same = res[0]
    print(f"[ep nccl N=1] rel-L2 vs vfmoe_forward {d:.3e}; graph replay bit-exact {same}")
    assert d < 2e-3 and same


def _no_peer_body(rank, world, port):
    import time
    moe.init(0)
    lib = _lib.load()
    import ctypes as C
    uid = ep.EpComm.unique_id()
    t0 = time.time()
    rc = lib.vfmoe_ep_init(2, 0, C.create_string_buffer(uid, 128), 2000)
    return rc, time.time() - t0, _lib.last_error()


_no_peer_worker = guarded(_no_peer_body)


def test_ep_init_gives_up_when_a_rank_never_joins():
    """Rank 1 of 2 never calls vfmoe_ep_init: rank 0 waits at most its 2 s limit, aborts the
    half-made communicator and returns VFMOE_ERR_NCCL with a message (no kernel is involved)."""
    res = run_ranks(_no_peer_worker, 1, timeout=120)
    rc, dt, msg = res[0]
    print(f"[ep init, missing rank] rc {rc} after {dt:.1f} s: {msg}")
    assert rc == _lib.ERR_NCCL and dt < 30


# ----------------------------------------------------------------------------- NCCL, two GPUs
def _two_gpu_body(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        moe.init(rank)
        cfg = synth.config("c1", tokens=32)
        x, w_r, bias, _ = synth.router_inputs(cfg)
        E = cfg.n_experts
        placement = ep.contiguous_placement(E, world)
        mine = [int(e) for e in np.nonzero(placement == rank)[0]] + [E]
        dev = synth.expert_q8_cuda(cfg, quantizer, experts=mine)
        L = MoELayer(gate=dev[0][:-1], up=dev[1][:-1], down=dev[2][:-1], shared=(dev[0][-1], dev[1][-1], dev[2][-1]),
                     n_local_experts=E // world, **_kw(cfg, w_r, bias, torch.float32))
        shard = np.array_split(np.arange(cfg.tokens), world)[rank]
        xd = torch.from_numpy(x[shard]).to(torch.bfloat16).cuda()
        comm = ep.EpComm.from_torch_dist(timeout_ms=60000)     # the id crosses over gloo; data over NCCL
        lay = ep.EpLayer(L, placement, rank, world, 16)
        out = lay.forward(comm, xd)
        torch.cuda.synchronize()
        L.check_device_error()
        res = out.cpu().numpy()
        dist.barrier()
        comm.close()
        return res
    finally:
        dist.destroy_process_group()


_two_gpu_worker = guarded(_two_gpu_body)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_nccl_match_single_gpu():
    world = 2
    res = run_ranks(_two_gpu_worker, world, timeout=300)
    got = np.concatenate([res[r] for r in range(world)])
    moe.init(0)
    cfg = synth.config("c1", tokens=32)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    dev = synth.expert_q8_cuda(cfg, quantizer)
    ref = _full(cfg, dev, w_r, bias, torch.float32).forward(_xdev(cfg, x)).cpu().numpy()
    print(f"[ep nccl N=2] rel-L2 vs single GPU {rel_l2(got, ref):.3e}")
    assert rel_l2(got, ref) < 1e-4
