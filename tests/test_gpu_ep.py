"""Expert parallelism on the GPU: the libvfmoe EP kernels (token-level plan, pack,
forward_routed, combine) driven by vybforge_b200/ep.py, against the fused single-GPU forward.

* N virtual ranks in one process on one GPU (the whole multi-rank data path, with a
  local all-to-all) -- runs wherever a GPU is;
* 2 processes x 2 GPUs over NCCL -- runs when two GPUs are visible."""

import os
import socket

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import ep, synth, moe
from vybforge_b200.moe import MoELayer, quantizer

from helpers import rel_l2, run_ranks, guarded

pytestmark = pytest.mark.gpu


def _layers(cfg, dev, w_r, bias, placement, world, partial_dtype=torch.float32, replica_of=None):
    E = cfg.n_experts
    kw = dict(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk, router_w=torch.from_numpy(w_r).cuda(),
              router_bias=torch.from_numpy(bias).cuda(), x_dtype=torch.bfloat16 if cfg.x_dtype == "bf16" else torch.float32,
              out_dtype=torch.float32)
    full = MoELayer(gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E], shared=(dev[0][E], dev[1][E], dev[2][E]), **kw)
    per = []
    for r in range(world):
        g, u, d, sh = ep.rank_experts(dev, placement, r, replica_of)
        L = MoELayer(gate=g, up=u, down=d, shared=sh, n_local_experts=len(placement) // world, **kw)
        per.append(ep.EpRank(r, world, ep.GpuBackend(L, placement, world, out_dtype=torch.float32,
                                                     partial_dtype=partial_dtype), replica_of=replica_of, n_experts=E))
    return full, per


# fp32 partial rows: the expert-parallel path reassociates only the fp32 lane sums (1e-4);
# fp16 partial rows (the default exchange format) add one fp16 rounding per partial (5e-4).
@pytest.mark.parametrize("cfg_name,world,T,partial", [("c0", 4, 48, "f32"), ("c1", 2, 16, "f32"),
                                                      ("c1", 8, 64, "f32"), ("c1", 8, 64, "f16")])
def test_virtual_ranks_match_single_gpu(cfg_name, world, T, partial):
    moe.init(0)
    cfg = synth.config(cfg_name, tokens=T)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    if cfg_name == "c0":
        ex = synth.expert_q8_numpy(cfg, rng)
        dev = {p: torch.from_numpy(ex[p]).cuda() for p in range(3)}
    else:
        dev = synth.expert_q8_cuda(cfg, quantizer)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    placement = ep.balanced_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    pdt = torch.float32 if partial == "f32" else torch.float16
    full, ranks = _layers(cfg, dev, w_r, bias, placement, world, pdt)
    xd = (torch.from_numpy(x).to(torch.bfloat16) if cfg.x_dtype == "bf16" else torch.from_numpy(x)).cuda()
    ref = full.forward(xd).cpu().numpy()
    shards = np.array_split(np.arange(T), world)
    outs = ep.ep_forward_virtual(ranks, [xd[s[0]:s[-1] + 1].contiguous() for s in shards], ep.VirtualTransport(world))
    got = torch.cat(outs).cpu().numpy()
    for r in ranks:
        r.b.layer.check_device_error()
    print(f"[ep virtual {cfg_name} N={world} T={T} {partial} partials] rel-L2 vs single GPU {rel_l2(got, ref):.3e}")
    assert rel_l2(got, ref) < (1e-4 if partial == "f32" else 5e-4)


@pytest.mark.parametrize("world", [2, 8])
def test_virtual_ranks_with_replicated_experts_match_single_gpu(world):
    """The hottest experts copied to a second rank (replicated_placement); odd tokens' lanes
    go to the copies.  Same result as the fused single-GPU forward up to fp32 lane order."""
    moe.init(0)
    cfg = synth.config("c1", tokens=64)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    dev = synth.expert_q8_cuda(cfg, quantizer)
    idx_all, _ = orc.route(x, w_r, bias, cfg.topk)
    pv, hot = ep.replicated_placement(np.bincount(idx_all.reshape(-1), minlength=cfg.n_experts), world)
    full, ranks = _layers(cfg, dev, w_r, bias, pv, world, torch.float32, replica_of=hot)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    ref = full.forward(xd).cpu().numpy()
    shards = np.array_split(np.arange(cfg.tokens), world)
    outs = ep.ep_forward_virtual(ranks, [xd[s[0]:s[-1] + 1].contiguous() for s in shards], ep.VirtualTransport(world))
    got = torch.cat(outs).cpu().numpy()
    for r in ranks:
        r.b.layer.check_device_error()
    print(f"[ep virtual replicas N={world}] rel-L2 vs single GPU {rel_l2(got, ref):.3e}")
    assert rel_l2(got, ref) < 1e-4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_body(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        moe.init(rank)
        cfg = synth.config("c1", tokens=32)
        x, w_r, bias, _ = synth.router_inputs(cfg)
        E = cfg.n_experts
        placement = ep.contiguous_placement(E, world)
        mine = [int(e) for e in np.nonzero(placement == rank)[0]] + [E]
        dev = synth.expert_q8_cuda(cfg, quantizer, experts=mine)
        L = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                     router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                     gate=dev[0][:-1], up=dev[1][:-1], down=dev[2][:-1], shared=(dev[0][-1], dev[1][-1], dev[2][-1]),
                     n_local_experts=E // world, out_dtype=torch.float32)
        shard = np.array_split(np.arange(cfg.tokens), world)[rank]
        xd = torch.from_numpy(x[shard]).to(torch.bfloat16).cuda()
        out = ep.ep_forward_dist(ep.EpRank(rank, world, ep.GpuBackend(L, placement, world, torch.float32)), xd,
                                 ep.DistTransport())   # default exchange: fp16 partial rows
        L.check_device_error()
        res = out.cpu().numpy()
        dist.barrier()
        return res
    finally:
        dist.destroy_process_group()


_nccl_worker = guarded(_nccl_body)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_nccl_match_single_gpu():
    world = 2
    res = run_ranks(_nccl_worker, world, timeout=300)
    got = np.concatenate([res[r] for r in range(world)])
    moe.init(0)
    cfg = synth.config("c1", tokens=32)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    dev = synth.expert_q8_cuda(cfg, quantizer)
    E = cfg.n_experts
    full = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk, router_w=torch.from_numpy(w_r).cuda(),
                    router_bias=torch.from_numpy(bias).cuda(), gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E],
                    shared=(dev[0][E], dev[1][E], dev[2][E]), out_dtype=torch.float32)
    ref = full.forward(torch.from_numpy(x).to(torch.bfloat16).cuda()).cpu().numpy()
    print(f"[ep nccl N=2] rel-L2 vs single GPU {rel_l2(got, ref):.3e}")
    assert rel_l2(got, ref) < 5e-4
