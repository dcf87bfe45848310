"""Shared builders for the GPU tests: synthetic layers on the device plus the
matching oracle getters (the oracle reads back exactly the bytes the GPU uses)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import synth
from vybforge_b200.moe import MoELayer, quantizer

TOL_MAX_ABS = 2e-2   # north_star: max-abs 2e-2 on the combined output
TOL_REL_L2 = 1e-3    # north_star: rel-L2 1e-3
TOL_REL_L2_F32 = 1e-4  # north_star: rel-L2 1e-4 where fp32 accumulation is checked (fp32 in/out layers)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_dev_x(x, cfg):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return (t.to(torch.bfloat16) if cfg.x_dtype == "bf16" else t).cuda()


class Built:
    """A device layer + host-side copies for the oracle."""

    def __init__(self, cfg, weights="numpy", out_dtype=torch.float32, router=None, path="auto", what="oracle"):
        """what="gpu" (EXL3 only): the oracle takes each expert's rotated-basis values W^ from
        vfmoe_exl3_decode, which tests/test_gpu_parity.py pins bit-exact to the oracle's own
        decode (and the reference's 4-bpw fixture), and reconstructs W in float64 itself; the
        numpy trellis decode costs seconds per full-size matrix."""
        self.path = path
        self.what = what
        self.cfg = cfg
        if router is None:
            x, w_r, bias, rng = synth.router_inputs(cfg)
        else:
            x, w_r, bias = router
            rng = np.random.default_rng(cfg.seed)
        self.x, self.w_r, self.bias = x, w_r, bias
        H, I, E = cfg.hidden, cfg.inter, cfg.n_experts
        if cfg.fmt == "exl3":
            if weights == "numpy":
                ex = synth.expert_exl3_numpy(cfg, rng)
                self.dev = {p: tuple(torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()
                                     for a in ex[p]) for p in range(3)}
            else:
                self.dev = synth.expert_exl3_cuda(cfg)
        elif weights == "numpy":
            ex = synth.expert_q8_numpy(cfg, rng)
            self.dev = {p: torch.from_numpy(ex[p]).cuda() for p in range(3)}
        else:
            self.dev = synth.expert_q8_cuda(cfg, quantizer)
        self.x_dev = to_dev_x(x, cfg)
        self.wr_dev = torch.from_numpy(w_r).cuda()
        self.bias_dev = torch.from_numpy(bias).cuda()
        self.layer = self.make_layer(out_dtype)
        self._cache = {}

    def make_layer(self, out_dtype, path=None):
        cfg, E = self.cfg, self.cfg.n_experts
        path = path or self.path
        g, u, d = self.dev[0], self.dev[1], self.dev[2]
        if cfg.fmt == "exl3":
            def head(m):
                return tuple(a[:E] for a in m)

            def tail(m):
                return tuple(a[E] for a in m)
            return MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                            router_w=self.wr_dev, router_bias=self.bias_dev,
                            gate=head(g), up=head(u), down=head(d), shared=(tail(g), tail(u), tail(d)),
                            fmt="exl3", exl3_bits=cfg.exl3_bits,
                            x_dtype=torch.bfloat16 if cfg.x_dtype == "bf16" else torch.float32,
                            out_dtype=out_dtype, path=path)
        return MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                        router_w=self.wr_dev, router_bias=self.bias_dev,
                        gate=g[:E], up=u[:E], down=d[:E], shared=(g[E], u[E], d[E]),
                        x_dtype=torch.bfloat16 if cfg.x_dtype == "bf16" else torch.float32,
                        out_dtype=out_dtype, path=path)

    def expert(self, e):
        if e not in self._cache and self.cfg.fmt == "exl3":
            def mat(p):
                if self.what == "gpu":
                    from vybforge_b200 import moe as _moe
                    tr_d, suh_d, svh_d = (a[e] for a in self.dev[p])
                    K, N = suh_d.shape[0], svh_d.shape[0]
                    what = _moe.exl3_decode(tr_d.contiguous(), K, N, self.cfg.exl3_bits).cpu().numpy()
                    return orc.dequant_exl3_from_what(what, suh_d.cpu().numpy(), svh_d.cpu().numpy())
                tr, suh, svh = (a[e].cpu().numpy() for a in self.dev[p])
                return orc.dequant_exl3(tr.view(np.uint16), suh, svh, self.cfg.exl3_bits)
            self._cache[e] = (mat(0), mat(1), mat(2))
        if e not in self._cache:
            H, I = self.cfg.hidden, self.cfg.inter
            g = self.dev[0][e].cpu().numpy()
            u = self.dev[1][e].cpu().numpy()
            d = self.dev[2][e].cpu().numpy()
            self._cache[e] = (orc.q8_0_expert_inout(g, I, H), orc.q8_0_expert_inout(u, I, H),
                              orc.q8_0_expert_inout(d, H, I))
        return self._cache[e]

    def oracle(self, tokens=None):
        """Oracle (out, idx, w) for all tokens or a subset (routing is per token)."""
        cfg = self.cfg
        x = self.x if tokens is None else self.x[tokens]
        return orc.moe_block_grouped(x, self.w_r, self.bias, self.expert,
                                     lambda: self.expert(cfg.n_experts), cfg.n_experts, cfg.topk)


def run_ranks(target, world, timeout=600):
    """Start `world` spawned processes target(rank, world, port, queue) and collect
    {rank: result}.  A worker reports ("error", traceback) on failure; the parent fails as
    soon as any worker dies or reports an error instead of waiting out the timeout."""
    import queue as _queue
    import socket
    import time
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    t0 = time.time()
    try:
        while len(res) < world:
            try:
                rank, val = q.get(timeout=5)
            except _queue.Empty:
                dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
                if dead:
                    raise AssertionError(f"a rank exited with code {dead[0]} before reporting")
                if time.time() - t0 > timeout:
                    raise AssertionError("ranks did not report within the timeout")
                continue
            if isinstance(val, tuple) and len(val) == 2 and val[0] == "error":
                raise AssertionError(f"rank {rank} failed:\n{val[1]}")
            res[rank] = val
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


def _guarded_run(fn, rank, world, port, q):
    import traceback
    try:
        q.put((rank, fn(rank, world, port)))
    except BaseException:
        q.put((rank, ("error", traceback.format_exc())))
        raise


def guarded(fn):
    """Wrap a module-level rank body fn(rank, world, port) -> result for run_ranks
    (picklable for the spawn start method)."""
    import functools
    return functools.partial(_guarded_run, fn)
