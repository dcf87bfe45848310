#!/usr/bin/env python
"""MoE-layer throughput on B200: the north-star metric of this repository.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c2|c3|c4d|c4p] [--tokens T]

One step = one forward of the GLM-style MoE layer (router, dispatch, routed +
shared SwiGLU experts over Q8_0 weights, weighted combine) on one batch of
synthetic tokens.  Default workload: BASELINE config 1 (H=6144, I=2048, E=256,
top-8, 1 shared expert, Q8_0, bf16 activations), decode batch T=32 per GPU.

Prints ONE JSON line (rank 0).  `value` is device-timed tokens/s over all ranks
(CUDA events on the launch stream, max over ranks, L2 flushed between steps);
`e2e` is the same metric through the public API with host (pinned) buffers and
the H2D/D2H copies inside the timed region; `roofline` is the dominant kernel
(the expert gate/up GEMV) against measured HBM bandwidth; `cpu_baseline` is the
numpy oracle timed on a bounded sample on this host.

`--impl reference` times the reference algorithm's CPU implementation (the numpy
restatement of native/glm53/moe_ref.py, which is what the reference runs on CPU;
its Vyb GPU kernels cannot be built here) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "MoE-layer tokens/s (decode b1/b32, prefill 4k) + % HBM/TC roofline, 1-8 GPU"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def args_parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c1", choices=["c1", "c2", "c3", "c4d", "c4p"])
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--fmt", default=None, choices=[None, "q8_0", "exl3"])
    ap.add_argument("--experts", type=int, default=None,
                    help="override the routed expert count (small cases for ncu captures only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the extra T=1 and prefill measurements")
    ap.add_argument("--cpu-budget-s", type=float, default=20.0)
    ap.add_argument("--ep-replicas", type=int, default=-1,
                    help="C4 at N > 1: copies of the hottest experts on other ranks (a multiple of N; 0 = none; "
                         "-1 = N copies at N >= 8, where one rank would otherwise carry a whole hottest expert)")
    ap.add_argument("--q8-layout", default="tiled", choices=["tiled", "rows"],
                    help="Q8_0 weights in HBM: stage-tiled (converted once at load, outside the timed "
                         "region) or GGUF row order")
    ap.add_argument("--profile-case", default=None, choices=list(PROFILE_CASES),
                    help="run one small fixed case for an ncu capture (no JSON line) and exit")
    return ap.parse_args()


# dram bytes / algorithmic bytes of the Q8_0 gate/up GEMV per weight layout, from ncu
# captures of the 64-expert case (--profile-case q8_decode_e64 [--q8-layout rows])
GEMV_Q8_TRAFFIC_RATIO = {"q8_0_tiled": 1.006, "q8_0": 1.015}

def q8_layout_weights(layout, dev):
    """A layer's Q8_0 weights in the bench's layout: stage-tiled by default (VFMOE_WFMT_Q8_0_TILED,
    one vfmoe_q8_0_tile pass at load, outside every timed region) or GGUF row order."""
    if layout == "rows":
        return dev, "q8_0"
    from vybforge_b200.moe import q8_0_tile
    return {p: q8_0_tile(dev[p]) for p in range(3)}, "q8_0_tiled"


# ----------------------------------------------------------------------------- ncu cases
def _profile_decode(fmt, layout="tiled"):
    """C1 (Q8_0) or C2 (EXL3 3 bpw) layer shapes with 64 routed experts, T=32: about 0.9 GB of
    weights (above L2, a few GB on the device at most); three forwards."""
    import torch
    from vybforge_b200 import synth
    from vybforge_b200.moe import MoELayer, init, quantizer
    init(0)
    cfg = synth.config("c1" if fmt == "q8_0" else "c2", tokens=32)
    cfg.n_experts = 64
    x, w_r, bias, _ = synth.router_inputs(cfg)
    E = cfg.n_experts
    if fmt == "q8_0":
        dev, wf = q8_layout_weights(layout, synth.expert_q8_cuda(cfg, quantizer))
        mats = dict(gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E], shared=(dev[0][E], dev[1][E], dev[2][E]),
                    fmt=wf)
    else:
        dev = synth.expert_exl3_cuda(cfg)
        mats = dict(gate=tuple(a[:E] for a in dev[0]), up=tuple(a[:E] for a in dev[1]),
                    down=tuple(a[:E] for a in dev[2]), shared=tuple(tuple(a[E] for a in dev[p]) for p in range(3)),
                    fmt="exl3")
    layer = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                     router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                     x_dtype=torch.bfloat16, out_dtype=torch.bfloat16, **mats)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    for _ in range(3):
        layer.forward(xd)
    torch.cuda.synchronize()
    layer.check_device_error()


def _profile_prefill(layout="tiled"):
    """C3 shapes (Q8_0, Zipf(1.1) routing, T=4096) with 64 routed experts: ~0.9 GB of weights;
    three forwards."""
    import torch
    from vybforge_b200 import synth
    from vybforge_b200.moe import MoELayer, init, quantizer
    init(0)
    cfg = synth.config("c3", tokens=4096)
    cfg.n_experts = 64
    x, w_r, bias, _, _ = synth.zipf_router_inputs(cfg)
    E = cfg.n_experts
    dev, wf = q8_layout_weights(layout, synth.expert_q8_cuda(cfg, quantizer))
    layer = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                     router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                     gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E], shared=(dev[0][E], dev[1][E], dev[2][E]),
                     x_dtype=torch.bfloat16, out_dtype=torch.bfloat16, fmt=wf)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    for _ in range(3):
        layer.forward(xd)
    torch.cuda.synchronize()
    layer.check_device_error()


def _profile_router():
    """Router alone at the C1 shape for T = 1 ... 8192 (13 calls per size), with the median
    CUDA-event time per size printed as one JSON line."""
    import torch
    from vybforge_b200 import synth
    from vybforge_b200.moe import MoELayer, init, quantizer
    init(0)
    cfg = synth.config("c1", tokens=8192)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    E = cfg.n_experts
    dev = synth.expert_q8_cuda(cfg, quantizer, experts=[0, E])
    layer = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                     router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                     gate=dev[0][:1], up=dev[1][:1], down=dev[2][:1], shared=(dev[0][1], dev[1][1], dev[2][1]),
                     x_dtype=torch.bfloat16, out_dtype=torch.bfloat16, n_local_experts=1)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    res = {}
    for T in [1, 8, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192]:
        xt = xd[:T].contiguous()
        for _ in range(3):
            layer.route(xt)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
        for s_, e_ in ev:
            s_.record()
            layer.route(xt)
            e_.record()
        torch.cuda.synchronize()
        res[T] = round(float(np.median([s_.elapsed_time(e_) for s_, e_ in ev])) * 1000, 1)
    layer.check_device_error()
    print(json.dumps({"route_us": res}))


def _profile_hc_mix():
    """vfmoe_hc_mix at the C3 token count (R = 4096 rows of 4 fp32 streams, H = 6144, bf16 hc_fn,
    the tensor-core mix), three calls; 0.5 GB on the device."""
    import torch
    from vybforge_b200.moe import HyperConnection, init
    init(0)
    R, D = 4096, 6144
    g = torch.Generator(device="cuda").manual_seed(5)
    fn = (torch.randn((24, 4 * D), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    site = HyperConnection(fn, torch.randn(24, generator=g, device="cuda") * 0.5,
                           torch.tensor([0.8, 1.3, 2.0], device="cuda"), 1 + 0.02 * torch.randn(D, generator=g, device="cuda"))
    streams = torch.randn((R, 4, D), generator=g, device="cuda")
    for _ in range(3):
        h, post, comb = site.mix(streams)
    torch.cuda.synchronize()
    print(json.dumps({"hc_mix_h_mean_abs": float(h.float().abs().mean())}))


PROFILE_CASES = {"q8_decode_e64": lambda a: _profile_decode("q8_0", a.q8_layout),
                 "exl3_decode_e64": lambda a: _profile_decode("exl3"),
                 "q8_prefill_e64": lambda a: _profile_prefill(a.q8_layout), "router_sweep": lambda a: _profile_router(),
                 "hc_mix": lambda a: _profile_hc_mix()}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        """Start sampling and return once the first sample has arrived (at most 3 s), so the
        sampler is live when the timed region begins."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 3.0:
                time.sleep(0.005)
        except Exception:
            self.proc = None
        self.t_begin = time.perf_counter()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def stop(self):
        t_end = time.perf_counter()
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.03)  # one more sampling period, so the region's last sample is read
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        # samples taken while the timed region ran (20 ms period): those stamped inside
        # [begin, end + 25 ms], else the first one after the region began
        inside = [ln for ts, ln in self.lines if self.t_begin <= ts <= t_end + 0.025]
        if not inside:
            inside = [ln for ts, ln in self.lines if ts >= self.t_begin][:1]
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in inside:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- workload
def algorithmic_bytes(cfg, n_distinct_experts, has_shared=True):
    H, I, E, T = cfg.hidden, cfg.inter, cfg.n_experts, cfg.tokens
    bits = getattr(cfg, "exl3_bits", 3)
    per_expert = 3 * H * I * 34 // 32 if cfg.fmt == "q8_0" else 3 * (H * I * bits // 8 + 2 * (H + I))
    gate_up = 2 * H * I * 34 // 32 if cfg.fmt == "q8_0" else 2 * (H * I * bits // 8 + 2 * (H + I))
    layer = (n_distinct_experts + (1 if has_shared else 0)) * per_expert + E * H * 4 + T * H * 4
    gu = (n_distinct_experts + (1 if has_shared else 0)) * gate_up
    return layer, gu


def build_ours(cfg, rank, layout):
    """The layer on GPU weights in `layout`; also returns the GGUF-row weights (for the CPU
    baseline) and the layer's own weights."""
    import torch
    from vybforge_b200 import synth
    from vybforge_b200.moe import MoELayer, quantizer
    x, w_r, bias, rng = synth.router_inputs(cfg)
    dev = synth.expert_q8_cuda(cfg, quantizer)
    devl, wf = q8_layout_weights(layout, dev)
    E = cfg.n_experts
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    layer = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                     router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(), fmt=wf,
                     gate=devl[0][:E], up=devl[1][:E], down=devl[2][:E], shared=(devl[0][E], devl[1][E], devl[2][E]),
                     x_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
    return layer, xd, (x, w_r, bias), dev, (devl, wf)


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline_ours(cfg, host, dev, idx, budget_s):
    """Oracle (numpy, f64) on a bounded sample of this step's tokens, same bytes as the GPU."""
    from oracle import moe_oracle as orc
    x, w_r, bias = host
    H, I, E = cfg.hidden, cfg.inter, cfg.n_experts
    # sample: the first n tokens whose distinct experts fit the CPU budget (~0.2 s per expert)
    n = 1
    while n < cfg.tokens and len(np.unique(idx[:n + 1])) + 1 <= max(4, int(budget_s / 0.25)):
        n += 1
    need = sorted(set(np.unique(idx[:n]).tolist()) | {E})
    raw = {e: tuple(dev[p][e].cpu().numpy() for p in range(3)) for e in need}

    def get(e):
        g, u, d = raw[e]
        return (orc.q8_0_expert_inout(g, I, H), orc.q8_0_expert_inout(u, I, H), orc.q8_0_expert_inout(d, H, I))
    t0 = time.perf_counter()
    orc.moe_block_grouped(x[:n], w_r, bias, get, lambda: get(E), E, cfg.topk)
    dt = time.perf_counter() - t0
    cores = os.cpu_count()
    return {"value": n / dt, "unit": "tokens/s", "cores": cores, "kind": "port", "cpu_model": cpu_model(),
            "sample": f"first {n} of {cfg.tokens} tokens ({len(need)} experts incl. shared), oracle "
                      f"dequant+f64 GEMM per expert, numpy/OpenBLAS on {cores} host threads, {dt:.1f} s"}


def time_layer(layer, xd, steps, warmup, flush, with_profile=True):
    """Device time per forward (CUDA events on the launch stream, L2 flushed between steps),
    per-stage times from the library's event marks and the kernel launch count."""
    import ctypes as C
    import torch
    st = torch.cuda.current_stream()
    T = xd.shape[0]
    out = torch.empty((T, layer.H), dtype=layer.out_dtype, device="cuda")
    idx = torch.empty((T, layer.k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, layer.k), dtype=torch.float32, device="cuda")
    ws = layer.workspace(T)
    for _ in range(max(3, warmup)):
        layer.forward(xd, out=out, idx=idx, w=w, workspace=ws)
    torch.cuda.synchronize()
    lib = layer.lib
    if with_profile:
        lib.vfmoe_profile_enable(layer.handle, 1)
        lib.vfmoe_profile_read(layer.handle, (C.c_double * 8)(), 8, None)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(st)
        layer.forward(xd, out=out, idx=idx, w=w, workspace=ws)
        ev[i][1].record(st)
    torch.cuda.synchronize()
    ms = float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))
    stage = (C.c_double * 8)()
    launches = C.c_int64(0)
    nf = max(1, lib.vfmoe_profile_read(layer.handle, stage, 8, C.byref(launches))) if with_profile else 1
    lib.vfmoe_profile_enable(layer.handle, 0)
    names = ["router", "dispatch_gather", "gate_up", "down", "combine"]
    return ms, {n: stage[i] / nf for i, n in enumerate(names)}, int(launches.value), idx


def time_graph(layer, xd, steps, flush):
    """Device time per forward replayed from a CUDA graph of one vfmoe_forward (caller
    workspace, no stage events), CUDA events around each replay, L2 flushed between replays."""
    import torch
    st = torch.cuda.current_stream()
    T = xd.shape[0]
    out = torch.empty((T, layer.H), dtype=layer.out_dtype, device="cuda")
    idx = torch.empty((T, layer.k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, layer.k), dtype=torch.float32, device="cuda")
    ws = layer.workspace(T)
    for _ in range(3):
        layer.forward(xd, out=out, idx=idx, w=w, workspace=ws)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer.forward(xd, out=out, idx=idx, w=w, workspace=ws)
    for _ in range(3):
        graph.replay()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        ev[i][0].record(st)
        graph.replay()
        ev[i][1].record(st)
    torch.cuda.synchronize()
    layer.check_device_error()
    del graph
    return float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))


def prefill_extra(a, cfg1, dev, wf, flush):
    """C3: T=4096 prefill, Zipf(1.1)-skewed routing, same Q8_0 expert weights as C1."""
    import torch
    from vybforge_b200 import synth
    from vybforge_b200.moe import MoELayer
    cfg = synth.config("c3", tokens=4096)
    x, w_r, bias, tgt, _ = synth.zipf_router_inputs(cfg)
    E = cfg.n_experts
    layer = MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                     router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                     gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E], shared=(dev[0][E], dev[1][E], dev[2][E]),
                     x_dtype=torch.bfloat16, out_dtype=torch.bfloat16, fmt=wf)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    ms, stages, launches, idx = time_layer(layer, xd, max(5, a.steps // 2), a.warmup, flush)
    T, H, I, k = cfg.tokens, cfg.hidden, cfg.inter, cfg.topk
    rows = T * k + T
    flops = 6.0 * H * I * rows + 2.0 * H * E * T
    gu_flops, dn_flops = 4.0 * H * I * rows, 2.0 * H * I * rows
    pk, pk_kind = peaks()
    cnt = np.bincount(idx.cpu().numpy().reshape(-1), minlength=E)
    gu_tf = gu_flops / (stages["gate_up"] * 1e-3) / 1e12
    dn_tf = dn_flops / (stages["down"] * 1e-3) / 1e12
    layer.close()
    return {"workload": "c3: prefill T=4096, Zipf(1.1) routing, Q8_0, same layer shapes as c1",
            "tokens_per_s": round(T / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
            "layer_tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "roofline": {"bound": "tensor", "kernel": "expert gate/up grouped GEMM (tcgen05, Q8_0 -> fp16 in TMEM)",
                         "achieved": round(gu_tf, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(gu_tf / pk["bf16_tflops"], 4),
                         "frac_of_sustained": round(gu_tf / pk.get("bf16_tflops_sustained", pk["bf16_tflops"]), 4),
                         "down_achieved": round(dn_tf, 1), "peak_source": pk_kind,
                         "algorithmic_flops_per_launch": gu_flops},
            "stage_ms_per_step": {n: round(v, 4) for n, v in stages.items()}, "gpu_launches": launches,
            "expert_tokens": {"max": int(cnt.max()), "median": float(np.median(cnt)), "min": int(cnt.min()),
                              "zipf_target_max": float(tgt.max())}}


def stack_extra(a, rank, world, local_rank, flush):
    """BASELINE C4: 4 pre-norm MoE layers of the C1 shape, Q8_0, bf16 activations.
    prefill T=8192 (Zipf(1.1) routers, calibrated per layer) and decode T=256 (plain routers);
    global token counts fixed (strong scaling).  N=1: MoEStack on one GPU.  N>1: expert-parallel
    (EpStack: vfmoe_ep_forward, the library's NCCL exchange), E/N experts per GPU placed by the
    load measured on calibration tokens disjoint from the timed ones, shared expert and routers
    replicated, tokens sharded."""
    import torch
    from vybforge_b200 import synth, ep
    from vybforge_b200.moe import MoELayer, quantizer
    from vybforge_b200.stack import MoEStack, EpStack, token_shards
    L = 4
    t_setup = time.perf_counter()
    cfgp, cfgd = synth.config("c4p"), synth.config("c4d")
    xp, norm_p, routers_p = synth.stack_inputs(cfgp, L)
    xd, norm_d, routers_d = synth.stack_inputs(cfgd, L)
    E, H, I, k = cfgp.n_experts, cfgp.hidden, cfgp.inter, cfgp.topk
    n_rep = (world if world >= 8 else 0) if a.ep_replicas < 0 else a.ep_replicas
    n_rep = n_rep if world > 1 else 0
    if n_rep:
        placed = [ep.replicated_placement(routers_p[l][2], world, n_rep) for l in range(L)]
        placements, replicas = [p_ for p_, _ in placed], [h for _, h in placed]
    else:
        placements = [ep.balanced_placement(routers_p[l][2], world) if world > 1 else np.zeros(E, np.int32)
                      for l in range(L)]
        replicas = [np.zeros(0, np.int32)] * L
    layers = {"p": [], "d": []}
    for l in range(L):
        # this rank's (virtual) experts in ascending order; copy E + j holds expert replicas[l][j]
        mine = [int(e) if e < E else int(replicas[l][e - E]) for e in np.nonzero(placements[l] == rank)[0]] + [E]
        dev, wf = q8_layout_weights(a.q8_layout, synth.expert_q8_cuda(cfgp, quantizer, layer=l, experts=mine))
        torch.cuda.empty_cache()
        for key, routers in (("p", routers_p), ("d", routers_d)):
            w_r, bias, _ = routers[l]
            lay = MoELayer(hidden=H, inter=I, n_experts=E, topk=k, router_w=torch.from_numpy(w_r).cuda(),
                           router_bias=torch.from_numpy(bias).cuda(), gate=dev[0][:-1], up=dev[1][:-1],
                           down=dev[2][:-1], shared=(dev[0][-1], dev[1][-1], dev[2][-1]),
                           n_local_experts=len(placements[l]) // world if world > 1 else 0, fmt=wf,
                           x_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
            layers[key].append(lay)
    t_setup = time.perf_counter() - t_setup
    st = torch.cuda.current_stream()
    comm = ep.EpComm.from_torch_dist() if world > 1 else None
    out = {}
    for key, cfg, x, norm in (("p", cfgp, xp, norm_p), ("d", cfgd, xd, norm_d)):
        T = cfg.tokens
        nw = [torch.from_numpy(w).cuda() for w in norm]
        if world > 1:
            shards = token_shards(T, world)
            cap = max(len(s_) for s_ in shards)
            stack = EpStack([ep.EpLayer(lay, placements[l], rank, world, cap, replicas[l])
                             for l, lay in enumerate(layers[key])], nw)
            sh = shards[rank]
            xl = torch.from_numpy(x[sh[0]:sh[-1] + 1]).to(torch.bfloat16).cuda()
            step = lambda: stack.forward(comm, xl)
        else:
            stack = MoEStack(layers[key], nw)
            xl = torch.from_numpy(x).to(torch.bfloat16).cuda()
            step = lambda: stack.forward(xl)
        steps = max(5, a.steps // 2)
        for _ in range(max(3, a.warmup)):
            step()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            if world > 1:
                torch.distributed.barrier()
            ev[i][0].record(st)
            step()
            ev[i][1].record(st)
        torch.cuda.synchronize()
        ms = float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))
        phases = None
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
            # one more step with the library's phase events on (vfmoe_ep_forward stages), all
            # layers summed, max over ranks per phase
            import ctypes as C
            for lay in layers[key]:
                lay.lib.vfmoe_profile_enable(lay.handle, 1)
                lay.lib.vfmoe_profile_read(lay.handle, (C.c_double * 8)(), 8, None)
            torch.distributed.barrier()
            step()
            torch.cuda.synchronize()
            tot = np.zeros(6)
            for lay in layers[key]:
                buf = (C.c_double * 8)()
                lay.lib.vfmoe_profile_read(lay.handle, buf, 8, None)
                lay.lib.vfmoe_profile_enable(lay.handle, 0)
                tot += np.array(buf[:6])
            names = ["route_plan_pack", "shared_expert", "dispatch_wait", "experts", "return_exchange", "combine"]
            pt = torch.tensor(tot, device="cuda")
            torch.distributed.all_reduce(pt, op=torch.distributed.ReduceOp.MAX)
            phases = {n_: round(float(v), 3) for n_, v in zip(names, pt.tolist())}
        else:
            # one more step with the library's stage events on: device ms per stage, all layers
            import ctypes as C
            for lay in layers[key]:
                lay.lib.vfmoe_profile_enable(lay.handle, 1)
                lay.lib.vfmoe_profile_read(lay.handle, (C.c_double * 8)(), 8, None)
            step()
            torch.cuda.synchronize()
            tot = np.zeros(5)
            for lay in layers[key]:
                buf = (C.c_double * 8)()
                lay.lib.vfmoe_profile_read(lay.handle, buf, 8, None)
                lay.lib.vfmoe_profile_enable(lay.handle, 0)
                tot += np.array(buf[:5])
            phases = {n_: round(float(v), 3) for n_, v in
                      zip(["router", "dispatch_gather", "gate_up", "down", "combine"], tot)}
        for lay in layers[key]:
            lay.check_device_error()
        pk, pk_kind = peaks()
        res = {"tokens_per_s": round(T / (ms * 1e-3), 1), "ms_per_step": round(ms, 4), "n_gpus": world,
               "global_tokens": T, "layers": L}
        if phases:
            res["phase_ms_per_step" + ("_max_over_ranks" if world > 1 else "")] = phases
        if key == "p":
            flops = L * (6.0 * H * I * T * (k + 1) + 2.0 * H * E * T)
            tf = flops / (ms * 1e-3) / 1e12
            res.update({"workload": "c4p: 4 layers x (RMSNorm + MoE + residual), prefill T=8192, Zipf(1.1) "
                                    "routers, Q8_0, bf16 activations",
                        "roofline": {"bound": "tensor", "achieved": round(tf, 1), "unit": "TFLOP/s",
                                     "peak": round(world * pk["bf16_tflops"], 1),
                                     "frac": round(tf / (world * pk["bf16_tflops"]), 4), "peak_source": pk_kind,
                                     "algorithmic_flops_per_step": flops}})
            if world > 1:
                def vload(l):  # expected rows per (virtual) expert: a copy and its expert share the rows
                    ld = np.concatenate([routers_p[l][2], np.zeros(len(replicas[l]))]).astype(np.float64)
                    ld[replicas[l]] = ld[E:] = routers_p[l][2][replicas[l]] / 2
                    return ld
                loads = np.array([[vload(l)[placements[l] == r].sum() for r in range(world)] for l in range(L)])
                res["placement_expected_rows_max_over_mean"] = round(float((loads.max(1) / loads.mean(1)).max()), 3)
                res["ep_replicas"] = n_rep
        else:
            res["workload"] = "c4d: 4 layers x (RMSNorm + MoE + residual), decode T=256, Q8_0, bf16 activations"
        out["c4" + key] = res
        del stack
    out["c4_setup_s"] = round(t_setup, 1)
    for key in layers:
        for lay in layers[key]:
            lay.close()
    if comm is not None:
        comm.close()
    return out


def hc_extra(a, flush):
    """The hyper-connection kernels around the MoE (vfmoe_hc_mix with the fused post-attention
    RMSNorm, vfmoe_hc_apply) at the C3 token count: R = 4096 rows of 4 fp32 streams, H = 6144, bf16
    hc_fn and h.  HBM-bound: mix moves 16 H + 2 H bytes per row (streams in, h out), apply 16 H + 2 H
    + 16 H (streams and y in, streams out)."""
    import torch
    from vybforge_b200.moe import HyperConnection
    try:
        R, D = 4096, 6144
        g = torch.Generator(device="cuda").manual_seed(5)
        fn = (torch.randn((24, 4 * D), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        base = torch.randn(24, generator=g, device="cuda") * 0.5
        scale = torch.tensor([0.8, 1.3, 2.0], device="cuda")
        norm_w = 1 + 0.02 * torch.randn(D, generator=g, device="cuda")
        site = HyperConnection(fn, base, scale, norm_w)
        streams = torch.randn((R, 4, D), generator=g, device="cuda")
        out = torch.empty_like(streams)
        st = torch.cuda.current_stream()
        for _ in range(3):
            h, post, comb = site.mix(streams)
            site.apply(streams, h, post, comb, out=out)
        torch.cuda.synchronize()
        times = {"mix": [], "apply": []}
        for _ in range(max(3, a.steps // 2)):
            for name in ("mix", "apply"):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                if name == "mix":
                    site.mix(streams)
                else:
                    site.apply(streams, h, post, comb, out=out)
                e1.record(st)
                torch.cuda.synchronize()
                times[name].append(e0.elapsed_time(e1))
        pk, pk_kind = peaks()
        res = {}
        for name, nbytes in (("mix", 18.0 * D * R), ("apply", 34.0 * D * R)):
            ms = float(np.mean(times[name]))
            res[name] = {"ms": round(ms, 4), "hbm_bytes": nbytes, "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)}
        return {"hc_site_c3": {"workload": "hyper-connection mix (+ RMSNorm) and apply, R=4096 rows x 4 fp32 streams, H=6144",
                               "peak_source": pk_kind, **res}}
    except Exception as e:  # an extra must not cost the headline line
        return {"hc_site_c3": {"error": str(e)[:300]}}


def exl3_extra(a, flush):
    """C2 (decode T=32 and T=1) and C3 with EXL3 3-bpw weights (prefill T=4096, Zipf(1.1)),
    on one GPU: the same layer shapes as C1."""
    import torch
    from vybforge_b200 import synth
    from vybforge_b200.moe import MoELayer
    cfg = synth.config("c2", tokens=32)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    dev = synth.expert_exl3_cuda(cfg)
    E, H, I = cfg.n_experts, cfg.hidden, cfg.inter
    pk, pk_kind = peaks()
    mats = dict(gate=tuple(t[:E] for t in dev[0]), up=tuple(t[:E] for t in dev[1]), down=tuple(t[:E] for t in dev[2]),
                shared=tuple(tuple(t[E] for t in dev[p]) for p in range(3)), fmt="exl3")

    def make(w_r_, bias_):
        return MoELayer(hidden=H, inter=I, n_experts=E, topk=cfg.topk, router_w=torch.from_numpy(w_r_).cuda(),
                        router_bias=torch.from_numpy(bias_).cuda(), x_dtype=torch.bfloat16,
                        out_dtype=torch.bfloat16, **mats)
    out = {}
    layer = make(w_r, bias)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    def decode_entry(T, c, ms, st_, idx, ms_plain, note):
        """tokens/s and the layer fraction from the step without the library's per-stage events;
        the event-timed step, its split and the gate/up GEMV's own fraction beside them."""
        lb, gub = algorithmic_bytes(c, len(np.unique(idx.cpu().numpy())))
        return {"tokens_per_s": round(T / (ms_plain * 1e-3), 1), "ms_per_step": round(ms_plain, 4),
                "layer_hbm_frac": round(lb / (ms_plain * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                "with_stage_events": {"ms_per_step": round(ms, 4),
                                      "gate_up_hbm_frac": round(gub / (st_["gate_up"] * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                                      "stage_ms_per_step": {n: round(v, 4) for n, v in st_.items()}},
                "note": note}

    for T in (32, 1):
        ms, st_, _, idx = time_layer(layer, xd[:T].contiguous(), a.steps, a.warmup, flush)
        ms_plain = time_layer(layer, xd[:T].contiguous(), a.steps, a.warmup, flush, with_profile=False)[0]
        out[f"c2_t{T}"] = decode_entry(T, synth.config("c2", tokens=T), ms, st_, idx, ms_plain,
                                       "EXL3 decode GEMV is bound by the trellis decode's integer work, not HBM")
    layer.close()
    c3 = synth.config("c3", tokens=4096, fmt="exl3")
    x3, w3, b3, _, _ = synth.zipf_router_inputs(c3)
    layer = make(w3, b3)
    ms, st_, launches, idx = time_layer(layer, torch.from_numpy(x3).to(torch.bfloat16).cuda(), max(5, a.steps // 2),
                                        a.warmup, flush)
    T, k = c3.tokens, c3.topk
    flops = 6.0 * H * I * T * (k + 1) + 2.0 * H * E * T
    out["c3_prefill_exl3"] = {"tokens_per_s": round(T / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
                              "layer_tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                              "frac_of_bf16_peak": round(flops / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4),
                              "stage_ms_per_step": {n: round(v, 4) for n, v in st_.items()},
                              "note": "tcgen05 EXL3 GEMMs (trellis decoded into TMEM, Hadamard epilogues); "
                                      "bound by the trellis decode's integer work"}
    layer.close()
    # the reference's own EXL3 format (4 bpw, its slot table in closed form) at C2 shapes, T=32
    del mats, dev
    torch.cuda.empty_cache()
    c4 = synth.config("c2", tokens=32)
    c4.exl3_bits = 4
    dev4 = synth.expert_exl3_cuda(c4)
    mats = dict(gate=tuple(t[:E] for t in dev4[0]), up=tuple(t[:E] for t in dev4[1]),
                down=tuple(t[:E] for t in dev4[2]), shared=tuple(tuple(t[E] for t in dev4[p]) for p in range(3)),
                fmt="exl3", exl3_bits=4)
    layer = make(w_r, bias)
    ms, st_, _, idx = time_layer(layer, xd[:32].contiguous(), a.steps, a.warmup, flush)
    ms_plain = time_layer(layer, xd[:32].contiguous(), a.steps, a.warmup, flush, with_profile=False)[0]
    out["c2_4bpw_t32"] = decode_entry(32, c4, ms, st_, idx, ms_plain, "EXL3 4 bpw (the reference's format), C2 shapes")
    layer.close()
    return out


def run_ours_ep(a, rank, world, local_rank):
    """N > 1: the C1 layer expert-parallel over NCCL.  Each rank holds E/N routed experts
    (contiguous placement; decode routing is uniform), the router and the shared expert,
    and routes its own T tokens (weak scaling: global batch = N*T)."""
    import torch
    import torch.distributed as dist
    from vybforge_b200 import synth, ep
    from vybforge_b200.moe import MoELayer, quantizer, init
    torch.cuda.set_device(local_rank)
    init(local_rank)
    T = a.tokens or 32
    cfg = synth.config(a.workload, tokens=T * world)
    x, w_r, bias, _ = synth.router_inputs(cfg)          # same draws on every rank (seed 0)
    E, H = cfg.n_experts, cfg.hidden
    placement = ep.contiguous_placement(E, world)
    mine = [int(e) for e in np.nonzero(placement == rank)[0]] + [E]
    dev, wf = q8_layout_weights(a.q8_layout, synth.expert_q8_cuda(cfg, quantizer, experts=mine))
    layer = MoELayer(hidden=H, inter=cfg.inter, n_experts=E, topk=cfg.topk, router_w=torch.from_numpy(w_r).cuda(),
                     router_bias=torch.from_numpy(bias).cuda(), gate=dev[0][:-1], up=dev[1][:-1], down=dev[2][:-1],
                     shared=(dev[0][-1], dev[1][-1], dev[2][-1]), n_local_experts=E // world, fmt=wf,
                     x_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
    comm = ep.EpComm.from_torch_dist()
    rs = ep.EpLayer(layer, placement, rank, world, T)
    xl = torch.from_numpy(x[rank * T:(rank + 1) * T]).to(torch.bfloat16).cuda()
    out_l = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(max(3, a.warmup)):
        rs.forward(comm, xl, out=out_l)
    dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    for i in range(a.steps):
        flush.zero_()
        dist.barrier()
        ev[i][0].record(st)
        rs.forward(comm, xl, out=out_l)
        ev[i][1].record(st)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    ms = float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev]))
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # e2e: host tokens in, host output back, through the same public path
    xh = xl.cpu().pin_memory()
    oh = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    xin = torch.empty_like(xl)
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    for i in range(a.steps):
        flush.zero_()
        dist.barrier()
        ev2[i][0].record(st)
        xin.copy_(xh, non_blocking=True)
        o = rs.forward(comm, xin, out=out_l)
        oh.copy_(o, non_blocking=True)
        ev2[i][1].record(st)
    torch.cuda.synchronize()
    e2e_ms = float(np.mean([s_.elapsed_time(e_) for s_, e_ in ev2]))
    t = torch.tensor([e2e_ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    comm.close()
    extra = None
    if not a.no_extra and a.workload == "c1" and a.tokens is None:
        layer_keep = layer
        extra = stack_extra(a, rank, world, local_rank, flush)
        layer = layer_keep
    # algorithmic bytes of the whole job: distinct experts touched (global routing) + shared per rank
    from vybforge_b200.moe import MoELayer as _L  # noqa: F401
    idx, _ = layer.route(torch.from_numpy(x).to(torch.bfloat16).cuda())
    n_distinct = len(np.unique(idx.cpu().numpy()))
    per_expert = 3 * H * cfg.inter * 34 // 32
    job_bytes = (n_distinct + world) * per_expert + world * E * H * 4 + world * T * H * 4
    pk, pk_kind = peaks()
    frac = job_bytes / (ms * 1e-3) / 1e9 / (world * pk["hbm_gbs"])
    res = {"metric": METRIC, "value": round(world * T / (ms * 1e-3), 2), "unit": "tokens/s", "n_gpus": world,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None,
           "dtype": "q8_0 weights x fp16 MMA operands, fp32 accumulate; bf16 in/out",
           "data": "synthetic (seeded N(0,1) bf16 tokens, N(0,0.02) weights quantized to Q8_0)",
           "config": {"workload": f"{a.workload}: decode T={T}/GPU, H={H}, I={cfg.inter}, E={E}, top-{cfg.topk} "
                                  f"+ 1 shared, Q8_0, expert-parallel {E // world} experts/GPU",
                      "tokens_per_gpu": T, "global_batch": T * world, "parallelism": f"ep{world} (vfmoe_ep_forward: NCCL send/recv inside libvfmoe)",
                      "distinct_experts": n_distinct, "q8_layout": wf,
                      "l2": "256 MiB memset between timed steps, outside the step events"},
           # per vfmoe_ep_forward: router 2, plan 1, pack 1, shared expert 8 (fill, count, dispatch,
           # gather, tile plan, gate/up, down, combine), routed experts 7, final combine 1
           "gpu_launches": 20 * a.steps, "clocks": clk,
           "roofline": {"bound": "hbm", "kernel": "whole expert-parallel layer (all ranks)",
                        "achieved": round(job_bytes / (ms * 1e-3) / 1e9, 1), "peak": world * pk["hbm_gbs"],
                        "unit": "GB/s", "frac": round(frac, 4), "peak_source": pk_kind, "traffic": None},
           "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                   "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2, "ms_per_step": round(e2e_ms, 4)}}
    if extra is not None:
        res.update(extra)
    return res


def run_ours(a, rank, world, local_rank):
    import torch
    from vybforge_b200 import synth, _lib
    from vybforge_b200.moe import init
    import ctypes as C
    torch.cuda.set_device(local_rank)
    init(local_rank)
    cfg = synth.config(a.workload, tokens=a.tokens, fmt=a.fmt, seed=rank)
    if a.experts:
        cfg.n_experts = a.experts
    if cfg.fmt != "q8_0" or a.workload not in ("c1", "c4d"):
        raise SystemExit(f"workload {a.workload}/{cfg.fmt} not wired into bench yet")
    layer, xd, host, dev, (devl, wf) = build_ours(cfg, rank, a.q8_layout)
    T = cfg.tokens
    st = torch.cuda.current_stream()
    out = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    idx = torch.empty((T, cfg.topk), dtype=torch.int32, device="cuda")
    w = torch.empty((T, cfg.topk), dtype=torch.float32, device="cuda")
    ws = layer.workspace(T)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")   # > 126 MB L2
    for _ in range(max(3, a.warmup)):
        layer.forward(xd, out=out, idx=idx, w=w, workspace=ws)
    torch.cuda.synchronize()
    lib = layer.lib
    lib.vfmoe_profile_enable(layer.handle, 1)
    lib.vfmoe_profile_read(layer.handle, (C.c_double * 8)(), 8, None)  # reset
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    clocks = ClockSampler(local_rank)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    for i in range(a.steps):
        flush.zero_()
        ev[i][0].record(st)
        layer.forward(xd, out=out, idx=idx, w=w, workspace=ws)
        ev[i][1].record(st)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    step_ms = [s.elapsed_time(e) for s, e in ev]
    stage = (C.c_double * 8)()
    launches = C.c_int64(0)
    nf = lib.vfmoe_profile_read(layer.handle, stage, 8, C.byref(launches))
    lib.vfmoe_profile_enable(layer.handle, 0)
    ms = float(np.mean(step_ms))
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T / (ms * 1e-3)

    # e2e through the public API with pinned host buffers, copies inside the timed region
    xh = xd.cpu().pin_memory()
    oh = torch.empty((T, cfg.hidden), dtype=torch.bfloat16).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    xin = torch.empty_like(xd)
    for i in range(a.steps):
        flush.zero_()
        ev2[i][0].record(st)
        xin.copy_(xh, non_blocking=True)
        o = layer.forward(xin, out=out, workspace=ws)
        oh.copy_(o, non_blocking=True)
        ev2[i][1].record(st)
    torch.cuda.synchronize()
    e2e_ms = float(np.mean([s.elapsed_time(e) for s, e in ev2]))
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())

    idx_np = idx.cpu().numpy()
    n_distinct = len(np.unique(idx_np))
    layer_bytes, gu_bytes = algorithmic_bytes(cfg, n_distinct)
    pk, pk_kind = peaks()
    gu_ms = stage[2] / max(nf, 1)
    layer_gbs = layer_bytes / (ms * 1e-3) / 1e9
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9
    # traffic: dram read+write per launch, scaled from the ncu capture of the same kernel on the
    # 64-expert case (--profile-case q8_decode_e64): 1.006 (tiled) or 1.015 (rows) x algorithmic bytes
    roof = {"bound": "hbm", "kernel": "expert gate/up GEMV (Q8_0, fused SwiGLU)", "achieved": round(achieved, 1),
            "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
            "peak_source": pk_kind, "traffic": round(gu_bytes * GEMV_Q8_TRAFFIC_RATIO[wf]),
            "traffic_source": "ncu capture of the 64-expert case, scaled by algorithmic bytes",
            "algorithmic_bytes_per_launch": gu_bytes,
            "layer_hbm_frac": round(layer_gbs / pk["hbm_gbs"], 4),
            "stage_ms_per_step": {n: round(stage[i] / max(nf, 1), 4) for i, n in
                                  enumerate(["router", "dispatch_gather", "gate_up", "down", "combine"])}}
    res = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
           "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "q8_0 weights x fp16 MMA operands, fp32 accumulate; bf16 in/out",
           "data": "synthetic (seeded N(0,1) bf16 tokens, N(0,0.02) weights quantized to Q8_0)",
           "config": {"workload": f"{a.workload}: decode T={T}/GPU, H={cfg.hidden}, I={cfg.inter}, "
                                  f"E={cfg.n_experts}, top-{cfg.topk} + 1 shared, Q8_0",
                      "tokens_per_gpu": T, "global_batch": T * world, "parallelism":
                          "replicas" if world > 1 else "single",
                      "distinct_experts": n_distinct, "q8_layout": wf,
                      "l2": "256 MiB memset between timed steps, outside the step events"},
           "gpu_launches": int(launches.value), "clocks": clk, "roofline": roof,
           "e2e": {"value": round(world * T / (e2e_ms * 1e-3), 2), "unit": "tokens/s",
                   "h2d_bytes_per_step": T * cfg.hidden * 2, "d2h_bytes_per_step": T * cfg.hidden * 2,
                   "ms_per_step": round(e2e_ms, 4)}}
    if not a.no_extra and a.workload == "c1" and a.tokens is None and not a.experts:
        extra = {}
        ms1, st1, _, idx1 = time_layer(layer, xd[:1].contiguous(), a.steps, a.warmup, flush)
        l1b, gu1b = algorithmic_bytes(synth.config("c1", tokens=1), len(np.unique(idx1.cpu().numpy())))
        # the T=1 step without the library's per-stage events (an event between two
        # programmatic-dependent launches keeps the second from starting early: about 26 us here)
        ms1_plain = time_layer(layer, xd[:1].contiguous(), a.steps, a.warmup, flush, with_profile=False)[0]
        try:
            ms1_graph = time_graph(layer, xd[:1].contiguous(), a.steps, flush)
            ms32_graph = time_graph(layer, xd, a.steps, flush)
            extra["cuda_graph"] = {
                "note": "one vfmoe_forward recorded in a CUDA graph and replayed; eager time without the "
                        "library's per-stage events beside it",
                "t1": {"ms_per_step": round(ms1_graph, 4), "tokens_per_s": round(1 / (ms1_graph * 1e-3), 1),
                       "eager_ms_per_step": round(ms1_plain, 4)},
                "t32": {"ms_per_step": round(ms32_graph, 4), "tokens_per_s": round(32 / (ms32_graph * 1e-3), 1)}}
        except Exception as e:  # an extra must not cost the headline line
            extra["cuda_graph"] = {"error": str(e)[:300]}
        extra["c1_t1"] = {"tokens_per_s": round(1 / (ms1_plain * 1e-3), 1), "ms_per_step": round(ms1_plain, 4),
                          "layer_hbm_frac": round(l1b / (ms1_plain * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                          "with_stage_events": {
                              "note": "the same step timed with the library's per-stage events on (their split "
                                      "below, and the gate/up GEMV's own fraction)",
                              "ms_per_step": round(ms1, 4),
                              "gate_up_hbm_frac": round(gu1b / (st1["gate_up"] * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                              "stage_ms_per_step": {n: round(v, 4) for n, v in st1.items()}}}
        extra["c3_prefill_q8_0"] = prefill_extra(a, cfg, devl, wf, flush)
        res.update(extra)
    if rank == 0 and not a.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline_ours(cfg, host, dev, idx_np, a.cpu_budget_s)
    if not a.no_extra and a.workload == "c1" and a.tokens is None and not a.experts:
        del dev, devl
        layer.close()
        torch.cuda.empty_cache()
        res.update(stack_extra(a, rank, world, local_rank, flush))
        torch.cuda.empty_cache()
        res.update(exl3_extra(a, flush))
        torch.cuda.empty_cache()
        res.update(hc_extra(a, flush))
    return res


# ----------------------------------------------------------------------------- reference arm
def run_reference(a):
    """The reference algorithm on the host cores: the numpy restatement of
    native/glm53/moe_ref.py (router, per-expert f64 FFN, combine) with the Q8_0 decode of
    native/tools/q8_0_ref.py, on the same workload, metric and config as our arm.  Each step is a
    bounded sample of the workload (the first n tokens, n chosen so that warm-up + steps end within
    a few minutes); value and ms_per_step are the sample's own (no extrapolation)."""
    from oracle import moe_oracle as orc
    from vybforge_b200 import synth
    cfg = synth.config(a.workload, tokens=a.tokens, fmt=a.fmt, seed=0)
    x, w_r, bias, rng = synth.router_inputs(cfg)
    H, I, E, T = cfg.hidden, cfg.inter, cfg.n_experts, cfg.tokens
    idx, wt = orc.route(x, w_r, bias, cfg.topk)
    per_step_s = min(a.cpu_budget_s, 150.0 / max(1, a.steps + a.warmup))
    # Q8_0 expert bytes from a seeded stream per (expert, projection); the CPU time of the
    # dequant + f64 GEMMs does not depend on the values
    raw = {}

    def make(e):
        g = np.random.default_rng((cfg.seed, 5000 + e))
        raw[e] = tuple(np.ascontiguousarray(
            g.integers(0, 256, size=(r, c // 32, 34), dtype=np.uint8).reshape(r, -1)) for r, c in ((I, H), (I, H), (H, I)))
        for m in raw[e]:
            m.reshape(m.shape[0], -1, 34)[:, :, 0:2] = np.frombuffer(
                np.full(m.shape[0] * (m.shape[1] // 34), 6e-4, np.float16).tobytes(), np.uint8).reshape(
                m.shape[0], -1, 2)

    def get(e):
        if e not in raw:
            make(e)
        g, u, d = raw[e]
        return (orc.q8_0_expert_inout(g, I, H), orc.q8_0_expert_inout(u, I, H), orc.q8_0_expert_inout(d, H, I))
    # sample size: one untimed calibration step on the first token sets the cost per expert, then
    # the first n tokens whose experts fit the per-step budget
    for e in set(np.unique(idx[:1]).tolist()) | {E}:
        make(e)
    t0 = time.perf_counter()
    orc.moe_block_grouped(x[:1], w_r, bias, get, lambda: get(E), E, cfg.topk)
    per_expert = (time.perf_counter() - t0) / (len(np.unique(idx[:1])) + 1)
    n = 1
    while n < T and (len(np.unique(idx[:n + 1])) + 1) * per_expert <= per_step_s:
        n += 1
    need = sorted(set(np.unique(idx[:n]).tolist()) | {E})
    times = []
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        orc.moe_block_grouped(x[:n], w_r, bias, get, lambda: get(E), E, cfg.topk)
        if i >= a.warmup:
            times.append(time.perf_counter() - t0)
    dt = float(np.mean(times))
    v = n / dt
    cores = os.cpu_count()
    sample = (f"first {n} of {T} tokens ({len(need)} experts incl. shared) per step; numpy f64 dequant + GEMM per "
              f"expert on {cores} host threads ({cpu_model()}); value and ms_per_step are the sample's")
    return {"metric": METRIC, "impl": "reference", "value": round(v, 3), "unit": "tokens/s", "n_gpus": a.gpus,
            "steps": len(times), "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 3),
            "tokens_per_step": n, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded N(0,1) bf16 tokens; Q8_0 expert bytes from a seeded stream)",
            "config": {"workload": f"{a.workload}: decode T={T}/GPU, H={H}, I={I}, E={E}, top-{cfg.topk} "
                                   f"+ 1 shared, Q8_0", "tokens_per_gpu": T, "global_batch": T * a.gpus,
                       "parallelism": "host cores (reference CPU path)"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "cpu_model": cpu_model(), "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    a = args_parse()
    if a.profile_case:
        PROFILE_CASES[a.profile_case](a)
        print("ok")
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(a)), flush=True)
        return
    import torch
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local_rank))
    res = run_ours_ep(a, rank, world, local_rank) if world > 1 else run_ours(a, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
