"""Seeded synthetic workloads for the MoE layer configurations C0-C4.

No checkpoint or dataset is used: every input is drawn from a seeded generator
with the shapes and value distributions of the configuration being measured.

Draw order (fixed): x, router weight W_r, selection bias, [Zipf bias], then for
each expert e = 0..E-1 its gate, up and down matrices, then the shared expert.
x, W_r and the bias come from ``numpy.random.default_rng(seed)``.  Expert weights
come either from the same numpy stream (``weights="numpy"``, small shapes) or,
for the full-size configurations whose weights run to gigabytes, from a CUDA
``torch.Generator`` seeded per (seed, expert, projection) and quantized on the
GPU (``weights="cuda"``), so any single expert can be regenerated or read back
on its own.

Q8_0 matrices are stored as output rows (gate/up: [I][H], down: [H][I]).
EXL3 matrices are stored as trellis tiles [K/16][N/16][16*bits] of the (in, out)
matrix (gate/up: K=H, N=I; down: K=I, N=H), with fp16 suh [K] and svh [N].
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .quant import quantize_q8_0, round_bf16, q8_0_row_bytes, exl3_words

PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2


@dataclass
class LayerConfig:
    name: str
    hidden: int
    inter: int
    n_experts: int
    topk: int
    tokens: int
    fmt: str = "q8_0"          # "q8_0" | "exl3"
    exl3_bits: int = 3
    x_dtype: str = "bf16"      # "f32" | "bf16"
    zipf_s: float = 0.0        # 0 = plain N(0, 0.01) selection bias
    seed: int = 0
    extra: dict = field(default_factory=dict)


def config(name: str, tokens: int | None = None, fmt: str | None = None, seed: int = 0) -> LayerConfig:
    """The BASELINE configurations (one MoE layer each; C4 stacks four)."""
    big = dict(hidden=6144, inter=2048, n_experts=256, topk=8)
    if name == "c0":
        c = LayerConfig("c0", 1024, 512, 16, 4, tokens or 16, "q8_0", x_dtype="f32")
    elif name == "c1":
        c = LayerConfig("c1", tokens=tokens or 32, fmt="q8_0", **big)
    elif name == "c2":
        c = LayerConfig("c2", tokens=tokens or 32, fmt="exl3", **big)
    elif name == "c3":
        c = LayerConfig("c3", tokens=tokens or 4096, fmt=fmt or "q8_0", zipf_s=1.1, **big)
    elif name == "c4p":
        c = LayerConfig("c4p", tokens=tokens or 8192, fmt="q8_0", zipf_s=1.1, **big)
    elif name == "c4d":
        c = LayerConfig("c4d", tokens=tokens or 256, fmt="q8_0", **big)
    else:
        raise ValueError(name)
    if fmt is not None:
        c.fmt = fmt
    c.seed = seed
    return c


# ----------------------------------------------------------------------------- routing inputs
def router_inputs(cfg: LayerConfig, rng=None):
    """(x float32 [T,H] exactly representable in x_dtype, W_r f32 [E,H], bias f32 [E], rng)."""
    rng = rng if rng is not None else np.random.default_rng(cfg.seed)
    T, H, E = cfg.tokens, cfg.hidden, cfg.n_experts
    x = rng.standard_normal((T, H)).astype(np.float32)
    if cfg.x_dtype == "bf16":
        x = round_bf16(x)
    w_r = rng.normal(0.0, 0.02, (E, H)).astype(np.float32)
    bias = rng.normal(0.0, 0.01, E).astype(np.float32)
    return x, w_r, bias, rng


def zipf_targets(n_experts: int, tokens: int, topk: int, s: float, rng) -> np.ndarray:
    """Expected selection count per expert: proportional to rank^-s over a seeded
    random rank order, scaled to tokens*topk selections, each capped at `tokens`
    (an expert can be chosen at most once per token); the excess is
    redistributed over the uncapped experts in proportion."""
    ranks = rng.permutation(n_experts) + 1
    p = ranks.astype(np.float64) ** (-s)
    total = float(tokens * topk)
    tgt = np.zeros(n_experts)
    free = np.ones(n_experts, dtype=bool)
    remaining = total
    for _ in range(n_experts):
        t = p * free
        t = t / t.sum() * remaining
        over = free & (t > tokens)
        if not over.any():
            tgt[free] = t[free]
            break
        tgt[over] = tokens
        remaining -= tokens * over.sum()
        free &= ~over
    return tgt


def calibrate_zipf_bias(logits, base_bias, topk, targets, iters=400):
    """Selection bias b (added to sigmoid scores for top-k only) whose realized
    per-expert selection counts on these logits follow ``targets``.

    Multiplicative fixed-point iteration on b; deterministic for given inputs.
    The routing weights use the raw sigmoid scores, so b changes only which
    experts are picked (native/glm53/moe_ref.py:72-77 semantics)."""
    scores = 1.0 / (1.0 + np.exp(-logits))
    T, E = scores.shape
    b = base_bias.astype(np.float64).copy()
    tgt = np.maximum(targets, 0.5)
    lr = 0.5
    for it in range(iters):
        choice = scores + b[None, :]
        sel = np.argpartition(-choice, topk - 1, axis=1)[:, :topk]
        cnt = np.bincount(sel.reshape(-1), minlength=E).astype(np.float64)
        err = np.log(tgt) - np.log(np.maximum(cnt, 0.5))
        if np.abs(err).max() < 0.02:
            break
        b += lr * 0.05 * np.clip(err, -2, 2)
    return b.astype(np.float32)


def zipf_router_inputs(cfg: LayerConfig):
    """x, W_r and a selection bias whose realized expert popularity on these tokens follows
    Zipf(cfg.zipf_s) over a seeded random rank order (BASELINE C3/C4 prefill).

    x and W_r are the config's ordinary draws; the bias starts from the ordinary
    N(0, 0.01) draw and is calibrated on the f64 logits of these very tokens, so the
    router itself is the unmodified reference router (selection-only bias).
    Returns (x, w_r, bias, targets, rng)."""
    x, w_r, bias0, rng = router_inputs(cfg)
    logits = x.astype(np.float64) @ w_r.astype(np.float64).T
    tgt = zipf_targets(cfg.n_experts, cfg.tokens, cfg.topk, cfg.zipf_s, np.random.default_rng(cfg.seed + 7))
    bias = calibrate_zipf_bias(logits, bias0, cfg.topk, tgt)
    return x, w_r, bias, tgt, rng


def stack_inputs(cfg: LayerConfig, n_layers: int, calib_tokens: int = 2048):
    """Inputs of a pre-norm stack of `n_layers` MoE layers of cfg's shape (BASELINE C4).

    Returns (x, norm_ws, routers): x the stack input (cfg's ordinary token draw), norm_ws
    a list of fp32 [H] RMSNorm weights 1 + N(0, 0.02), routers a list of (w_r, bias,
    load) per layer.  Layer l's router (W_r ~ N(0, 0.02), bias ~ N(0, 0.01)) is drawn
    from the stream seeded (seed, 1000 + l).

    Everything fitted to tokens is fitted on a calibration batch drawn from its own stream
    (seed, 3000), disjoint from x, as a server fits its placement on earlier traffic: with
    cfg.zipf_s > 0 the selection bias is calibrated (as in zipf_router_inputs) on the first
    `calib_tokens` calibration rows of RMSNorm_l, and load is the layer's selection count per
    expert over a calibration batch of x's size (the expert-placement input).  Layers after the
    first see the residual stream, so their realized popularity is only approximately Zipf and
    their load an estimate."""
    x, _, _, rng = router_inputs(cfg)
    norm_ws = [(1.0 + rng.normal(0.0, 0.02, cfg.hidden)).astype(np.float32) for _ in range(n_layers)]
    xc = np.random.default_rng((cfg.seed, 3000)).standard_normal(x.shape).astype(np.float32)
    if cfg.x_dtype == "bf16":
        xc = round_bf16(xc)
    routers = []
    for l in range(n_layers):
        r_l = np.random.default_rng((cfg.seed, 1000 + l))
        w_r = r_l.normal(0.0, 0.02, (cfg.n_experts, cfg.hidden)).astype(np.float32)
        bias0 = r_l.normal(0.0, 0.01, cfg.n_experts).astype(np.float32)
        if cfg.zipf_s > 0:
            xs = xc[:calib_tokens].astype(np.float64)
            h = xs / np.sqrt(np.mean(xs * xs, axis=1, keepdims=True) + 1e-5) * norm_ws[l]
            logits = h @ w_r.astype(np.float64).T
            tgt = zipf_targets(cfg.n_experts, len(xs), cfg.topk, cfg.zipf_s, np.random.default_rng((cfg.seed, 2000 + l)))
            bias = calibrate_zipf_bias(logits, bias0, cfg.topk, tgt)
        else:
            bias = bias0
        routers.append((w_r, bias, selection_counts(xc, norm_ws[l], w_r, bias, cfg.topk)))
    return x, norm_ws, routers


def selection_counts(x, norm_w, w_r, bias, topk, chunk=2048):
    """Per-expert selection counts of RMSNorm(x) under a router (fp32 logits; used only to
    estimate expert load for placement, so near ties do not matter)."""
    cnt = np.zeros(w_r.shape[0], dtype=np.int64)
    wt = np.ascontiguousarray(w_r.T, dtype=np.float32)
    for a in range(0, x.shape[0], chunk):
        xs = x[a:a + chunk].astype(np.float32)
        h = xs / np.sqrt(np.mean(xs * xs, axis=1, keepdims=True) + 1e-5) * norm_w
        s = 1.0 / (1.0 + np.exp(-(h @ wt)))
        sel = np.argpartition(-(s + bias[None, :]), topk - 1, axis=1)[:, :topk]
        cnt += np.bincount(sel.reshape(-1), minlength=w_r.shape[0])
    return cnt


def realized_counts(idx, n_experts):
    return np.bincount(np.asarray(idx).reshape(-1), minlength=n_experts)


# ----------------------------------------------------------------------------- experts, numpy
def _proj_shape(cfg: LayerConfig, proj: int):
    """(rows=out, cols=in) of a projection in Q8_0 row storage."""
    H, I = cfg.hidden, cfg.inter
    return (I, H) if proj in (PROJ_GATE, PROJ_UP) else (H, I)


def expert_q8_numpy(cfg: LayerConfig, rng):
    """All E+1 experts (last = shared) as Q8_0 bytes, drawn from the numpy stream.

    Returns dict proj -> uint8 [E+1, rows, row_bytes]."""
    E = cfg.n_experts
    out = {}
    for proj in (PROJ_GATE, PROJ_UP, PROJ_DOWN):
        rows, cols = _proj_shape(cfg, proj)
        out[proj] = np.empty((E + 1, rows, q8_0_row_bytes(cols)), dtype=np.uint8)
    for e in range(E + 1):
        for proj in (PROJ_GATE, PROJ_UP, PROJ_DOWN):
            rows, cols = _proj_shape(cfg, proj)
            w = rng.normal(0.0, 0.02, (rows, cols)).astype(np.float32)
            out[proj][e] = quantize_q8_0(w)
    return out


def expert_exl3_numpy(cfg: LayerConfig, rng):
    """All E+1 experts as EXL3 (trellis uint16 [E+1, K/16, N/16, 16*bits],
    suh fp16 [E+1, K], svh fp16 [E+1, N]) per projection (in, out) orientation."""
    E, H, I, bits = cfg.n_experts, cfg.hidden, cfg.inter, cfg.exl3_bits
    words = exl3_words(bits)
    out = {}
    for proj in (PROJ_GATE, PROJ_UP, PROJ_DOWN):
        k, n = (H, I) if proj != PROJ_DOWN else (I, H)
        out[proj] = (np.empty((E + 1, k // 16, n // 16, words), np.uint16),
                     np.empty((E + 1, k), np.float16), np.empty((E + 1, n), np.float16))
    for e in range(E + 1):
        for proj in (PROJ_GATE, PROJ_UP, PROJ_DOWN):
            tr, suh, svh = out[proj]
            k, n = suh.shape[1], svh.shape[1]
            tr[e] = rng.integers(0, 1 << 16, size=tr.shape[1:], dtype=np.uint32).astype(np.uint16)
            suh[e] = np.where(rng.random(k) < 0.5, -1.0, 1.0).astype(np.float16)
            sgn = np.where(rng.random(n) < 0.5, -1.0, 1.0)
            svh[e] = (sgn * rng.uniform(0.01, 0.03, n)).astype(np.float16)
    return out


# ----------------------------------------------------------------------------- experts, CUDA
def cuda_seed(cfg: LayerConfig, e: int, proj: int, layer: int = 0) -> int:
    return int((int(cfg.seed) * 1_000_003 + int(layer) * 7919 + int(e) * 3 + int(proj)) & 0x7FFFFFFFFFFF)


def expert_q8_cuda(cfg: LayerConfig, lib, device="cuda", layer: int = 0, experts=None):
    """Experts as Q8_0 on the GPU: torch.randn per (expert, projection) from a CUDA
    generator seeded by (seed, layer, expert, projection), times 0.02, quantized by the
    library's ``vfmoe_q8_0_quantize`` kernel (bit-identical to ``quantize_q8_0``).

    experts: ids to generate (E = the shared expert); default all 0..E.  Any subset
    reproduces exactly the same bytes for its experts.
    Returns dict proj -> torch.uint8 [len(experts), rows, row_bytes] on `device`."""
    import torch
    E = cfg.n_experts
    ids = list(range(E + 1)) if experts is None else list(experts)
    out = {}
    g = torch.Generator(device=device)
    for proj in (PROJ_GATE, PROJ_UP, PROJ_DOWN):
        rows, cols = _proj_shape(cfg, proj)
        buf = torch.empty((len(ids), rows, q8_0_row_bytes(cols)), dtype=torch.uint8, device=device)
        tmp = torch.empty((rows, cols), dtype=torch.float32, device=device)
        for i, e in enumerate(ids):
            g.manual_seed(cuda_seed(cfg, e, proj, layer))
            torch.randn((rows, cols), generator=g, out=tmp)
            tmp.mul_(0.02)
            lib.q8_0_quantize(tmp, buf[i])
        out[proj] = buf
    return out


def expert_exl3_cuda(cfg: LayerConfig, device="cuda", layer: int = 0):
    """All E+1 experts as EXL3 tensors on the GPU (uniform random trellis words,
    suh = +-1, svh = +-U(0.01, 0.03)), seeded per (expert, projection)."""
    import torch
    E, H, I, bits = cfg.n_experts, cfg.hidden, cfg.inter, cfg.exl3_bits
    words = exl3_words(bits)
    out = {}
    g = torch.Generator(device=device)
    for proj in (PROJ_GATE, PROJ_UP, PROJ_DOWN):
        k, n = (H, I) if proj != PROJ_DOWN else (I, H)
        tr = torch.empty((E + 1, k // 16, n // 16, words), dtype=torch.int16, device=device)
        suh = torch.empty((E + 1, k), dtype=torch.float16, device=device)
        svh = torch.empty((E + 1, n), dtype=torch.float16, device=device)
        for e in range(E + 1):
            g.manual_seed(cuda_seed(cfg, e, proj, layer))
            tr[e].random_(-32768, 32768, generator=g)
            suh[e] = torch.where(torch.rand(k, generator=g, device=device) < 0.5, -1.0, 1.0).half()
            sgn = torch.where(torch.rand(n, generator=g, device=device) < 0.5, -1.0, 1.0)
            svh[e] = (sgn * (0.01 + 0.02 * torch.rand(n, generator=g, device=device))).half()
        out[proj] = (tr, suh, svh)
    return out
