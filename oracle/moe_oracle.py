"""CPU oracle for the GLM-style MoE layer -- TEST INFRASTRUCTURE ONLY.

This module is the checker that the CUDA path is compared against.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs may import it; the product (``vybforge_b200``) never does.

It restates, in numpy with float64 arithmetic, the reference algorithms of
rickenator/VybForge for this path (paths relative to the reference project):

* router            native/glm53/moe_ref.py:64-78   (``sigmoid``, ``route``)
* clamped SwiGLU    native/glm53/moe_ref.py:81-89   (``swiglu``, ``ffn``)
* MoE block         native/glm53/moe_ref.py:92-112  (``moe_block``)
* Q8_0 decode       native/tools/q8_0_ref.py:50-56  (``q8_0_ours``)
* EXL3 value decode native/exl3/exl3_ref.py:37-47   (``decode_mcg``)
* EXL3 reconstruct  native/exl3/exl3_ref.py:58-63, 84-120
* RMSNorm           native/kernels/rmsnorm.vyb (y = x * w / sqrt(mean(x^2) + eps))
* hyper-connections native/glm53/hc_ref.py:27-63 (``hc_mix``, ``hc_apply``); the engine's
                    hc_glue / hc_apply, native/glm53/glm_engine.vyb:437-612, :783-809

Deliberate differences from the reference, each required by the task spec:

* top-k uses ``np.argsort(-choice, kind="stable")`` so ties go to the lowest
  expert index.  The reference uses the default (unstable) sort at
  moe_ref.py:74, while its GPU kernel scans experts ascending with a strict
  ``>`` (native/kernels/moe.vyb:69) -- i.e. lowest index wins.  The stable
  sort reproduces the kernel rule.
* H, I, E, k are parameters instead of module constants (moe_ref.py:25-30).
* ``moe_block_grouped`` computes each expert once over all of its tokens
  (dequantize one expert, matmul its gathered rows, scatter) instead of the
  per-token loop of moe_ref.py:102-110; the arithmetic per (token, lane) is
  the same f64 math, so results agree with ``moe_block`` to f64 rounding.
* EXL3 at 3 bits/weight uses the bitstream layout defined in
  ``exl3_windows_3bpw`` (the reference only has 4 bpw); 4 bpw uses the
  reference's verified slot composition table, or its closed form
  ``exl3_windows_4bpw_words`` (equal on every slot; the GPU path uses the latter).

Parity pinning: ``tests/test_oracle.py`` checks this module against the
reference's committed golden data (native/glm53/prep/ref_{out,idx,w}.f32,
the EXL3 known answer decode_mcg(0) = 1.84375) and against golden vectors in
``tests/golden/`` produced by importing the reference's own Python modules
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np

SCALE = 2.5           # routed_scaling_factor, moe_ref.py:29
SWIGLU_LIMIT = 10.0   # moe_ref.py:30
Q8_BLOCK = 32         # values per Q8_0 block
Q8_BYTES = 34         # fp16 d + 32 int8 (native/kernels/q8_0.vyb:6, GGUF block_q8_0)


# --------------------------------------------------------------------------- router
def sigmoid(x):
    """moe_ref.py:64-65."""
    return 1.0 / (1.0 + np.exp(-x))


def router_logits(x, w_r):
    """logits = x . W_r^T in float64 (moe_ref.py:71).  x [T,H], w_r [E,H]."""
    return np.asarray(x, dtype=np.float64) @ np.asarray(w_r, dtype=np.float64).T


def route(x, w_r, bias, topk, scale=SCALE, logits=None):
    """Sigmoid + selection-bias top-k router (moe_ref.py:68-78).

    Returns ``(idx int32 [T,k], w float64 [T,k])``.  ``idx`` is ordered by
    descending choice = sigmoid(logit) + bias with the lowest expert index
    first among equal choices; ``w`` is the RAW sigmoid score of each selected
    expert renormalised over the selection and multiplied by ``scale``.
    """
    if logits is None:
        logits = router_logits(x, w_r)
    scores = sigmoid(logits)
    choice = scores + np.asarray(bias, dtype=np.float64)[None, :]
    idx = np.argsort(-choice, axis=-1, kind="stable")[:, :topk]
    w = np.take_along_axis(scores, idx, axis=-1)
    w = w / (w.sum(axis=-1, keepdims=True) + 1e-20)
    w = w * scale
    return idx.astype(np.int32), w


# --------------------------------------------------------------------------- expert FFN
def swiglu(g, u, limit=SWIGLU_LIMIT):
    """Clamped SwiGLU (moe_ref.py:81-84): silu(min(g, L)) * clip(u, -L, L)."""
    g = np.minimum(g, limit)
    u = np.clip(u, -limit, limit)
    return (g * sigmoid(g)) * u


def ffn(x, wg, wu, wd, limit=SWIGLU_LIMIT):
    """moe_ref.py:87-89 with (in, out) weight layout: wg/wu [H,I], wd [I,H]."""
    return swiglu(x @ wg, x @ wu, limit) @ wd


def moe_block(x, w_r, bias, expert_w, shared_w, topk, scale=SCALE, limit=SWIGLU_LIMIT):
    """Per-token restatement of moe_ref.py:92-112 (small shapes only).

    expert_w: callable or dict e -> (wg, wu, wd) in (in, out) layout.
    """
    x = np.asarray(x, dtype=np.float64)
    idx, w = route(x, w_r, bias, topk, scale)
    T, H = x.shape
    get = expert_w if callable(expert_w) else expert_w.__getitem__
    out = np.zeros((T, H), dtype=np.float64)
    for t in range(T):
        for lane in range(topk):
            wg, wu, wd = get(int(idx[t, lane]))
            out[t] += w[t, lane] * ffn(x[t:t + 1], wg, wu, wd, limit)[0]
    out += ffn(x, *shared_w, limit=limit)
    return out, idx, w


def dispatch_order(idx, n_experts):
    """Canonical permutation (expert ascending, token ascending).

    Follows the host gather of native/glm53/glm_engine.vyb:2827-2845: for each
    expert e in ascending order, the tokens t (ascending) with idx[t, l] == e.
    Returns (perm_token int32 [T*k], perm_lane int32 [T*k], offsets int64 [E+1]).
    """
    idx = np.asarray(idx)
    T, k = idx.shape
    flat_e = idx.reshape(-1).astype(np.int64)
    flat_t = np.repeat(np.arange(T, dtype=np.int64), k)
    flat_l = np.tile(np.arange(k, dtype=np.int64), T)
    order = np.lexsort((flat_t, flat_e))          # primary expert, secondary token
    counts = np.bincount(flat_e, minlength=n_experts)
    offsets = np.zeros(n_experts + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    return flat_t[order].astype(np.int32), flat_l[order].astype(np.int32), offsets


def moe_block_grouped(x, w_r, bias, get_expert, get_shared, n_experts, topk,
                      scale=SCALE, limit=SWIGLU_LIMIT, route_out=None):
    """Expert-grouped restatement of moe_ref.py:92-112 for large shapes.

    ``get_expert(e)`` / ``get_shared()`` return (wg [H,I], wu [H,I], wd [I,H])
    float64 on demand, so only the selected experts are ever dequantized.
    Per (token, lane) the math is moe_ref's: out[t] = sum_l w[t,l]*ffn_e(x[t])
    + ffn_shared(x[t]).  Lanes are accumulated in lane order per token.
    """
    x = np.asarray(x, dtype=np.float64)
    T, H = x.shape
    if route_out is None:
        idx, w = route(x, w_r, bias, topk, scale)
    else:
        idx, w = route_out
    perm_t, perm_l, offs = dispatch_order(idx, n_experts)
    y_lane = np.zeros((T, topk, H), dtype=np.float64)
    for e in range(n_experts):
        a, b = int(offs[e]), int(offs[e + 1])
        if a == b:
            continue
        toks = perm_t[a:b]
        wg, wu, wd = get_expert(e)
        y_lane[toks, perm_l[a:b]] = ffn(x[toks], wg, wu, wd, limit)
    out = np.zeros((T, H), dtype=np.float64)
    for lane in range(topk):
        out += w[:, lane:lane + 1] * y_lane[:, lane]
    out += ffn(x, *get_shared(), limit=limit)
    return out, idx, w


def rmsnorm(x, weight, eps=1e-5):
    """native/kernels/rmsnorm.vyb: y = x * w / sqrt(mean(x^2) + eps), f64."""
    x = np.asarray(x, dtype=np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * r * np.asarray(weight, dtype=np.float64)[None, :]


def moe_stack(x, layers, eps=1e-5, round_act=None):
    """Pre-norm MoE stack: x <- x + MoE_l(RMSNorm_l(x)) for each layer.

    layers: list of (norm_w, run) where run(h) -> (y, idx, w) is one MoE layer
    (e.g. a closure over ``moe_block_grouped``).  round_act, if given, is applied to
    every activation the GPU stores (normed input, layer output, residual stream),
    mirroring bf16 activations.  Returns (x, per-layer list of (h, y, idx))."""
    rnd = round_act if round_act is not None else (lambda a: a)
    x = rnd(np.asarray(x, dtype=np.float64))
    trace = []
    for norm_w, run in layers:
        h = rnd(rmsnorm(x, norm_w, eps))
        y, idx, _ = run(h)
        y = rnd(y)
        x = rnd(x + y)
        trace.append((h, y, idx))
    return x, trace


# --------------------------------------------------------------------------- Q8_0
def dequant_q8_0(raw, rows, k):
    """Q8_0 rows -> float64 [rows, k] (native/tools/q8_0_ref.py:50-56).

    raw: uint8 bytes, rows of k/32 blocks; block = fp16 d at +0, int8 q[32] at +2.
    value = d * q, computed exactly in float64.
    """
    nb = k // Q8_BLOCK
    b = np.frombuffer(np.ascontiguousarray(raw).tobytes(), np.uint8).reshape(rows * nb, Q8_BYTES)
    d = b[:, 0:2].copy().view("<f2").astype(np.float64)[:, 0]
    qs = b[:, 2:Q8_BYTES].copy().view(np.int8).astype(np.float64)
    return (qs * d[:, None]).reshape(rows, k)


def q8_0_expert_inout(raw_rows_out, n_out, k_in):
    """Q8_0 matrix stored as [out rows][in] -> float64 (in, out) layout for ffn()."""
    return dequant_q8_0(raw_rows_out, n_out, k_in).T


def q8_0_tile(raw):
    """GGUF Q8_0 rows -> the stage-tiled byte order (VFMOE_WFMT_Q8_0_TILED, this library's
    load-time layout; the reference has no counterpart and reads the rows in place).

    raw: uint8 [..., rows, k/32*34], rows % 64 == 0, k % 256 == 0.  Tiles of 64 rows x 256 K
    (64 x 272 B, each tile row = that row's 8 blocks), tile (rt, kr) at ((rt * k/256) + kr)
    * 17408.  Returns uint8 of raw's shape."""
    raw = np.ascontiguousarray(raw)
    rows, rb = raw.shape[-2], raw.shape[-1]
    kr = rb // 272
    t = raw.reshape(-1, rows // 64, 64, kr, 272).transpose(0, 1, 3, 2, 4)
    return np.ascontiguousarray(t).reshape(raw.shape)


def q8_0_untile(tiled):
    """Inverse of q8_0_tile."""
    tiled = np.ascontiguousarray(tiled)
    rows, rb = tiled.shape[-2], tiled.shape[-1]
    kr = rb // 272
    t = tiled.reshape(-1, rows // 64, kr, 64, 272).transpose(0, 1, 3, 2, 4)
    return np.ascontiguousarray(t).reshape(tiled.shape)


# --------------------------------------------------------------------------- EXL3
MCG_MUL = 0xCBAC1FED
MCG_AND = 0x8FFF8FFF
MCG_XOR = 0x3B603B60
R_SCALE = 0.08838834764831845  # 1/sqrt(128), exl3_ref.py:35


def decode_mcg(w16):
    """16-bit windows -> fp16 values (exl3_ref.py:37-47).

    prod = w16 * 0xCBAC1FED mod 2^32; y = (prod & 0x8FFF8FFF) ^ 0x3B603B60;
    value = fp16(y & 0xFFFF) + fp16(y >> 16) rounded to fp16.  Both halves
    lie in [0.125, 2) in magnitude, so the float32 sum is exact and the single
    rounding to fp16 equals a hardware fp16 add.
    """
    w = np.asarray(w16).astype(np.uint32)
    prod = w * np.uint32(MCG_MUL)                      # uint32 arithmetic wraps mod 2^32
    y = (prod & np.uint32(MCG_AND)) ^ np.uint32(MCG_XOR)
    lo = (y & np.uint32(0xFFFF)).astype(np.uint16).view(np.float16)
    hi = (y >> np.uint32(16)).astype(np.uint16).view(np.float16)
    return (lo.astype(np.float32) + hi.astype(np.float32)).astype(np.float16)


def exl3_windows_3bpw_bits(tiles):
    """3-bpw window extraction, bit by bit (the layout this build defines; no reference one exists).

    tiles: uint16 [..., 48] -- one 16x16 tile = 768 bits, LSB-first in each word.
    Window j (j = 0..255) is the 16 bits starting at bit 3*j of the tile's
    circular bitstream: w16 = sum_i bit[(3j + i) mod 768] << i.
    Window j decodes the weight at tile slot (row r = j % 16, col c = j // 16):
    the stream runs down each output column, so the 16 input rows of one output
    column are 16 consecutive windows.
    Returns uint16 [..., 16 (r), 16 (c)].
    """
    t = np.asarray(tiles).astype(np.uint64)
    lead = t.shape[:-1]
    assert t.shape[-1] == 48
    bits = ((t[..., :, None] >> np.arange(16, dtype=np.uint64)) & np.uint64(1)).reshape(*lead, 768)
    j = np.arange(256)
    pos = (3 * j[:, None] + np.arange(16)[None, :]) % 768           # [256, 16]
    w = (bits[..., pos] << np.arange(16, dtype=np.uint64)).sum(axis=-1)  # [..., 256]
    w = w.astype(np.uint16)
    # j = 16*c + r  ->  [..., c, r] -> transpose to [..., r, c]
    return np.swapaxes(w.reshape(*lead, 16, 16), -1, -2)

def exl3_windows_3bpw(tiles):
    """Same windows as `exl3_windows_3bpw_bits`, from whole words: window j starts in word
    (3j) // 16 at bit (3j) % 16 <= 15, so words (3j)//16 and the next one (circularly) hold
    all 16 of its bits.  Memory O(windows) instead of O(bits); used for full-size matrices."""
    t = np.asarray(tiles)
    if t.dtype == np.int16:
        t = t.view(np.uint16)
    lead = t.shape[:-1]
    assert t.shape[-1] == 48
    j = np.arange(256)
    w0 = (3 * j) // 16
    sh = ((3 * j) % 16).astype(np.uint32)
    t32 = t.astype(np.uint32)
    v = (t32[..., w0] | (t32[..., (w0 + 1) % 48] << np.uint32(16))) >> sh
    w = (v & np.uint32(0xFFFF)).astype(np.uint16)
    return np.swapaxes(w.reshape(*lead, 16, 16), -1, -2)


def exl3_windows_4bpw(tiles, slot_nibble, slot_pos):
    """4-bpw window composition from the reference's verified slot table.

    Follows exl3_ref.py:97-107: nibble m of the tile stream = bits [4m, 4m+4)
    of the 64 words (LSB-first); slot s = (r, c) has window
    w16 = sum_i nib[slot_nibble[s, i]] << (4 * slot_pos[s, i]).
    slot_nibble / slot_pos: int [256, 4], slots ordered row-major (s = 16r + c).
    Returns uint16 [..., 16, 16].
    """
    t = np.asarray(tiles).astype(np.uint32)
    lead = t.shape[:-1]
    assert t.shape[-1] == 64
    nib = ((t[..., :, None] >> (4 * np.arange(4, dtype=np.uint32))) & np.uint32(0xF)).reshape(*lead, 256)
    w = np.zeros((*lead, 256), dtype=np.uint32)
    for i in range(4):
        w |= nib[..., slot_nibble[:, i]] << (4 * slot_pos[:, i]).astype(np.uint32)
    return w.astype(np.uint16).reshape(*lead, 16, 16)


def exl3_windows_4bpw_words(tiles):
    """4-bpw windows in closed form (equal to ``exl3_windows_4bpw`` with the reference's slot
    table, checked on every slot by tests/test_oracle.py).  Tile words w[0..63] (uint16);
    output column c takes four 32-bit pairs v_j = A_j | B_j << 16, j = 0..3:
      c <  8:  A_j = w[8c + 2j + 1], B_j = w[(8c + 2j - 2) mod 64]
      c >= 8:  A_j = w[8(c-8) + 2j], B_j = w[8(c-8) + 2j + 1]
    and the window of row 2j + (9, 8, 1, 0)[t] is bits [4t, 4t + 16) of v_j.
    Returns uint16 [..., 16, 16] (row r, column c)."""
    t = np.asarray(tiles)
    if t.dtype == np.int16:
        t = t.view(np.uint16)
    t = t.astype(np.uint32)
    lead = t.shape[:-1]
    assert t.shape[-1] == 64
    out = np.zeros((*lead, 16, 16), np.uint32)
    for c in range(16):
        for j in range(4):
            if c < 8:
                a, b = t[..., 8 * c + 2 * j + 1], t[..., (8 * c + 2 * j - 2) % 64]
            else:
                a, b = t[..., 8 * (c - 8) + 2 * j], t[..., 8 * (c - 8) + 2 * j + 1]
            v = a | (b << np.uint32(16))
            for tt, r0 in enumerate((9, 8, 1, 0)):
                out[..., r0 + 2 * j, c] = (v >> np.uint32(4 * tt)) & np.uint32(0xFFFF)
    return out.astype(np.uint16)


def hadamard128():
    """Natural-order Sylvester H_128 (exl3_ref.py:58-63)."""
    h = np.ones((1, 1), dtype=np.float64)
    while h.shape[0] < 128:
        h = np.block([[h, h], [h, -h]])
    return h


def exl3_what(trellis, bits, slot_table=None):
    """Rotated-basis matrix W^ [K, N] (float64 of fp16 values) from the trellis.

    trellis: uint16 [K/16, N/16, 16*bits].  Tile (kb, nb) covers input rows
    16kb..16kb+15 and output columns 16nb..16nb+15 (exl3_ref.py:109-115).
    """
    tr = np.asarray(trellis)
    if tr.dtype == np.int16:
        tr = tr.view(np.uint16)
    kb, nb, words = tr.shape
    if bits == 3:
        w16 = exl3_windows_3bpw(tr)
    elif bits == 4:
        # the reference's slot table when given, else its closed form (pinned equal)
        w16 = exl3_windows_4bpw(tr, *slot_table) if slot_table is not None else exl3_windows_4bpw_words(tr)
    else:
        raise ValueError(f"unsupported EXL3 bits {bits}")
    vals = decode_mcg(w16).astype(np.float64)             # [kb, nb, 16, 16]
    return vals.transpose(0, 2, 1, 3).reshape(kb * 16, nb * 16)


def dequant_exl3(trellis, suh, svh, bits, slot_table=None):
    """Original-basis W [K, N] in float64 (exl3_ref.py:84-120).

    W = diag(suh) . Hb . W^ . Hb . diag(svh), Hb = blockdiag(H128 / sqrt(128)).
    The reference evaluates this in float32 and rounds W to fp16; the oracle
    keeps float64 so the only rounding left is the GPU's own.
    """
    return dequant_exl3_from_what(exl3_what(trellis, bits, slot_table), suh, svh)


def dequant_exl3_from_what(what, suh, svh):
    """The reconstruction step of dequant_exl3 alone (exl3_ref.py:116-120): W from the decoded
    rotated-basis values W^ [K, N], float64."""
    what = np.asarray(what, np.float64)
    k, n = what.shape
    hs = hadamard128() * R_SCALE
    # per 128x128 block (i, j): Hs . W^[i, j] . Hs
    w = (hs @ what.reshape(k // 128, 128, n)).reshape(k, n // 128, 128) @ hs
    w = w.reshape(k, n)
    return w * np.asarray(suh, np.float64)[:, None] * np.asarray(svh, np.float64)[None, :]


# --------------------------------------------------------------------------- hyper-connections
HC_EPS = 1e-6          # hc_eps (hc_ref.py:23)
SINKHORN_ITERS = 20    # hc_sinkhorn_iters (hc_ref.py:24)


def hc_mix(streams, fn, base, scale, rms_eps, hc_eps=HC_EPS, sinkhorn_iters=SINKHORN_ITERS):
    """Multi-stream mix of hc_ref.py:31-57 in float64.

    streams (R, HC, D); fn (24, HC*D) (out, in); base (24,); scale (3,).
    Returns (post (R, HC), comb (R, HC, HC), collapsed (R, D), pre (R, HC))."""
    streams = np.asarray(streams, np.float64)
    R, hc, D = streams.shape
    flat = streams.reshape(R, hc * D)
    flat = flat / np.sqrt(np.mean(flat * flat, axis=-1, keepdims=True) + rms_eps)
    mv = flat @ np.asarray(fn, np.float64).T
    base = np.asarray(base, np.float64)
    s0, s1, s2 = (float(v) for v in scale)
    pre = sigmoid(mv[:, :hc] * s0 + base[:hc]) + hc_eps
    post = 2.0 * sigmoid(mv[:, hc:2 * hc] * s1 + base[hc:2 * hc])
    comb = mv[:, 2 * hc:].reshape(R, hc, hc) * s2 + base[2 * hc:].reshape(hc, hc)
    e = np.exp(comb - comb.max(axis=-1, keepdims=True))
    comb = e / e.sum(axis=-1, keepdims=True) + hc_eps
    comb = comb / (comb.sum(axis=-2, keepdims=True) + hc_eps)
    for _ in range(sinkhorn_iters - 1):
        comb = comb / (comb.sum(axis=-1, keepdims=True) + hc_eps)
        comb = comb / (comb.sum(axis=-2, keepdims=True) + hc_eps)
    collapsed = (pre[:, :, None] * streams).sum(axis=1)
    return post, comb, collapsed, pre


def hc_apply(streams, y, post, comb):
    """Residual update of hc_ref.py:60-63: out[r, h] = post[r, h] y[r] + sum_j comb[r, j, h] streams[r, j]."""
    streams = np.asarray(streams, np.float64)
    return (np.asarray(post, np.float64)[:, :, None] * np.asarray(y, np.float64)[:, None, :]
            + np.einsum("rjh,rjd->rhd", np.asarray(comb, np.float64), streams))

