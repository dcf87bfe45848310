"""GPU checks of the parity objects and numerics that the layer-level tests reach only indirectly.

* The dispatch permutation (north_star: "Expert ids and the permutation must be bit-exact"):
  vfmoe_dispatch runs the forward's own count + dispatch kernels; perm_tok, the lane of every
  permuted row and the expert offsets must equal the oracle's canonical order (experts ascending,
  tokens ascending; native/glm53/glm_engine.vyb:2827-2845) at C0, C1 T=32 and C3 T=4096 Zipf.
* The clamped SwiGLU (native/glm53/moe_ref.py:81-84): weights scaled so that the oracle sees
  g > 10 and |u| > 10 on a large share of the entries, through the decode GEMV, the tcgen05 GEMM
  and both EXL3 kernels.
* The fp32 clause of the tolerance (rel-L2 1e-4) on fp32-in, fp32-out layers, which run the
  split-precision decode GEMV at every T.
* The device-error path: a bounded wait that a test makes run out (nothing is in flight when it
  does), an expert slot out of range, an id out of range in the dispatch.
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import _lib, moe, synth
from vybforge_b200.quant import quantize_q8_0

from helpers import Built, rel_l2, TOL_MAX_ABS, TOL_REL_L2, TOL_REL_L2_F32

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------------------- permutation
def _check_dispatch(idx_np, n_experts, tag):
    idx = torch.from_numpy(np.ascontiguousarray(idx_np, dtype=np.int32)).cuda()
    perm, pos, offs, counts = moe.dispatch(idx, n_experts)
    torch.cuda.synchronize()
    want_t, want_l, want_off = orc.dispatch_order(idx_np, n_experts)
    perm, pos = perm.cpu().numpy(), pos.cpu().numpy()
    T, k = idx_np.shape
    lane = np.full(T * k, -1, dtype=np.int32)
    lane[pos] = np.tile(np.arange(k, dtype=np.int32), T)       # lane of each permuted row
    np.testing.assert_array_equal(perm, want_t)
    np.testing.assert_array_equal(lane, want_l)
    np.testing.assert_array_equal(offs.cpu().numpy().astype(np.int64), want_off)
    np.testing.assert_array_equal(counts.cpu().numpy(), np.diff(want_off))
    print(f"[dispatch {tag}] {T * k} rows bit-exact")


def test_dispatch_permutation_c0_golden():
    moe.init(0)
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "c0_moe_block.npz"))
    _check_dispatch(g["idx"], 16, "c0 golden ids")


def test_dispatch_permutation_c1_t32_router_ids():
    """The router's own ids at C1 T=32 (bit-exact with the oracle's) through the dispatch."""
    moe.init(0)
    cfg = synth.config("c1", tokens=32)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    from test_gpu_parity import _router_layer
    layer = _router_layer(w_r, bias, cfg.hidden, cfg.n_experts, cfg.topk)
    idx, _ = layer.route(torch.from_numpy(x).to(torch.bfloat16).cuda())
    ri, _ = orc.route(x, w_r, bias, cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    _check_dispatch(idx.cpu().numpy(), cfg.n_experts, "c1 T=32")
    layer.close()


def test_dispatch_permutation_c3_zipf():
    moe.init(0)
    cfg = synth.config("c3", tokens=4096)
    x, w_r, bias, _, _ = synth.zipf_router_inputs(cfg)
    ri, _ = orc.route(x, w_r, bias, cfg.topk)
    _check_dispatch(ri, cfg.n_experts, "c3 T=4096 zipf")


def test_dispatch_flags_an_id_out_of_range():
    moe.init(0)
    idx = torch.tensor([[0, 3], [5, 1], [2, 9]], dtype=torch.int32, device="cuda")   # 9 >= E = 8
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    perm, pos, offs, counts = moe.dispatch(idx, 8, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1                                 # DEV_BAD_EXPERT_ID
    assert int(pos[5].item()) == -1                             # the bad lane has no row
    assert counts.cpu().numpy().sum() == 5


# ----------------------------------------------------------------------------- clamp
GU_SCALE, DOWN_SCALE = 30.0, 0.05   # gate/up ~ N(0, 0.6): |pre-activation| ~ 19 at H = 1024


def _rescale_q8(b: Built):
    """Requantize b's Q8_0 experts with gate/up x GU_SCALE and down x DOWN_SCALE."""
    cfg = b.cfg
    H, I = cfg.hidden, cfg.inter
    for p, (rows, cols, sc) in enumerate([(I, H, GU_SCALE), (I, H, GU_SCALE), (H, I, DOWN_SCALE)]):
        raw = b.dev[p].cpu().numpy()
        new = np.stack([quantize_q8_0((orc.dequant_q8_0(raw[e], rows, cols) * sc).astype(np.float32))
                        for e in range(raw.shape[0])])
        b.dev[p] = torch.from_numpy(new).cuda()
    b._cache = {}


def _rescale_exl3(b: Built):
    for p, sc in enumerate([GU_SCALE, GU_SCALE, DOWN_SCALE]):
        tr, suh, svh = b.dev[p]
        b.dev[p] = (tr, suh, (svh.float() * sc).half())
    b._cache = {}


def _clamp_fractions(b: Built, tokens, idx):
    """Share of gate pre-activations above the limit and of up pre-activations outside it, over
    every (token, selected expert) pair and the shared expert, in the oracle's f64 arithmetic."""
    E = b.cfg.n_experts
    g_all, u_all = [], []
    for t in tokens:
        for e in list(idx[t]) + [E]:
            wg, wu, _ = b.expert(int(e))
            x = b.x[t].astype(np.float64)
            g_all.append(x @ wg)
            u_all.append(x @ wu)
    g, u = np.concatenate(g_all), np.concatenate(u_all)
    return float((g > 10).mean()), float((np.abs(u) > 10).mean())


def _clamp_case(b: Built, T, tag):
    x = b.x_dev[:T].contiguous()
    out, idx, w = b.layer.moe_block(x)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    tokens = np.arange(T)
    ro, ri, rw = b.oracle(tokens)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    fg, fu = _clamp_fractions(b, tokens, ri)
    assert fg >= 0.05 and fu >= 0.05, (fg, fu)
    # without the clamp the oracle's output is a different function altogether
    cfg = b.cfg
    unclamped, _, _ = orc.moe_block_grouped(b.x[tokens], b.w_r, b.bias, b.expert, lambda: b.expert(cfg.n_experts),
                                            cfg.n_experts, cfg.topk, limit=1e30)
    assert rel_l2(unclamped, ro) > 0.5
    o = out.cpu().numpy()
    print(f"[clamp {tag}] g>10 {fg:.2f} |u|>10 {fu:.2f}; max-abs {np.abs(o - ro).max():.3e} "
          f"rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2


@pytest.fixture(scope="module")
def clamp_q8():
    moe.init(0)
    cfg = synth.config("c0", tokens=256)
    cfg.x_dtype = "bf16"
    b = Built(cfg)
    _rescale_q8(b)
    b.layer = b.make_layer(torch.float32)
    return b


def test_clamp_decode_gemv(clamp_q8):
    _clamp_case(clamp_q8, 16, "q8_0 decode GEMV T=16")


def test_clamp_tcgen05_gemm(clamp_q8):
    clamp_q8.layer = clamp_q8.make_layer(torch.float32, path="tc")
    _clamp_case(clamp_q8, 256, "q8_0 tcgen05 T=256")


def test_clamp_split_precision_gemv():
    """fp32 activations: the split-precision GEMV's epilogue clamps too (fp32 bar)."""
    moe.init(0)
    b = Built(synth.config("c0", tokens=16))
    _rescale_q8(b)
    b.layer = b.make_layer(torch.float32)
    out, idx, w = b.layer.moe_block(b.x_dev)
    ro, ri, rw = b.oracle(np.arange(16))
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    fg, fu = _clamp_fractions(b, np.arange(16), ri)
    assert fg >= 0.05 and fu >= 0.05
    o = out.cpu().numpy()
    print(f"[clamp q8_0 split-precision T=16] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert rel_l2(o, ro) <= TOL_REL_L2_F32


@pytest.fixture(scope="module")
def clamp_exl3():
    moe.init(0)
    cfg = synth.config("c0", tokens=256, fmt="exl3")
    cfg.x_dtype = "bf16"
    b = Built(cfg)
    _rescale_exl3(b)
    b.layer = b.make_layer(torch.float32)
    return b


def test_clamp_exl3_decode_gemv(clamp_exl3):
    _clamp_case(clamp_exl3, 16, "exl3 decode GEMV T=16")


def test_clamp_exl3_tcgen05_gemm(clamp_exl3):
    _clamp_case(clamp_exl3, 256, "exl3 tcgen05 T=256")


# ----------------------------------------------------------------------------- fp32 clause
@pytest.mark.parametrize("T", [1, 16, 256])
def test_fp32_layers_meet_the_fp32_tolerance(T):
    """fp32-in, fp32-out layers take the split-precision GEMV at every T (T=256: 64 rows per
    expert, where bf16 layers use the tcgen05 GEMM); rel-L2 <= 1e-4 against the f64 oracle."""
    moe.init(0)
    b = Built(synth.config("c0", tokens=256))
    x = b.x_dev[:T].contiguous()
    out, idx, w = b.layer.moe_block(x)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    ro, ri, rw = b.oracle(np.arange(T))
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    o = out.cpu().numpy()
    print(f"[fp32 split-precision T={T}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert rel_l2(o, ro) <= TOL_REL_L2_F32


# ----------------------------------------------------------------------------- device errors
@pytest.fixture(scope="module")
def c0_bf16():
    moe.init(0)
    cfg = synth.config("c0", tokens=16)
    cfg.x_dtype = "bf16"
    return Built(cfg)


def test_expired_wait_is_reported_and_the_context_stays_usable(c0_bf16):
    """The decode GEMV's producer issues no loads (VFMOE_INJECT_STALL_LOADS) and the wait bound
    is 1 ms: every consumer's first wait expires with nothing in flight, the kernels raise
    DEV_WAIT_TIMEOUT and return.  The host sees VFMOE_ERR_DEVICE with code 2, and the next
    forward without the injection is correct."""
    b = c0_bf16
    ref = b.layer.forward(b.x_dev).clone()
    b.layer.debug_inject(_lib.INJECT_STALL_LOADS, 1_000_000)
    try:
        b.layer.forward(b.x_dev)
        with pytest.raises(_lib.VfmoeError) as ei:
            b.layer.check_device_error()
        assert ei.value.code == _lib.ERR_DEVICE
        assert "code 2" in str(ei.value)
    finally:
        b.layer.debug_inject(_lib.INJECT_NONE)
    again = b.layer.forward(b.x_dev)
    b.layer.check_device_error()
    assert torch.equal(again, ref)


def test_expert_slot_out_of_range_is_reported(c0_bf16):
    """vfmoe_forward_routed with one lane's slot past the shared expert: the count kernel flags
    DEV_BAD_EXPERT_ID before any memory is indexed by it, that lane is dropped, the other lanes
    are computed as usual."""
    b = c0_bf16
    L = b.layer
    n, k = 8, 2
    rows = b.x_dev[:n].contiguous()
    slots = torch.tensor([[i % L.E, (i + 3) % L.E] for i in range(n)], dtype=torch.int32, device="cuda")
    w = torch.full((n, k), 0.5, dtype=torch.float32, device="cuda")
    good = L.forward_routed(rows, slots, w, y_dtype=torch.float32).clone()
    L.check_device_error()
    bad = slots.clone()
    bad[3, 1] = L.n_local + 5
    y = L.forward_routed(rows, bad, w, y_dtype=torch.float32)
    with pytest.raises(_lib.VfmoeError) as ei:
        L.check_device_error()
    assert ei.value.code == _lib.ERR_DEVICE and "code 1" in str(ei.value)
    keep = [i for i in range(n) if i != 3]
    torch.testing.assert_close(y[keep], good[keep], rtol=1e-5, atol=1e-6)
    one = L.forward_routed(rows[3:4].contiguous(), slots[3:4, :1].contiguous(), w[3:4, :1].contiguous(),
                           y_dtype=torch.float32)
    torch.testing.assert_close(y[3:4], one, rtol=1e-5, atol=1e-6)


# ----------------------------------------------------------------------------- router first level
def _cancelling_router(rng, T, H, E):
    """bf16 tokens (columns scaled by 2^-2 .. 2^2) and a router in which every 16th row nearly
    cancels against one token: its products span 2^-4 .. 2^4 in magnitude and sum to ~0 on that
    token, so sum |x_i w_i| is orders of magnitude above |sum x_i w_i| there."""
    from vybforge_b200.quant import round_bf16
    x = round_bf16((rng.standard_normal((T, H)) * np.exp2(rng.integers(-2, 3, (1, H)))).astype(np.float32))
    w_r = rng.normal(0, 0.02, (E, H)).astype(np.float64)
    for e in range(0, E, 16):
        t = (e // 16) % T
        sign = np.where(rng.random(H) < 0.5, -1.0, 1.0)
        w = 0.004 * sign * np.exp2(rng.integers(-4, 5, H)) / np.maximum(np.abs(x[t]), 1e-3)
        w -= (x[t] @ w) / (x[t] @ x[t]) * x[t]                   # cancellation on token t
        w_r[e] = w
    return x, w_r.astype(np.float32)


@pytest.mark.parametrize("case,T", [("random", 40), ("random", 4096), ("cancel", 64), ("cancel", 1024)])
def test_router_first_level_error_within_its_bound(case, T):
    """The first-level logits (tcgen05 on bf16 parts of W_r for bf16 x at T > 32) against exact fp64
    logits: every |error| stays below the bound c |x_t| |w_e| the refinement relies on, and the
    routing is bit-exact."""
    moe.init(0)
    rng = np.random.default_rng(T + (7 if case == "cancel" else 0))
    H, E, k = 6144, 256, 8
    if case == "random":
        cfg = synth.config("c1", tokens=T)
        x, w_r, bias, _ = synth.router_inputs(cfg)
    else:
        x, w_r = _cancelling_router(rng, T, H, E)
        bias = rng.normal(0, 0.01, E).astype(np.float32)
    from test_gpu_parity import _router_layer
    layer = _router_layer(w_r, bias, H, E, k)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    logits, c = layer.route_logits(xd)
    torch.cuda.synchronize()
    layer.check_device_error()
    exact = x.astype(np.float64) @ w_r.astype(np.float64).T
    bound = c * np.linalg.norm(x.astype(np.float64), axis=1)[:, None] * np.linalg.norm(w_r.astype(np.float64), axis=1)[None, :]
    err = np.abs(logits.cpu().numpy().astype(np.float64) - exact)
    ratio = float((err / bound).max())
    scale = np.abs(x.astype(np.float64)) @ np.abs(w_r.astype(np.float64)).T
    print(f"[router L1 {case} T={T}] c = {c:.3e}; max |err| / bound = {ratio:.3e}; "
          f"max |err| / sum|x w| = {float((err / scale).max()):.3e}")
    assert ratio < 1.0
    idx, w = layer.route(xd)
    torch.cuda.synchronize()
    layer.check_device_error()
    ri, rw = orc.route(x, w_r, bias, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    layer.close()
