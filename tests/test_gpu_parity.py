"""GPU parity: the CUDA path (through the C ABI) against the oracle.

Bars (north_star): expert ids and the permutation bit-exact (lowest-index ties);
combined output max-abs <= 2e-2 and rel-L2 <= 1e-3; standalone weight decoders
bit-exact."""

import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import synth, moe
from vybforge_b200.quant import quantize_q8_0

from helpers import Built, rel_l2, TOL_MAX_ABS, TOL_REL_L2, TOL_REL_L2_F32

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def c0():
    moe.init(0)
    return Built(synth.config("c0"))


def test_c0_matches_reference_golden(c0):
    """C0 is the fp32-in, fp32-out gate: the split-precision decode GEMV must meet the fp32
    clause of the tolerance (rel-L2 1e-4) against the reference's own moe_block output."""
    g = np.load(os.path.join(GOLD, "c0_moe_block.npz"))
    out, idx, w = c0.layer.moe_block(c0.x_dev)
    torch.cuda.synchronize()
    c0.layer.check_device_error()
    np.testing.assert_array_equal(idx.cpu().numpy(), g["idx"])
    np.testing.assert_allclose(w.cpu().numpy(), g["w"], rtol=0, atol=1e-6)
    o = out.cpu().numpy()
    print(f"[parity c0 golden] max-abs {np.abs(o - g['out']).max():.3e} rel-L2 {rel_l2(o, g['out']):.3e}")
    assert np.abs(o - g["out"]).max() <= TOL_MAX_ABS
    assert rel_l2(o, g["out"]) <= TOL_REL_L2_F32


def test_c0_bf16_output_is_rounded_fp32_output(c0):
    l16 = c0.make_layer(torch.bfloat16)
    o16 = l16.forward(c0.x_dev)
    o32 = c0.layer.forward(c0.x_dev)
    torch.testing.assert_close(o16, o32.to(torch.bfloat16), rtol=0, atol=0)


def test_c0_deterministic(c0):
    a = c0.layer.forward(c0.x_dev).clone()
    b = c0.layer.forward(c0.x_dev)
    assert torch.equal(a, b)


def test_route_only_matches_forward_routing(c0):
    idx, w = c0.layer.route(c0.x_dev)
    _, idx2, w2 = c0.layer.moe_block(c0.x_dev)
    assert torch.equal(idx, idx2) and torch.equal(w, w2)


@pytest.mark.parametrize("T", [1, 3, 16])
def test_c0_token_counts(c0, T):
    out, idx, w = c0.layer.moe_block(c0.x_dev[:T].contiguous())
    ro, ri, rw = c0.oracle(np.arange(T))
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    o = out.cpu().numpy()
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2_F32


def test_zero_tokens_is_noop(c0):
    out = torch.full((0, c0.cfg.hidden), 7.0, device="cuda")
    c0.layer.forward(c0.x_dev[:0], out=out)
    torch.cuda.synchronize()


def test_workspace_too_small_is_an_error(c0):
    from vybforge_b200 import _lib
    ws = torch.empty(256, dtype=torch.uint8, device="cuda")
    with pytest.raises(_lib.VfmoeError) as ei:
        c0.layer.forward(c0.x_dev, workspace=ws)
    assert ei.value.code == _lib.ERR_WORKSPACE


def test_route_ties_lowest_index():
    moe.init(0)
    cfg = synth.config("c0")
    b = Built(cfg)
    w_r = b.w_r.copy()
    w_r[2] = 0.0                    # experts 2 and 9: logit exactly 0 on every token
    w_r[9] = 0.0
    bias = np.zeros_like(b.bias)
    bias[2] = bias[9] = 1.0         # choice 1.5 for both: top-2, exact tie -> 2 before 9
    b.wr_dev = torch.from_numpy(w_r).cuda()
    b.bias_dev = torch.from_numpy(bias).cuda()
    layer = b.make_layer(torch.float32)
    idx, w = layer.route(b.x_dev)
    ri, rw = orc.route(b.x, w_r, bias, cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float32])
def test_route_ties_lowest_index_prefill_batch(x_dtype):
    """Exact ties at a prefill batch (T=4096: tensor-core or tiled first level, one warp per token
    in the refinement): experts 2 and 9 have zero router rows and equal bias, so their choices tie
    exactly on every token and the lower id must come first, as in the f64 oracle."""
    moe.init(0)
    cfg = synth.config("c1", tokens=4096)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    w_r = w_r.copy()
    bias = bias.copy()
    w_r[2] = 0.0
    w_r[9] = 0.0
    bias[2] = bias[9] = 1.0
    layer = _router_layer(w_r, bias, cfg.hidden, cfg.n_experts, cfg.topk, x_dtype=x_dtype)
    xd = torch.from_numpy(x).to(x_dtype).cuda()
    idx, w = layer.route(xd)
    ri, rw = orc.route(xd.float().cpu().numpy(), w_r, bias, cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    assert (idx.cpu().numpy()[:, :2] == [2, 9]).all()
    layer.check_device_error()
    layer.close()


# ----------------------------------------------------------------------------- full-size C1 (Q8_0 decode)
@pytest.fixture(scope="module")
def c1():
    moe.init(0)
    return Built(synth.config("c1", tokens=32), weights="cuda")


@pytest.mark.parametrize("T", [1, 8])
def test_c1_decode_parity(c1, T):
    x = c1.x_dev[:T].contiguous()
    out, idx, w = c1.layer.moe_block(x)
    ro, ri, rw = c1.oracle(np.arange(T))
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    o = out.cpu().numpy()
    print(f"[parity c1 T={T}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS
    assert rel_l2(o, ro) <= TOL_REL_L2


def test_c1_t32_routing_and_token_subset(c1):
    out, idx, w = c1.layer.moe_block(c1.x_dev)
    ri, rw = orc.route(c1.x, c1.w_r, c1.bias, c1.cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    sub = np.array([0, 13, 31])
    ro, _, _ = c1.oracle(sub)
    o = out.cpu().numpy()[sub]
    print(f"[parity c1 T=32 tokens {sub.tolist()}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2
    c1.layer.check_device_error()


# ----------------------------------------------------------------------------- standalone decoders
def test_q8_0_quantize_bit_exact():
    moe.init(0)
    rng = np.random.default_rng(4)
    w = rng.normal(0, 0.02, (64, 512)).astype(np.float32)
    w[1, :32] = 0
    w[2, :] = rng.normal(0, 50.0, 512)
    dst = torch.empty((64, 512 // 32 * 34), dtype=torch.uint8, device="cuda")
    moe.q8_0_quantize(torch.from_numpy(w).cuda(), dst)
    np.testing.assert_array_equal(dst.cpu().numpy(), quantize_q8_0(w))


def test_q8_0_dequant_bit_exact():
    g = np.load(os.path.join(GOLD, "q8_0_kat.npz"))
    raw, deq = g["raw"], g["deq"]
    rows, k = raw.shape[0], raw.shape[1] // 34 * 32
    d32 = moe.q8_0_dequant(torch.from_numpy(raw).cuda(), rows, k, torch.float32)
    np.testing.assert_array_equal(d32.cpu().numpy().astype(np.float64), deq)
    d16 = moe.q8_0_dequant(torch.from_numpy(raw).cuda(), rows, k, torch.float16)
    np.testing.assert_array_equal(d16.cpu().numpy(), deq.astype(np.float16))


def test_exl3_3bpw_decode_bit_exact():
    rng = np.random.default_rng(8)
    K, N = 256, 384
    tr = rng.integers(0, 1 << 16, size=(K // 16, N // 16, 48), dtype=np.uint32).astype(np.uint16)
    got = moe.exl3_decode(torch.from_numpy(tr.view(np.int16)).cuda(), K, N, 3)
    want = orc.exl3_what(tr, 3).astype(np.float16)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_exl3_4bpw_decode_bit_exact():
    """4 bpw (the reference's format) through the GPU's closed-form window extraction against
    the oracle's decode with the reference's slot table, and against the reference's own
    trellis fixture."""
    rng = np.random.default_rng(9)
    K, N = 256, 384
    tr = rng.integers(0, 1 << 16, size=(K // 16, N // 16, 64), dtype=np.uint32).astype(np.uint16)
    got = moe.exl3_decode(torch.from_numpy(tr.view(np.int16)).cuda(), K, N, 4)
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "exl3_kat.npz"))
    table = (g["slot_nibble"].astype(int), g["slot_pos"].astype(int))
    want = orc.exl3_what(tr, 4, table).astype(np.float16)
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), want.view(np.uint16))
    tr4 = g["tr4"]
    got4 = moe.exl3_decode(torch.from_numpy(tr4.view(np.int16)).cuda(), 16 * tr4.shape[0], 16 * tr4.shape[1], 4)
    want4 = orc.exl3_what(tr4, 4, table).astype(np.float16)
    np.testing.assert_array_equal(got4.cpu().numpy().view(np.uint16), want4.view(np.uint16))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm(dtype):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((7, 6144)).astype(np.float32) * 3
    w = (1 + rng.normal(0, 0.02, 6144)).astype(np.float32)
    xd = torch.from_numpy(x).cuda().to(dtype)
    y = moe.rmsnorm(xd, torch.from_numpy(w).cuda(), 1e-5).float().cpu().numpy()
    ref = orc.rmsnorm(xd.float().cpu().numpy(), w, 1e-5)
    tol = 1e-5 if dtype == torch.float32 else 8e-3
    assert rel_l2(y, ref) < tol


# ----------------------------------------------------------------------------- stage-tiled Q8_0 layout
def test_q8_0_tile_matches_oracle():
    moe.init(0)
    rng = np.random.default_rng(5)
    w = rng.integers(0, 256, (3, 128, 1024 // 32 * 34), dtype=np.uint8)
    got = moe.q8_0_tile(torch.from_numpy(w).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, orc.q8_0_tile(w))


@pytest.fixture(scope="module")
def c1_tiled(c1):
    E = c1.cfg.n_experts
    g, u, d = (moe.q8_0_tile(c1.dev[p]) for p in range(3))
    layer = moe.MoELayer(hidden=c1.cfg.hidden, inter=c1.cfg.inter, n_experts=E, topk=c1.cfg.topk,
                         router_w=c1.wr_dev, router_bias=c1.bias_dev, gate=g[:E], up=u[:E], down=d[:E],
                         shared=(g[E], u[E], d[E]), fmt="q8_0_tiled", x_dtype=torch.bfloat16,
                         out_dtype=torch.float32)
    yield layer
    layer.close()


@pytest.mark.parametrize("T", [1, 8, 32, 1024, 4096])
def test_tiled_weights_give_identical_output(c1, c1_tiled, T):
    """Same kernels, same arithmetic: only the byte order of the weights in HBM differs
    (decode GEMV at T <= 32, tcgen05 grouped GEMM above)."""
    g = torch.Generator(device="cuda").manual_seed(T)
    x = torch.randn((T, c1.cfg.hidden), generator=g, device="cuda").to(torch.bfloat16)
    ref = c1.layer.forward(x)
    got = c1_tiled.forward(x)
    torch.cuda.synchronize()
    c1_tiled.check_device_error()
    assert torch.equal(ref, got)


# ----------------------------------------------------------------------------- CUDA graph capture
@pytest.mark.parametrize("T", [1, 32, 1024])
def test_forward_is_cuda_graph_capturable(c1_tiled, T):
    """With a caller workspace, vfmoe_forward makes no host synchronisation and no allocation:
    it records into a CUDA graph (programmatic-dependent launches included), and a replay
    reproduces the eager result bit for bit (decode GEMV at T <= 32, tcgen05 GEMM above)."""
    layer = c1_tiled
    H, k = layer.H, layer.k
    g = torch.Generator(device="cuda").manual_seed(100 + T)
    x = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    ws = torch.empty(layer.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    layer.forward(x, out=out, idx=idx, w=w, workspace=ws)
    torch.cuda.synchronize()
    ref, ref_idx, ref_w = out.clone(), idx.clone(), w.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer.forward(x, out=out, idx=idx, w=w, workspace=ws)
    out.zero_()
    idx.zero_()
    graph.replay()
    torch.cuda.synchronize()
    layer.check_device_error()
    assert torch.equal(out, ref) and torch.equal(idx, ref_idx) and torch.equal(w, ref_w)
    del graph


# ----------------------------------------------------------------------------- tcgen05 path vs SIMT path
def _simt_layer(built, out_dtype=torch.float32):
    return built.make_layer(out_dtype, path="simt")


@pytest.mark.parametrize("cfg_name,T", [("c0", 16), ("c1", 1), ("c1", 32)])
def test_tensor_core_path_matches_simt_path(c0, c1, cfg_name, T):
    """Same fp16 operands on both sides (C0's fp32 activations: the tcgen05 kernels forced with
    expert_path TC, since the automatic choice there is the split-precision GEMV)."""
    b = c0 if cfg_name == "c0" else c1
    x = b.x_dev[:T].contiguous()
    layer = b.make_layer(torch.float32, path="tc") if cfg_name == "c0" else b.layer
    tc = layer.forward(x).cpu().numpy()
    simt = _simt_layer(b).forward(x).cpu().numpy()
    torch.cuda.synchronize()
    b.layer.check_device_error()
    # both paths use identical fp16 operands; they differ only in fp32 accumulation order
    # (the tensor core sums K=16 products per step), measured ~1e-4 rel-L2 at K=6144
    print(f"[tc-vs-simt {cfg_name} T={T}] rel-L2 {rel_l2(tc, simt):.3e} max-abs {np.abs(tc - simt).max():.3e}")
    assert rel_l2(tc, simt) < 5e-4, rel_l2(tc, simt)
    assert np.abs(tc - simt).max() < 5e-3


# ----------------------------------------------------------------------------- router precision levels
def _router_layer(w_r, bias, H, E, k, x_dtype=torch.bfloat16):
    """A routing-only layer (expert weights are never read by vfmoe_route)."""
    from vybforge_b200.moe import MoELayer
    I = 256
    gu = torch.zeros((E, I, H // 32 * 34), dtype=torch.uint8, device="cuda")
    dn = torch.zeros((E, H, I // 32 * 34), dtype=torch.uint8, device="cuda")
    return MoELayer(hidden=H, inter=I, n_experts=E, topk=k, router_w=torch.from_numpy(w_r).cuda(),
                    router_bias=torch.from_numpy(bias).cuda(), gate=gu, up=gu, down=dn, x_dtype=x_dtype,
                    out_dtype=torch.float32)


@pytest.mark.parametrize("reps", [1, 12, 1024])
def test_router_on_real_glm_router_weights(reps):
    """The reference's real-weight router case (tests/golden/glm_router_prep.npz, from its
    native/glm53/prep: GLM router weights of one layer, E=288, H=4096, k=8, four fp32 hidden rows):
    ids equal the reference's ref_idx and weights its ref_w.  reps=12 and 1024 repeat the rows (T=48,
    T=4096) to take the multi-token first level and the one-warp-per-token refinement; every copy
    must route alike."""
    moe.init(0)
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "glm_router_prep.npz"))
    w_r = (g["gate_bits"].astype(np.uint32) << 16).view(np.float32)
    H, E, k = 4096, 288, 8
    layer = _router_layer(np.ascontiguousarray(w_r), g["bias"], H, E, k, x_dtype=torch.float32)
    x = torch.from_numpy(np.tile(g["y"], (reps, 1))).cuda()
    idx, w = layer.route(x)
    torch.cuda.synchronize()
    layer.check_device_error()
    ref_idx, ref_w = np.tile(g["ref_idx"], (reps, 1)), np.tile(g["ref_w"], (reps, 1))
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    d = float(np.abs(w.cpu().numpy() - ref_w).max())
    print(f"[real GLM router T={4 * reps}] ids equal ref_idx; max |w - ref_w| {d:.2e}")
    assert d <= 1e-6
    layer.close()


@pytest.mark.parametrize("T", [16, 96, 4096])
def test_router_near_ties_take_the_f64_level(T):
    """Pairs of experts whose router rows differ by one fp32 ulp in one element: their
    logits differ by ~1e-9, below the float-float bound, so the f64 level must order them."""
    moe.init(0)
    rng = np.random.default_rng(21)
    H, E, k = 6144, 256, 8
    from vybforge_b200.quant import round_bf16
    x = round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    w_r = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    bias = rng.normal(0, 0.01, E).astype(np.float32)
    for p in range(4):
        a = 10 + 2 * p
        w_r[a + 1] = w_r[a]
        w_r[a + 1, 7 * p] = np.nextafter(w_r[a, 7 * p], np.float32(1.0))   # one ulp up
        bias[a] = bias[a + 1] = 1.0                                          # both always selected
    layer = _router_layer(w_r, bias, H, E, k)
    idx, w = layer.route(torch.from_numpy(x).to(torch.bfloat16).cuda())
    ri, rw = orc.route(x, w_r, bias, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    layer.check_device_error()


def test_router_prefill_size_bit_exact():
    moe.init(0)
    cfg = synth.config("c3", tokens=4096)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    layer = _router_layer(w_r, bias, cfg.hidden, cfg.n_experts, cfg.topk)
    idx, w = layer.route(torch.from_numpy(x).to(torch.bfloat16).cuda())
    ri, rw = orc.route(x, w_r, bias, cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    layer.check_device_error()


# ----------------------------------------------------------------------------- decode GEMV vs tcgen05 GEMM
@pytest.mark.parametrize("T", [1, 32])
def test_decode_gemv_matches_tcgen05_gemm(c1, T):
    """The decode path (register-operand MMA GEMV) and the tcgen05 GEMM forced onto the
    same decode shapes (expert_path TC) compute the same fp16 operands; they differ in
    accumulation order."""
    x = c1.x_dev[:T].contiguous()
    gv = c1.layer.forward(x).cpu().numpy()
    tc = c1.make_layer(torch.float32, path="tc").forward(x).cpu().numpy()
    torch.cuda.synchronize()
    c1.layer.check_device_error()
    print(f"[gemv-vs-tcgen05 c1 T={T}] rel-L2 {rel_l2(gv, tc):.3e}")
    assert rel_l2(gv, tc) < 5e-4


@pytest.mark.parametrize("T", [32, 1024, 4096])
def test_cta_pair_gemm_matches_single_cta_tiles(c1, c1_tiled, T):
    """Prefill tiles (N >= 32) run on CTA pairs (tcgen05 cta_group::2, 256 channels per tile);
    expert_path "tc1" keeps single-CTA tiles.  Same fp16 operands, same K order per output: the
    outputs agree to fp32 accumulation (GGUF rows and stage-tiled weights alike)."""
    g = torch.Generator(device="cuda").manual_seed(7 + T)
    x = torch.randn((T, c1.cfg.hidden), generator=g, device="cuda").to(torch.bfloat16)
    path = "tc" if T == 32 else "auto"   # T = 32 averages one row per expert: force the GEMM
    pair = c1.make_layer(torch.float32, path=path)
    single = c1.make_layer(torch.float32, path="tc1")
    a, b = pair.forward(x), single.forward(x)
    t = c1_tiled.forward(x) if T > 32 else a   # the tiled layer takes the GEMV at T = 32
    torch.cuda.synchronize()
    for L in (pair, single, c1_tiled):
        L.check_device_error()
    d = rel_l2(a.cpu().numpy(), b.cpu().numpy())
    print(f"[cta pair vs single-CTA tiles T={T}] rel-L2 {d:.3e}, bit-identical {bool(torch.equal(a, b))}, "
          f"tiled weights identical {bool(torch.equal(a, t))}")
    assert d < 1e-6
    assert torch.equal(a, t)
    pair.close()
    single.close()


@pytest.mark.parametrize("T", [1, 8, 32, 64, 65])
def test_decode_front_end_matches_separate_launches(c1, T):
    """At T <= 64 the AUTO path runs dispatch, gather and the GEMV's tile plan as one launch
    (decode_front_kernel); a layer forced onto the GEMV path keeps the separate launches (as AUTO
    does from T = 65).  Same permutation, rows and tiles into the same GEMV: outputs, ids and
    weights bit-identical."""
    g = torch.Generator(device="cuda").manual_seed(11 + T)
    x = torch.randn((T, c1.cfg.hidden), generator=g, device="cuda").to(torch.bfloat16)
    sep = c1.make_layer(torch.float32, path="gemv")
    a, ia, wa = c1.layer.moe_block(x)
    b, ib, wb = sep.moe_block(x)
    torch.cuda.synchronize()
    c1.layer.check_device_error()
    sep.check_device_error()
    print(f"[decode front end T={T}] bit-identical {bool(torch.equal(a, b))}")
    assert torch.equal(ia, ib) and torch.equal(wa, wb)
    assert torch.equal(a, b)
    sep.close()


def test_decode_front_end_split_precision(c0):
    """The same at C0 (fp32 activations: the front end also writes the residual plane)."""
    sep = c0.make_layer(torch.float32, path="gemv")
    a, ia, wa = c0.layer.moe_block(c0.x_dev)
    b, ib, wb = sep.moe_block(c0.x_dev)
    torch.cuda.synchronize()
    c0.layer.check_device_error()
    sep.check_device_error()
    assert torch.equal(ia, ib) and torch.equal(wa, wb)
    assert torch.equal(a, b)
    sep.close()


def test_c0_prefill_size_tcgen05_path(c0):
    """T=256 at C0 shapes: 64 tokens per routed expert on average, tcgen05 GEMM forced (C0's fp32
    activations would otherwise take the split-precision GEMV)."""
    cfg = synth.config("c0", tokens=256)
    b = Built(cfg, path="tc")
    out, idx, w = b.layer.moe_block(b.x_dev)
    ro, ri, rw = b.oracle()
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    o = out.cpu().numpy()
    print(f"[parity c0 T=256 tcgen05] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2
    b.layer.check_device_error()


def test_c1_prefill_1024_tcgen05_path():
    """T=1024 at C1 shapes (32 tokens per routed expert on average -> tcgen05 GEMM):
    routing bit-exact for all tokens, output checked on a token subset."""
    moe.init(0)
    b = Built(synth.config("c1", tokens=1024), weights="cuda")
    out, idx, w = b.layer.moe_block(b.x_dev)
    ri, rw = orc.route(b.x, b.w_r, b.bias, b.cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    sub = np.array([0, 511, 1023])
    ro, _, _ = b.oracle(sub)
    o = out.cpu().numpy()[sub]
    print(f"[parity c1 T=1024 tcgen05 tokens {sub.tolist()}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2
    b.layer.check_device_error()


def test_c3_zipf_prefill_parity():
    """BASELINE C3: T=4096 prefill with Zipf(1.1)-skewed routing (the hottest expert gets
    ~4000 tokens, the tail a handful).  Routing bit-exact for every token; output within
    tolerance on tokens of the hottest and of a tail expert."""
    moe.init(0)
    cfg = synth.config("c3", tokens=4096)
    x, w_r, bias, tgt, _ = synth.zipf_router_inputs(cfg)
    b = Built(cfg, weights="cuda", router=(x, w_r, bias))
    out, idx, w = b.layer.moe_block(b.x_dev)
    ri, rw = orc.route(x, w_r, bias, cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    cnt = np.bincount(ri.reshape(-1), minlength=cfg.n_experts)
    assert cnt.max() > 3000                                   # skew reached the kernels
    hot, cold = int(np.argmax(cnt)), int(np.argmin(np.where(cnt > 0, cnt, 10**9)))
    toks = sorted({int(np.nonzero((ri == hot).any(1))[0][-1]), int(np.nonzero((ri == cold).any(1))[0][0]), 2048})
    sub = np.array(toks)
    ro, _, _ = b.oracle(sub)
    o = out.cpu().numpy()[sub]
    print(f"[parity c3 zipf T=4096 tokens {toks}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2
    b.layer.check_device_error()


# ----------------------------------------------------------------------------- packed layer files
@pytest.mark.parametrize("which", ["q8_0_tiled", "exl3"])
def test_packed_layer_file_round_trip(c1_tiled, tmp_path, which):
    """A layer written with vfmoe_pack_save and read back with vfmoe_pack_load (one device buffer,
    chunked reads) gives bit-identical forwards: the file holds the kernels' own byte layout."""
    if which == "exl3":
        moe.init(0)
        src = Built(synth.config("c0", tokens=64, fmt="exl3")).layer
        x = torch.randn((64, src.H), generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
    else:
        src = c1_tiled
        g = torch.Generator(device="cuda").manual_seed(11)
        x = torch.randn((32, src.H), generator=g, device="cuda").to(torch.bfloat16)
    path = str(tmp_path / f"layer_{which}.vfpk")
    src.save_packed(path)
    back = moe.MoELayer.from_packed(path)
    assert back.fmt == which and back.E == src.E
    a = src.forward(x.to(src.x_dtype))
    b = back.forward(x.to(back.x_dtype))
    torch.cuda.synchronize()
    back.check_device_error()
    assert torch.equal(a, b)
    back.close()
