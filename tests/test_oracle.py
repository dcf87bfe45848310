"""CPU checks of the oracle (oracle/moe_oracle.py) against the reference's own
golden data, and of the host-side packing/generator.  No GPU."""

import hashlib
import os

import numpy as np
import pytest

from oracle import moe_oracle as orc
from vybforge_b200 import synth
from vybforge_b200.quant import quantize_q8_0, round_bf16, f32_to_bf16_bits

GOLD = os.path.join(os.path.dirname(__file__), "golden")
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference checkout (only the real-weight fixture test reads it; skipped when absent)
REF = os.environ.get("VYBFORGE_REFERENCE", os.path.normpath(os.path.join(REPO, os.pardir, "reference")))
PREP = os.path.join(REF, "native/glm53/prep")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def c0_inputs():
    cfg = synth.config("c0")
    x, w_r, bias, rng = synth.router_inputs(cfg)
    experts = synth.expert_q8_numpy(cfg, rng)
    return cfg, x, w_r, bias, experts


def c0_getters(cfg, experts):
    H, I, E = cfg.hidden, cfg.inter, cfg.n_experts

    def mats(e):
        return (orc.q8_0_expert_inout(experts[0][e], I, H), orc.q8_0_expert_inout(experts[1][e], I, H),
                orc.q8_0_expert_inout(experts[2][e], H, I))
    return mats, (lambda: mats(E))


# ----------------------------------------------------------------------------- pinned to the reference
def test_c0_inputs_match_golden_hashes():
    g = np.load(os.path.join(GOLD, "c0_moe_block.npz"))
    cfg, x, w_r, bias, experts = c0_inputs()
    assert sha(x) == str(g["x_sha"]) and sha(w_r) == str(g["w_r_sha"]) and sha(bias) == str(g["bias_sha"])
    assert sha(experts[0]) == str(g["gate_sha"])
    assert sha(experts[1]) == str(g["up_sha"])
    assert sha(experts[2]) == str(g["down_sha"])


def test_c0_oracle_matches_reference_moe_block():
    """Golden output of the reference's native/glm53/moe_ref.py:moe_block on C0."""
    g = np.load(os.path.join(GOLD, "c0_moe_block.npz"))
    cfg, x, w_r, bias, experts = c0_inputs()
    get_e, get_s = c0_getters(cfg, experts)
    out, idx, w = orc.moe_block(x, w_r, bias, get_e, get_s(), cfg.topk)
    np.testing.assert_array_equal(idx, g["idx"])
    np.testing.assert_allclose(w, g["w"], rtol=0, atol=1e-15)
    np.testing.assert_allclose(out, g["out"], rtol=1e-12, atol=1e-12)
    out2, idx2, w2 = orc.moe_block_grouped(x, w_r, bias, get_e, get_s, cfg.n_experts, cfg.topk)
    np.testing.assert_array_equal(idx2, g["idx"])
    np.testing.assert_allclose(out2, g["out"], rtol=1e-12, atol=1e-12)


@pytest.mark.skipif(not os.path.isdir(PREP), reason="reference prep fixture not mounted")
def test_prep_fixture_bit_exact():
    """native/glm53/prep: S=4, H=4096, E=288, k=8 with real GLM router weights.
    The restatement reproduces the committed ref_{out,idx,w}.f32 exactly."""
    H, I, E, k = 4096, 2048, 288, 8

    def f(n, shape):
        return np.fromfile(os.path.join(PREP, n + ".f32"), dtype="<f4").reshape(shape)
    y = f("y", (4, H))
    gate, bias = f("gate", (E, H)), f("bias", (E,))
    ew = tuple(f(n, s).astype(np.float64) for n, s in (("wg_e", (H, I)), ("wu_e", (H, I)), ("wd_e", (I, H))))
    sw = tuple(f(n, s) for n, s in (("wg_s", (H, I)), ("wu_s", (H, I)), ("wd_s", (I, H))))
    out, idx, w = orc.moe_block(y.astype(np.float64), gate, bias, lambda e: ew, sw, k)
    np.testing.assert_array_equal(idx.astype(np.float32), f("ref_idx", (4, k)))
    np.testing.assert_array_equal(w.astype(np.float32), f("ref_w", (4, k)))
    np.testing.assert_array_equal(out.astype(np.float32), f("ref_out", (4, H)))


def test_real_router_fixture_reproduced():
    """tests/golden/glm_router_prep.npz (the router part of the reference's native/glm53/prep: real
    GLM router weights of one layer, its correction bias, four hidden rows): the oracle's route
    gives the reference's ids exactly and its weights to the f32 rounding."""
    g = np.load(os.path.join(GOLD, "glm_router_prep.npz"))
    w_r = (g["gate_bits"].astype(np.uint32) << 16).view(np.float32)
    idx, w = orc.route(g["y"].astype(np.float64), w_r, g["bias"], 8)
    np.testing.assert_array_equal(idx, g["ref_idx"])
    np.testing.assert_array_equal(w.astype(np.float32), g["ref_w"])


def test_q8_0_decode_matches_reference_kat():
    g = np.load(os.path.join(GOLD, "q8_0_kat.npz"))
    raw, deq = g["raw"], g["deq"]
    ours = orc.dequant_q8_0(raw, raw.shape[0], raw.shape[1] // 34 * 32)
    np.testing.assert_array_equal(ours, deq)


def test_q8_0_tiled_layout_is_a_permutation_of_gguf_rows():
    rng = np.random.default_rng(4)
    raw = rng.integers(0, 256, (2, 128, 512 // 32 * 34), dtype=np.uint8)
    t = orc.q8_0_tile(raw)
    assert t.shape == raw.shape
    np.testing.assert_array_equal(orc.q8_0_untile(t), raw)
    flat = t.reshape(2, -1)
    KR = 2
    for m, r, kr in [(0, 0, 0), (0, 63, 1), (1, 64, 0), (1, 127, 1), (0, 70, 1)]:
        off = ((r // 64) * KR + kr) * 17408 + (r % 64) * 272
        np.testing.assert_array_equal(flat[m, off:off + 272], raw[m, r, kr * 272:(kr + 1) * 272])


def test_q8_0_quantizer_matches_gguf():
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(3)
    for scale in (0.02, 1.0, 1e-5):
        w = rng.normal(0, scale, (32, 256)).astype(np.float32)
        w[0, :32] = 0.0
        ref = gguf.quants.quantize(w, gguf.GGMLQuantizationType.Q8_0)
        np.testing.assert_array_equal(quantize_q8_0(w), ref)
        deq = gguf.quants.dequantize(ref, gguf.GGMLQuantizationType.Q8_0)
        np.testing.assert_array_equal(orc.dequant_q8_0(ref, 32, 256), deq.astype(np.float64))


def test_mcg_decode_all_windows_matches_reference():
    g = np.load(os.path.join(GOLD, "exl3_kat.npz"))
    ours = orc.decode_mcg(np.arange(1 << 16, dtype=np.uint32).astype(np.uint16))
    np.testing.assert_array_equal(ours.view(np.uint16), g["mcg_bits"])
    assert float(orc.decode_mcg(np.array([0], np.uint16))[0]) == 1.84375  # native/exl3/README.md:40


def slot_table():
    g = np.load(os.path.join(GOLD, "exl3_kat.npz"))
    rc = g["slot_rc"].astype(np.int64)
    order = np.lexsort((rc[:, 1], rc[:, 0]))
    assert np.array_equal(rc[order, 0] * 16 + rc[order, 1], np.arange(256))
    return g["slot_nibble"].astype(np.int64)[order], g["slot_pos"].astype(np.int64)[order]


def test_exl3_4bpw_dequant_matches_reference():
    """Reference dequant_exl3 (f32 math, fp16 result) vs the f64 restatement."""
    g = np.load(os.path.join(GOLD, "exl3_kat.npz"))
    ref = g["w4"].view(np.float16).astype(np.float64)
    ours = orc.dequant_exl3(g["tr4"], g["suh4"], g["svh4"], 4, slot_table())
    ulp = np.abs(np.spacing(ref.astype(np.float16))).astype(np.float64)
    assert np.all(np.abs(ours - ref) <= ulp + 1e-7)


def test_exl3_4bpw_closed_form_equals_reference_slot_table():
    """The GPU's word-pair form of the 4-bpw windows equals the reference's verified slot
    composition (exl3_ref.py:66-81, 97-107) on every slot of random tiles and of the
    reference's own trellis fixture."""
    g = np.load(os.path.join(GOLD, "exl3_kat.npz"))
    rng = np.random.default_rng(11)
    tiles = rng.integers(0, 1 << 16, size=(64, 64), dtype=np.uint32).astype(np.uint16)
    np.testing.assert_array_equal(orc.exl3_windows_4bpw_words(tiles), orc.exl3_windows_4bpw(tiles, *slot_table()))
    np.testing.assert_array_equal(orc.exl3_windows_4bpw_words(g["tr4"]), orc.exl3_windows_4bpw(g["tr4"], *slot_table()))
    ref = g["w4"].view(np.float16).astype(np.float64)
    ours = orc.dequant_exl3(g["tr4"], g["suh4"], g["svh4"], 4)
    ulp = np.abs(np.spacing(ref.astype(np.float16))).astype(np.float64)
    assert np.all(np.abs(ours - ref) <= ulp + 1e-7)


# ----------------------------------------------------------------------------- restatement-internal checks
def test_exl3_3bpw_windows_bit_by_bit():
    rng = np.random.default_rng(5)
    tiles = rng.integers(0, 1 << 16, size=(3, 48), dtype=np.uint32).astype(np.uint16)
    w = orc.exl3_windows_3bpw_bits(tiles)
    for t in range(3):
        bits = [(int(tiles[t, i // 16]) >> (i % 16)) & 1 for i in range(768)]
        for j in (0, 1, 15, 16, 100, 250, 255):
            v = sum(bits[(3 * j + i) % 768] << i for i in range(16))
            assert int(w[t, j % 16, j // 16]) == v


def test_exl3_3bpw_word_windows_match_bit_windows():
    rng = np.random.default_rng(6)
    tiles = rng.integers(0, 1 << 16, size=(4, 5, 48), dtype=np.uint32).astype(np.uint16)
    np.testing.assert_array_equal(orc.exl3_windows_3bpw(tiles), orc.exl3_windows_3bpw_bits(tiles))


def test_exl3_activation_side_hadamard_identity():
    """x . W == ((x*suh) Hb) W^ Hb * svh  -- the rewrite the GPU kernels use."""
    rng = np.random.default_rng(9)
    K, N = 256, 128
    tr = rng.integers(0, 1 << 16, size=(K // 16, N // 16, 48), dtype=np.uint32).astype(np.uint16)
    suh = np.where(rng.random(K) < 0.5, -1.0, 1.0)
    svh = np.where(rng.random(N) < 0.5, -1.0, 1.0) * rng.uniform(0.01, 0.03, N)
    W = orc.dequant_exl3(tr, suh, svh, 3)
    What = orc.exl3_what(tr, 3)
    x = rng.standard_normal((5, K))
    H = orc.hadamard128() * orc.R_SCALE
    xr = ((x * suh).reshape(5, K // 128, 128) @ H).reshape(5, K)
    z = xr @ What
    y = (z.reshape(5, N // 128, 128) @ H).reshape(5, N) * svh
    np.testing.assert_allclose(y, x @ W, rtol=1e-10, atol=1e-10)


def test_route_ties_go_to_lowest_index():
    H, E = 64, 16
    w_r = np.zeros((E, H), np.float32)
    w_r[3] = w_r[7] = w_r[12] = 0.25      # identical rows -> identical logits
    w_r[5] = 0.5
    bias = np.zeros(E, np.float32)
    x = np.ones((2, H), np.float32)
    idx, w = orc.route(x, w_r, bias, 3)
    assert idx[0].tolist() == [5, 3, 7]
    np.testing.assert_allclose(w.sum(axis=1), 2.5, rtol=1e-12)


def test_dispatch_order_canonical():
    idx = np.array([[2, 0], [0, 1], [2, 1]], np.int32)
    perm_t, perm_l, offs = orc.dispatch_order(idx, 3)
    assert offs.tolist() == [0, 2, 4, 6]
    assert perm_t.tolist() == [0, 1, 1, 2, 0, 2]
    assert perm_l.tolist() == [1, 0, 1, 1, 0, 0]


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-3, 3.0e38], np.float32)
    b = f32_to_bf16_bits(x)
    import torch
    tb = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(b, tb)
    np.testing.assert_array_equal(round_bf16(x), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_zipf_bias_calibration_follows_targets():
    rng = np.random.default_rng(1)
    T, E, k = 2048, 64, 4
    logits = rng.normal(0, 1.5, (T, E))
    tgt = synth.zipf_targets(E, T, k, 1.1, rng)
    assert abs(tgt.sum() - T * k) < 1e-6 and tgt.max() <= T + 1e-9
    b = synth.calibrate_zipf_bias(logits, np.zeros(E, np.float32), k, tgt)
    idx, _ = orc.route(None, None, b, k, logits=logits)
    cnt = np.bincount(idx.reshape(-1), minlength=E)
    big = tgt > 20
    assert np.all(np.abs(np.log(cnt[big] / tgt[big])) < 0.25)


# ----------------------------------------------------------------------------- hyper-connections
def test_hc_oracle_matches_reference_hc_ref():
    """oracle.hc_mix / hc_apply against the reference's own hc_ref.mix / apply_ outputs
    (tests/golden/hc_kat.npz, made by tests/golden/make_golden.py)."""
    g = np.load(os.path.join(GOLD, "hc_kat.npz"))
    fn = (g["fn_bits"].astype(np.uint32) << 16).view(np.float32)
    post, comb, collapsed, pre = orc.hc_mix(g["streams"], fn, g["base"], g["scale"], float(g["rms_eps"]),
                                            float(g["hc_eps"]), int(g["iters"]))
    for a, b in ((post, g["post"]), (comb, g["comb"]), (collapsed, g["collapsed"]), (pre, g["pre"])):
        np.testing.assert_allclose(a, b, rtol=1e-12, atol=1e-14)
    out = orc.hc_apply(g["streams"], g["y"], post, comb)
    np.testing.assert_allclose(out, g["out"], rtol=1e-12, atol=1e-14)
    # the last Sinkhorn pass normalises columns: they sum to 1 (up to the hc_eps term)
    np.testing.assert_allclose(comb.sum(axis=-2), 1.0, atol=1e-5)

