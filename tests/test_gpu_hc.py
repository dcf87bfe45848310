"""Hyper-connections around the MoE (GLM-5.3 multi-stream residual) on the GPU.

* vfmoe_hc_mix / vfmoe_hc_apply against the reference's own hc_ref.mix / apply_ outputs
  (tests/golden/hc_kat.npz) and against the oracle at D = 4096 (GLM-5.3) and 6144 (the C1
  shape), with the weighted RMSNorm that feeds the MoE fused into the mix.
* The whole MoE site (tail_site, native/glm53/glm_engine.vyb:2562-3019): mix -> RMSNorm ->
  MoE -> apply, against the oracle's composition; the MoE ids teacher-forced bit-exact.
Bars: fp32 outputs of the mix within 1e-5 relative (fp32 products, fp64 reductions); the MoE
site within the MoE bars (max-abs 2e-2, rel-L2 1e-3).
"""

import os

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import moe, synth
from vybforge_b200.moe import HyperConnection, MoELayer, hc_moe_site
from vybforge_b200.quant import f32_to_bf16_bits, quantize_q8_0

from helpers import rel_l2, TOL_MAX_ABS, TOL_REL_L2

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bf16_tensor(bits):
    return torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)


def test_hc_matches_reference_golden():
    moe.init(0)
    g = np.load(os.path.join(GOLD, "hc_kat.npz"))
    site = HyperConnection(_bf16_tensor(g["fn_bits"]), torch.from_numpy(g["base"]).cuda(),
                           torch.from_numpy(g["scale"]).cuda(), norm_w=None, rms_eps=float(g["rms_eps"]),
                           hc_eps=float(g["hc_eps"]), sinkhorn_iters=int(g["iters"]))
    streams = torch.from_numpy(g["streams"]).cuda()
    h, post, comb = site.mix(streams, h_dtype=torch.float32)
    out = site.apply(streams, torch.from_numpy(g["y"]).cuda(), post, comb)
    torch.cuda.synchronize()
    np.testing.assert_allclose(post.cpu().numpy(), g["post"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(comb.cpu().numpy(), g["comb"], rtol=1e-5, atol=1e-7)
    d_col = rel_l2(h.cpu().numpy(), g["collapsed"])
    d_out = rel_l2(out.cpu().numpy(), g["out"])
    print(f"[hc golden] collapsed rel-L2 {d_col:.2e}, apply rel-L2 {d_out:.2e}")
    assert d_col < 1e-6 and d_out < 1e-6


@pytest.mark.parametrize("D,fn_bf16,R", [(4096, True, 37), (6144, True, 37), (2048, False, 37), (8192, True, 37),
                                          (6144, True, 1030), (2048, False, 1030), (4096, True, 257),
                                          (8192, True, 300)])
def test_hc_mix_and_apply_match_oracle(D, fn_bf16, R):
    """R = 37 takes the one-row-per-CTA mix; from R = 256 a bf16 hc_fn takes the tensor-core mix
    (16 rows per CTA; R = 257 and 300 end in a partial block), an fp32 one the two-rows-per-CTA
    mix (R = 1030)."""
    moe.init(0)
    rng = np.random.default_rng(D + R)
    streams = (rng.standard_normal((R, 4, D)) * rng.uniform(0.2, 3.0, (R, 4, 1))).astype(np.float32)
    fn = (rng.standard_normal((24, 4 * D)) * 0.02).astype(np.float32)
    if fn_bf16:
        bits = f32_to_bf16_bits(fn)
        fn = (bits.astype(np.uint32) << 16).view(np.float32)
        fn_dev = _bf16_tensor(bits)
    else:
        fn_dev = torch.from_numpy(fn).cuda()
    base = rng.normal(0, 0.5, 24).astype(np.float32)
    scale = np.array([0.7, 1.1, 1.9], np.float32)
    norm_w = (1 + rng.normal(0, 0.05, D)).astype(np.float32)
    site = HyperConnection(fn_dev, torch.from_numpy(base).cuda(), torch.from_numpy(scale).cuda(),
                           norm_w=torch.from_numpy(norm_w).cuda())
    sd = torch.from_numpy(streams).cuda()
    h32, post, comb = site.mix(sd, h_dtype=torch.float32)
    h16, _, _ = site.mix(sd, h_dtype=torch.bfloat16)
    rp, rc, rcol, _ = orc.hc_mix(streams, fn, base, scale, 1e-5)
    rh = orc.rmsnorm(rcol, norm_w, 1e-5)
    np.testing.assert_allclose(post.cpu().numpy(), rp, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(comb.cpu().numpy(), rc, rtol=1e-5, atol=1e-7)
    d32, d16 = rel_l2(h32.cpu().numpy(), rh), rel_l2(h16.float().cpu().numpy(), rh)
    y = rng.standard_normal((R, D)).astype(np.float32)
    yd = torch.from_numpy(y).to(torch.bfloat16).cuda()
    out = site.apply(sd, yd, post, comb)
    ro = orc.hc_apply(streams, yd.float().cpu().numpy(), post.cpu().numpy().astype(np.float64),
                      comb.cpu().numpy().astype(np.float64))
    d_out = rel_l2(out.cpu().numpy(), ro)
    inplace = sd.clone()
    site.apply(inplace, yd, post, comb, out=inplace)
    torch.cuda.synchronize()
    print(f"[hc D={D} R={R} fn {'bf16' if fn_bf16 else 'f32'}] h fp32 {d32:.2e}, h bf16 {d16:.2e}, apply {d_out:.2e}")
    assert d32 < 1e-5 and d16 < 4e-3 and d_out < 1e-6
    assert torch.equal(inplace, out)


def test_hc_moe_site_matches_oracle_composition():
    """tail_site: streams -> mix + post-attention RMSNorm -> MoE (Q8_0, D = 2048, 16 experts,
    top-4, bf16 activations) -> residual update, against the oracle composition run on the GPU's
    own normed input (teacher-forced routing)."""
    moe.init(0)
    rng = np.random.default_rng(5)
    R, D, I, E, k = 24, 2048, 512, 16, 4
    streams = rng.standard_normal((R, 4, D)).astype(np.float32)
    bits = f32_to_bf16_bits((rng.standard_normal((24, 4 * D)) * 0.02).astype(np.float32))
    fn = (bits.astype(np.uint32) << 16).view(np.float32)
    base = rng.normal(0, 0.5, 24).astype(np.float32)
    scale = np.array([0.7, 1.1, 1.9], np.float32)
    norm_w = (1 + rng.normal(0, 0.02, D)).astype(np.float32)
    w_r = rng.normal(0, 0.02, (E, D)).astype(np.float32)
    bias = rng.normal(0, 0.01, E).astype(np.float32)
    mats = {p: np.stack([quantize_q8_0(rng.normal(0, 0.02, (I, D) if p < 2 else (D, I)).astype(np.float32))
                         for _ in range(E + 1)]) for p in range(3)}
    dev = {p: torch.from_numpy(mats[p]).cuda() for p in range(3)}
    layer = MoELayer(hidden=D, inter=I, n_experts=E, topk=k, router_w=torch.from_numpy(w_r).cuda(),
                     router_bias=torch.from_numpy(bias).cuda(), gate=dev[0][:E], up=dev[1][:E], down=dev[2][:E],
                     shared=(dev[0][E], dev[1][E], dev[2][E]), x_dtype=torch.bfloat16, out_dtype=torch.bfloat16)
    site = HyperConnection(_bf16_tensor(bits), torch.from_numpy(base).cuda(), torch.from_numpy(scale).cuda(),
                           norm_w=torch.from_numpy(norm_w).cuda())
    sd = torch.from_numpy(streams).cuda()
    h, post, comb = site.mix(sd, h_dtype=torch.bfloat16)
    out = hc_moe_site(site, layer, sd)
    _, idx, _ = layer.moe_block(h)
    torch.cuda.synchronize()
    layer.check_device_error()

    def get(e):
        return (orc.q8_0_expert_inout(mats[0][e], I, D), orc.q8_0_expert_inout(mats[1][e], I, D),
                orc.q8_0_expert_inout(mats[2][e], D, I))
    hf = h.float().cpu().numpy().astype(np.float64)
    y, ri, _ = orc.moe_block_grouped(hf, w_r, bias, get, lambda: get(E), E, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    rp, rc, rcol, _ = orc.hc_mix(streams, fn, base, scale, 1e-5)
    ro = orc.hc_apply(streams, y, rp, rc)
    o = out.cpu().numpy()
    print(f"[hc moe site] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2
