"""Parity at the BASELINE configurations' full shapes (H=6144, I=2048, 256 experts, top-8), where
the other files check decode token subsets or C0-shaped stand-ins.

* C2 decode at T=1 (EXL3 3 bpw): the only token, against the oracle.
* C3 prefill with EXL3 3-bpw weights, T=4096, Zipf(1.1) routing: ids bit-exact for every token
  (the tcgen05 EXL3 GEMMs on hot and cold experts), output on tokens of the hottest and the
  coldest expert.
* C4 shape: four pre-norm layers at T=256: each layer teacher-forced (the oracle routes the GPU's
  own normed input), ids bit-exact for every token at every layer, an fp32-output twin of each
  layer within the bars on a token subset, and the stack's bf16 layer output equal to that twin
  rounded.

EXL3 oracles here take W^ from vfmoe_exl3_decode (pinned bit-exact to the oracle's decode
elsewhere) and reconstruct W in float64 (helpers.Built(what="gpu")).
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import moe, synth
from vybforge_b200.moe import MoELayer, quantizer
from vybforge_b200.stack import MoEStack

from helpers import Built, rel_l2, TOL_MAX_ABS, TOL_REL_L2

pytestmark = pytest.mark.gpu


def _check(tag, o, ro):
    print(f"[{tag}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2


def test_c2_t1_full_shape():
    moe.init(0)
    b = Built(synth.config("c2", tokens=1), weights="cuda", what="gpu")
    out, idx, w = b.layer.moe_block(b.x_dev)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    ro, ri, rw = b.oracle()
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    _check("c2 T=1 full shape", out.cpu().numpy(), ro)


def test_c3_exl3_full_shape():
    moe.init(0)
    cfg = synth.config("c3", tokens=4096, fmt="exl3")
    x, w_r, bias, _, _ = synth.zipf_router_inputs(cfg)
    b = Built(cfg, weights="cuda", router=(x, w_r, bias), what="gpu")
    out, idx, w = b.layer.moe_block(b.x_dev)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    ri, rw = orc.route(x, w_r, bias, cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    cnt = np.bincount(ri.reshape(-1), minlength=cfg.n_experts)
    assert cnt.max() > 3000
    hot, cold = int(np.argmax(cnt)), int(np.argmin(np.where(cnt > 0, cnt, 10**9)))
    toks = np.array(sorted({int(np.nonzero((ri == hot).any(1))[0][-1]), int(np.nonzero((ri == cold).any(1))[0][0])}))
    ro, _, _ = b.oracle(toks)
    _check(f"c3 exl3 T=4096 zipf tokens {toks.tolist()} (hot expert {hot}: {cnt[hot]} rows, cold {cold}: "
           f"{cnt[cold]})", out.cpu().numpy()[toks], ro)


class FullStack:
    """Four C1-shaped layers, Q8_0 on the GPU, bf16 activations, T tokens."""

    def __init__(self, T):
        cfg = synth.config("c4d", tokens=T)
        self.cfg = cfg
        self.x, self.norm_ws, self.routers = synth.stack_inputs(cfg, 4)
        self.dev = [synth.expert_q8_cuda(cfg, quantizer, layer=l) for l in range(4)]
        self.norm_dev = [torch.from_numpy(w).cuda() for w in self.norm_ws]
        self._mats = {}

    def layer(self, l, out_dtype=torch.bfloat16):
        cfg, E, d = self.cfg, self.cfg.n_experts, self.dev[l]
        w_r, bias, _ = self.routers[l]
        return MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk,
                        router_w=torch.from_numpy(w_r).cuda(), router_bias=torch.from_numpy(bias).cuda(),
                        gate=d[0][:E], up=d[1][:E], down=d[2][:E], shared=(d[0][E], d[1][E], d[2][E]),
                        x_dtype=torch.bfloat16, out_dtype=out_dtype)

    def mats(self, l, e):
        if (l, e) not in self._mats:
            H, I = self.cfg.hidden, self.cfg.inter
            g, u, d = (self.dev[l][p][e].cpu().numpy() for p in range(3))
            self._mats[(l, e)] = (orc.q8_0_expert_inout(g, I, H), orc.q8_0_expert_inout(u, I, H),
                                  orc.q8_0_expert_inout(d, H, I))
        return self._mats[(l, e)]


def test_c4_shape_stack_teacher_forced():
    moe.init(0)
    st = FullStack(256)
    cfg, E, k = st.cfg, st.cfg.n_experts, st.cfg.topk
    layers = [st.layer(l) for l in range(4)]
    s = MoEStack(layers, st.norm_dev)
    out, trace = s.forward(torch.from_numpy(st.x).to(torch.bfloat16).cuda(), trace=True)
    torch.cuda.synchronize()
    sub = np.array([0, 128, 255])
    for l, (h, y, idx) in enumerate(trace):
        w_r, bias, _ = st.routers[l]
        hf = h.float().cpu().numpy().astype(np.float64)
        ri, _ = orc.route(hf, w_r, bias, k)
        np.testing.assert_array_equal(idx.cpu().numpy(), ri)
        twin = st.layer(l, out_dtype=torch.float32)
        y32 = twin.forward(h)
        assert torch.equal(y, y32.to(torch.bfloat16))
        ro, _, _ = orc.moe_block_grouped(hf[sub], w_r, bias, lambda e: st.mats(l, e), lambda: st.mats(l, E), E, k)
        _check(f"c4 shape layer {l} teacher-forced, tokens {sub.tolist()}", y32.cpu().numpy()[sub], ro)
        twin.close()
    for lay in layers:
        lay.check_device_error()
