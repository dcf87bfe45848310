"""GLM-5.3 layers as a checkpoint stores them, on the GPU.

* The dense (bf16-stored) shared expert (shared_format VFMOE_WFMT_BF16) beside Q8_0 routed experts,
  on the decode GEMV and the tcgen05 paths, against the oracle.
* A GLM-style MoE layer read from a synthetic sharded safetensors checkpoint (bf16 router, EXL3
  4-bpw routed experts with trellis/suh/svh/mcg per expert, bf16 shared expert) through
  vfmoe_ckpt_* and ckpt.glm_moe_layer: ids bit-exact and the output within the bars, against the
  oracle computed from the same tensors; expert parallelism on 2 virtual ranks; a packed-file round
  trip.  (The real checkpoint is not available here; the tensor names, dtypes and layouts are those
  of native/glm53/loader.py and gx_ref.py.)
"""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import ep, moe, synth
from vybforge_b200.ckpt import Checkpoint, glm_moe_layer
from vybforge_b200.moe import MoELayer

from ckpt_writer import glm_moe_tensors, write_sharded
from helpers import rel_l2, TOL_MAX_ABS, TOL_REL_L2

pytestmark = pytest.mark.gpu


def _bf16_to_f64(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _check(tag, o, ro):
    print(f"[{tag}] max-abs {np.abs(o - ro).max():.3e} rel-L2 {rel_l2(o, ro):.3e}")
    assert np.abs(o - ro).max() <= TOL_MAX_ABS and rel_l2(o, ro) <= TOL_REL_L2


@pytest.mark.parametrize("T,path", [(16, "auto"), (256, "auto")])
def test_dense_shared_expert_with_q8_0_routed(T, path):
    """Q8_0 routed experts (C0 shapes, bf16 x) + a bf16 shared expert [out, in]."""
    moe.init(0)
    from vybforge_b200.quant import f32_to_bf16_bits
    cfg = synth.config("c0", tokens=T)
    cfg.x_dtype = "bf16"
    x, w_r, bias, rng = synth.router_inputs(cfg)
    ex = synth.expert_q8_numpy(cfg, rng)
    H, I, E, k = cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk
    sh_bits = [f32_to_bf16_bits(rng.normal(0, 0.02, (I, H) if p < 2 else (H, I)).astype(np.float32)) for p in range(3)]
    dev = {p: torch.from_numpy(ex[p][:E]).cuda() for p in range(3)}
    sh_dev = tuple(torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16) for b in sh_bits)
    layer = MoELayer(hidden=H, inter=I, n_experts=E, topk=k, router_w=torch.from_numpy(w_r).cuda(),
                     router_bias=torch.from_numpy(bias).cuda(), gate=dev[0], up=dev[1], down=dev[2], shared=sh_dev,
                     shared_format="bf16", x_dtype=torch.bfloat16, out_dtype=torch.float32, path=path)
    out, idx, w = layer.moe_block(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    layer.check_device_error()

    def get(e):
        return (orc.q8_0_expert_inout(ex[0][e], I, H), orc.q8_0_expert_inout(ex[1][e], I, H),
                orc.q8_0_expert_inout(ex[2][e], H, I))
    shared = tuple(_bf16_to_f64(b).T for b in sh_bits)   # (in, out)
    ro, ri, rw = orc.moe_block_grouped(x, w_r, bias, get, lambda: shared, E, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    _check(f"dense shared expert + q8_0 T={T}", out.cpu().numpy(), ro)


@pytest.fixture(scope="module")
def glm_ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("glm53")
    rng = np.random.default_rng(53)
    H, I, E = 1024, 512, 16
    t = glm_moe_tensors(rng, 3, H, I, E, bits=4)
    write_sharded(str(d), t, n_shards=3)
    return str(d), t, (H, I, E)


def _oracle_for(t, H, I, E):
    pre = "model.language_model.layers.3.mlp."
    w_r = _bf16_to_f64(t[pre + "gate.weight"][1]).astype(np.float32)
    bias = t[pre + "gate.e_score_correction_bias"][1]
    cache = {}

    def get(e):
        if e not in cache:
            mats = []
            for p in ("gate_proj", "up_proj", "down_proj"):
                q = f"{pre}experts.{e}.{p}."
                mats.append(orc.dequant_exl3(t[q + "trellis"][1].view(np.uint16), t[q + "suh"][1], t[q + "svh"][1], 4))
            cache[e] = tuple(mats)
        return cache[e]
    shared = tuple(_bf16_to_f64(t[f"{pre}shared_experts.{p}.weight"][1]).T for p in ("gate_proj", "up_proj", "down_proj"))
    return w_r, bias, get, shared


@pytest.mark.parametrize("T", [8, 256])
def test_glm_layer_from_checkpoint_matches_oracle(glm_ckpt, T):
    moe.init(0)
    path, t, (H, I, E) = glm_ckpt
    ck = Checkpoint(path)
    layer, info = glm_moe_layer(ck, 3, topk=4, out_dtype=torch.float32)
    assert info == {"H": H, "I": I, "E": E, "bits": 4}
    rng = np.random.default_rng(T)
    from vybforge_b200.quant import round_bf16
    x = round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    out, idx, w = layer.moe_block(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    layer.check_device_error()
    w_r, bias, get, shared = _oracle_for(t, H, I, E)
    ro, ri, rw = orc.moe_block_grouped(x, w_r, bias, get, lambda: shared, E, 4)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=0, atol=1e-6)
    _check(f"glm layer from checkpoint T={T}", out.cpu().numpy(), ro)
    layer.close()
    ck.close()


def test_glm_layer_from_checkpoint_expert_parallel_and_packed(glm_ckpt, tmp_path):
    """The same layer on 2 virtual ranks (each rank's layer holds its 8 experts and the bf16 shared
    expert), and written to / read from a packed layer file: both equal the single layer."""
    moe.init(0)
    path, t, (H, I, E) = glm_ckpt
    ck = Checkpoint(path)
    full, _ = glm_moe_layer(ck, 3, topk=4, out_dtype=torch.float32)
    rng = np.random.default_rng(2)
    from vybforge_b200.quant import round_bf16
    T, world = 32, 2
    x = torch.from_numpy(round_bf16(rng.standard_normal((T, H)).astype(np.float32))).to(torch.bfloat16).cuda()
    ref = full.forward(x)
    # packed file round trip (EXL3 routed + bf16 shared sections)
    pk = str(tmp_path / "glm3.vfpk")
    full.save_packed(pk)
    back = MoELayer.from_packed(pk)
    assert torch.equal(back.forward(x), ref)
    # expert parallel: placement halves, rank r's experts sliced from the full stacks
    placement = ep.contiguous_placement(E, world)
    ranks = []
    for r in range(world):
        ids = torch.as_tensor(np.nonzero(placement == r)[0], device="cuda")
        g, u, dn = ([a[ids].contiguous() for a in m] for m in (full._keep[2], full._keep[3], full._keep[4]))
        L = MoELayer(hidden=H, inter=I, n_experts=E, topk=4, router_w=full._keep[0], router_bias=full._keep[1],
                     gate=tuple(g), up=tuple(u), down=tuple(dn), shared=full._keep[5], fmt="exl3", exl3_bits=4,
                     x_dtype=torch.bfloat16, out_dtype=torch.float32, shared_format="bf16", n_local_experts=E // world)
        ranks.append(ep.EpLayer(L, placement, r, world, T // world))
    outs = ep.ep_forward_virtual(ranks, [x[:T // 2].contiguous(), x[T // 2:].contiguous()])
    got = torch.cat(outs).cpu().numpy()
    for r in ranks:
        r.layer.check_device_error()
    d = rel_l2(got, ref.cpu().numpy())
    print(f"[glm layer from checkpoint, ep virtual N=2] rel-L2 vs single layer {d:.3e}")
    assert d < 1e-4
    back.close()
    full.close()
    ck.close()
