"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own
Python modules (rickenator/VybForge):

  native/glm53/moe_ref.py   route / moe_block (router + clamped SwiGLU block)
  native/tools/q8_0_ref.py  q8_0_ours (Q8_0 block decode)
  native/exl3/exl3_ref.py   decode_mcg, dequant_exl3 (4-bpw, verified slot map)
  native/glm53/hc_ref.py    mix / apply_ (GLM-5.3 hyper-connections)

and by copying the reference's committed real-weight router case (native/glm53/prep: GLM router
weights of one layer, bf16-valued, its correction bias, four hidden rows and the reference's
ids and weights for them).

Usage (needs the reference checkout; the fixtures are committed, so the tests
themselves never read the reference):

    python tests/golden/make_golden.py [REFERENCE_ROOT [c0 q8 exl3 hc prep]]

REFERENCE_ROOT defaults to $VYBFORGE_REFERENCE, else a "reference" checkout beside this
repository.

Inputs are regenerated from seeds by vybforge_b200.synth; each fixture stores
the sha256 of every input array so generator drift is caught, plus the
reference outputs.
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from vybforge_b200 import synth  # noqa: E402
from vybforge_b200.quant import quantize_q8_0, f32_to_bf16_bits  # noqa: E402


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def c0_fixture(ref):
    """Config C0 through the reference moe_ref.moe_block (H patched to 1024)."""
    moe_ref = load_module("moe_ref", os.path.join(ref, "native/glm53/moe_ref.py"))
    q8 = load_module("q8_0_ref", os.path.join(ref, "native/tools/q8_0_ref.py"))
    cfg = synth.config("c0")
    x, w_r, bias, rng = synth.router_inputs(cfg)
    experts = synth.expert_q8_numpy(cfg, rng)
    H, I, E, k = cfg.hidden, cfg.inter, cfg.n_experts, cfg.topk

    def deq(proj, e):
        rows, cols = (I, H) if proj != synth.PROJ_DOWN else (H, I)
        return q8.q8_0_ours(experts[proj][e].tobytes()).reshape(rows, cols).T.copy()  # (in, out)

    ew = {e: (deq(0, e), deq(1, e), deq(2, e)) for e in range(E)}
    sw = (deq(0, E), deq(1, E), deq(2, E))
    moe_ref.HIDDEN = H                      # moe_block allocates [S, HIDDEN]
    out, idx, w = moe_ref.moe_block(x.astype(np.float64), w_r, bias, ew, sw, topk=k)
    np.savez_compressed(
        os.path.join(HERE, "c0_moe_block.npz"),
        x_sha=sha(x), w_r_sha=sha(w_r), bias_sha=sha(bias),
        gate_sha=sha(experts[0]), up_sha=sha(experts[1]), down_sha=sha(experts[2]),
        idx=idx.astype(np.int64), w=w.astype(np.float64), out=out.astype(np.float64),
        x=x, w_r=w_r, bias=bias)
    print("c0_moe_block.npz: out", out.shape, "idx", idx.shape)


def q8_fixture(ref):
    """Q8_0 decode known answers from the reference q8_0_ours on edge-case blocks."""
    q8 = load_module("q8_0_ref", os.path.join(ref, "native/tools/q8_0_ref.py"))
    rng = np.random.default_rng(7)
    rows = [rng.normal(0, 0.02, 64), np.zeros(64), rng.normal(0, 100.0, 64),
            np.concatenate([np.full(32, -3.5), np.linspace(-1, 1, 32)]),
            rng.normal(0, 1e-4, 64)]
    w = np.stack(rows).astype(np.float32)
    raw = quantize_q8_0(w)
    dq = q8.q8_0_ours(raw.tobytes()).reshape(w.shape)
    np.savez_compressed(os.path.join(HERE, "q8_0_kat.npz"), raw=raw, deq=dq)
    print("q8_0_kat.npz:", raw.shape)


def exl3_fixture(ref):
    """EXL3: decode_mcg over all 2^16 windows, and a 4-bpw 128x128 dequant_exl3."""
    ex = load_module("exl3_ref", os.path.join(ref, "native/exl3/exl3_ref.py"))
    allw = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    vals = ex.decode_mcg(allw)
    rng = np.random.default_rng(11)
    tr = rng.integers(0, 1 << 16, size=(8, 8, 64), dtype=np.uint32).astype(np.uint16)
    suh = np.where(rng.random(128) < 0.5, -1.0, 1.0).astype(np.float16)
    svh = (np.where(rng.random(128) < 0.5, -1.0, 1.0) * rng.uniform(0.01, 0.03, 128)).astype(np.float16)
    w4 = ex.dequant_exl3(tr, suh, svh)
    slots, cidx, cpos = ex.load_slot_composition()
    np.savez_compressed(os.path.join(HERE, "exl3_kat.npz"), mcg_bits=vals.view(np.uint16),
                        tr4=tr, suh4=suh, svh4=svh, w4=w4.view(np.uint16),
                        slot_rc=slots.astype(np.int16), slot_nibble=cidx.astype(np.int16),
                        slot_pos=cpos.astype(np.int8))
    print("exl3_kat.npz: 65536 windows, W", w4.shape)


def hc_fixture(ref):
    """Hyper-connections: the reference's hc_ref.mix / apply_ on seeded streams (R=3, HC=4, D=2048)
    with bf16-valued fn, and the reference engine's default eps values."""
    hc = load_module("hc_ref", os.path.join(ref, "native/glm53/hc_ref.py"))
    rng = np.random.default_rng(23)
    R, HC, D = 3, 4, 2048
    streams = (rng.standard_normal((R, HC, D)) * rng.uniform(0.5, 2.0, (R, HC, 1))).astype(np.float32)
    fn_bits = f32_to_bf16_bits((rng.standard_normal((24, HC * D)) * 0.02).astype(np.float32))
    fn = (fn_bits.astype(np.uint32) << 16).view(np.float32)
    base = rng.normal(0, 0.5, 24).astype(np.float32)
    scale = np.array([0.8, 1.3, 2.0], np.float32)
    y = rng.standard_normal((R, D)).astype(np.float32)
    post, comb, collapsed, pre = hc.mix(streams, fn, base, scale, 1e-5)
    out = hc.apply_(streams, y, post, comb)
    np.savez_compressed(os.path.join(HERE, "hc_kat.npz"), streams=streams, fn_bits=fn_bits, base=base, scale=scale,
                        y=y, rms_eps=np.float64(1e-5), hc_eps=np.float64(hc.Hc_EPS),
                        iters=np.int64(hc.SINKHORN_ITERS), post=post, comb=comb, collapsed=collapsed, pre=pre,
                        out=out)
    print("hc_kat.npz: R", R, "D", D)


def prep_router_fixture(ref):
    """The router part of native/glm53/prep (S=4, H=4096, E=288, k=8): gate.f32 holds bf16 values,
    so it is stored as bf16 bits; y, bias and the reference's ref_idx / ref_w as they are."""
    d = os.path.join(ref, "native/glm53/prep")
    H, E, k = 4096, 288, 8

    def f(n, shape):
        return np.fromfile(os.path.join(d, n + ".f32"), dtype="<f4").reshape(shape)
    gate = f("gate", (E, H))
    bits = (gate.view(np.uint32) >> 16).astype(np.uint16)
    assert np.array_equal((bits.astype(np.uint32) << 16).view(np.float32), gate), "gate.f32 is not bf16-valued"
    np.savez_compressed(os.path.join(HERE, "glm_router_prep.npz"), gate_bits=bits, bias=f("bias", (E,)),
                        y=f("y", (4, H)), ref_idx=f("ref_idx", (4, k)).astype(np.int32), ref_w=f("ref_w", (4, k)))
    print("glm_router_prep.npz: S 4, H", H, "E", E, "k", k)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get(
        "VYBFORGE_REFERENCE", os.path.normpath(os.path.join(REPO, os.pardir, "reference")))
    if not os.path.isdir(os.path.join(ref, "native")):
        sys.exit(f"reference checkout not found at {ref}")
    which = sys.argv[2:] or ["c0", "q8", "exl3", "hc", "prep"]
    for name in which:
        {"c0": c0_fixture, "q8": q8_fixture, "exl3": exl3_fixture, "hc": hc_fixture,
         "prep": prep_router_fixture}[name](ref)


if __name__ == "__main__":
    main()
