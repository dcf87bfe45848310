"""GPU parity of the EXL3 expert paths (3 bpw, and the reference's 4 bpw) against the oracle.

The oracle dequantizes every expert matrix the reference way (exl3_ref.py:84-120:
W = diag(suh) Hb W^ Hb diag(svh), float64 here) and runs the per-expert FFN; the GPU
rotates activations instead (fp16 rotated rows, fp32 accumulation).  Bars as for Q8_0:
ids bit-exact, output max-abs <= 2e-2 and rel-L2 <= 1e-3."""

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from vybforge_b200 import synth, moe

from helpers import Built, rel_l2, TOL_MAX_ABS, TOL_REL_L2

pytestmark = pytest.mark.gpu


def _check(b, out, idx, w, tokens, tag):
    ro, ri, rw = b.oracle(tokens)
    np.testing.assert_array_equal(idx, ri)
    np.testing.assert_allclose(w, rw, rtol=0, atol=1e-6)
    print(f"[parity {tag}] max-abs {np.abs(out - ro).max():.3e} rel-L2 {rel_l2(out, ro):.3e}")
    assert np.abs(out - ro).max() <= TOL_MAX_ABS
    assert rel_l2(out, ro) <= TOL_REL_L2


@pytest.fixture(scope="module")
def small():
    """C0 shapes (H=1024, I=512, 16 experts, top-4) with EXL3 weights, 64 tokens."""
    moe.init(0)
    return Built(synth.config("c0", tokens=64, fmt="exl3"))


@pytest.mark.parametrize("T", [1, 3, 16, 64])   # token tiles of 8, 8, 16 and 32 rows
def test_exl3_small_parity(small, T):
    x = small.x_dev[:T].contiguous()
    out, idx, w = small.layer.moe_block(x)
    torch.cuda.synchronize()
    small.layer.check_device_error()
    _check(small, out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), np.arange(T), f"exl3 c0-shape T={T}")


@pytest.fixture(scope="module")
def prefill():
    """C0 shapes with EXL3 weights, 256 tokens: 64 rows per expert on average, so the
    tcgen05 prefill kernels run (128-row gate/up tiles, 256-row down tiles)."""
    moe.init(0)
    return Built(synth.config("c0", tokens=256, fmt="exl3"))


def test_exl3_prefill_tcgen05_parity(prefill):
    b = prefill
    out, idx, w = b.layer.moe_block(b.x_dev)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    _check(b, out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), np.arange(b.cfg.tokens),
           "exl3 c0-shape T=256 tcgen05")


def test_exl3_prefill_and_decode_paths_agree(prefill):
    """Rows 0..15 through the decode GEMV (T=16: 4 rows per expert) and inside the T=256
    prefill batch (tcgen05): same per-token results up to fp32 summation order."""
    b = prefill
    full = b.layer.forward(b.x_dev)
    part = b.layer.forward(b.x_dev[:16].contiguous())
    d = rel_l2(part.cpu().numpy(), full[:16].cpu().numpy())
    print(f"[exl3 prefill vs decode path] rel-L2 {d:.3e}")
    assert d < 5e-4


def test_exl3_bf16_output_is_rounded_fp32_output(small):
    l16 = small.make_layer(torch.bfloat16)
    o16 = l16.forward(small.x_dev)
    o32 = small.layer.forward(small.x_dev)
    torch.testing.assert_close(o16, o32.to(torch.bfloat16), rtol=0, atol=0)


def test_exl3_deterministic(small):
    a = small.layer.forward(small.x_dev).clone()
    b = small.layer.forward(small.x_dev)
    assert torch.equal(a, b)


def test_exl3_forward_rows_matches_forward(small):
    """forward_rows (the expert-parallel entry) on the rows a forward would dispatch:
    slot = expert id, plus the shared expert as slot E; recombined equals forward."""
    T, k, E = 16, small.cfg.topk, small.cfg.n_experts
    x = small.x_dev[:T].contiguous()
    out, idx, w = small.layer.moe_block(x)
    rows = torch.cat([x.repeat_interleave(k, 0), x])
    slots = torch.cat([idx.reshape(-1), torch.full((T,), E, dtype=torch.int32, device=x.device)])
    y = small.layer.forward_rows(rows, slots)
    pos = torch.arange(T * k, dtype=torch.int32, device=x.device)
    got = moe.combine(y[:T * k], pos, w, T, k, y_shared=y[T * k:], out_dtype=torch.float32)
    torch.testing.assert_close(got, out, rtol=0, atol=1e-5)


def test_exl3_format_errors():
    """Bit widths other than 3 and 4 are declined with a status."""
    moe.init(0)
    cfg = synth.config("c0", tokens=4, fmt="exl3")
    b = Built(cfg)
    E = cfg.n_experts
    with pytest.raises(RuntimeError, match="exl3_bits must be 3 or 4"):
        moe.MoELayer(hidden=cfg.hidden, inter=cfg.inter, n_experts=E, topk=cfg.topk, router_w=b.wr_dev,
                     router_bias=b.bias_dev, gate=tuple(a[:E] for a in b.dev[0]),
                     up=tuple(a[:E] for a in b.dev[1]), down=tuple(a[:E] for a in b.dev[2]),
                     fmt="exl3", exl3_bits=5, x_dtype=torch.float32)


# ----------------------------------------------------------------------------- 4 bpw
def _cfg4(tokens):
    cfg = synth.config("c0", tokens=tokens, fmt="exl3")
    cfg.exl3_bits = 4
    return cfg


@pytest.fixture(scope="module")
def small4():
    """C0 shapes with EXL3 4-bpw weights (the reference's format), 64 tokens."""
    moe.init(0)
    return Built(_cfg4(64))


@pytest.mark.parametrize("T", [1, 16, 64])   # decode GEMV: token tiles of 8, 16 and 32 rows
def test_exl3_4bpw_decode_path_parity(small4, T):
    x = small4.x_dev[:T].contiguous()
    out, idx, w = small4.layer.moe_block(x)
    torch.cuda.synchronize()
    small4.layer.check_device_error()
    _check(small4, out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), np.arange(T), f"exl3-4bpw c0-shape T={T}")


def test_exl3_4bpw_prefill_tcgen05_parity():
    """256 tokens (64 rows per expert): the tcgen05 prefill kernels with 4-bpw tiles."""
    moe.init(0)
    b = Built(_cfg4(256))
    out, idx, w = b.layer.moe_block(b.x_dev)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    _check(b, out.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), np.arange(256), "exl3-4bpw c0-shape T=256 tcgen05")


# ----------------------------------------------------------------------------- full-size C2
def test_c2_decode_parity():
    """BASELINE C2 shapes (H=6144, I=2048, 256 experts, top-8, EXL3 3 bpw, bf16 x): T=32
    routed bit-exact; output checked on two tokens (the oracle dequantizes each of their
    experts' matrices in float64)."""
    moe.init(0)
    b = Built(synth.config("c2", tokens=32), weights="cuda")
    out, idx, w = b.layer.moe_block(b.x_dev)
    torch.cuda.synchronize()
    b.layer.check_device_error()
    ri, rw = orc.route(b.x, b.w_r, b.bias, b.cfg.topk)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    sub = np.array([0, 31])
    _check(b, out.cpu().numpy()[sub], idx.cpu().numpy()[sub], w.cpu().numpy()[sub], sub, "c2 T=32 tokens [0, 31]")
