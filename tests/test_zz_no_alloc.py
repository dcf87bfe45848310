"""vfmoe_route_noalloc, the router entry point that allocates no device memory.

It exists for hosts that cannot call cudaMalloc while routing: cudaMalloc may synchronize
the device, and it fails once a host has reserved all of device memory in its own pool.
Its scratch is a fixed-size device array inside libvfmoe.so that every call shares.
These tests call it through the C ABI and compare it with vfmoe_route, the entry point
that takes a workspace, on two calls in a row.  The file is collected last on purpose
and is self-contained, so it also passes alone in a fresh process.
"""

import numpy as np
import pytest
import torch

from vybforge_b200 import _lib, synth
from vybforge_b200.moe import MoELayer, init

pytestmark = pytest.mark.gpu


def _stream():
    return int(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def routing_layer():
    init(0)
    cfg = synth.config("c1", tokens=64)
    x, w_r, bias, _ = synth.router_inputs(cfg)
    E, H, I = cfg.n_experts, cfg.hidden, 256
    # expert weights are never read by the router; small zero stacks satisfy the descriptor
    gu = torch.zeros((E, I, H // 32 * 34), dtype=torch.uint8, device="cuda")
    dn = torch.zeros((E, H, I // 32 * 34), dtype=torch.uint8, device="cuda")
    layer = MoELayer(hidden=H, inter=I, n_experts=E, topk=cfg.topk, router_w=torch.from_numpy(w_r).cuda(),
                     router_bias=torch.from_numpy(bias).cuda(), gate=gu, up=gu, down=dn,
                     x_dtype=torch.bfloat16, out_dtype=torch.float32)
    return layer, torch.from_numpy(x).to(torch.bfloat16).cuda(), cfg


def _route_noalloc(layer, x, T):
    k = layer.k
    idx = torch.full((T, k), -1, dtype=torch.int32, device="cuda")
    w = torch.full((T, k), -1.0, dtype=torch.float32, device="cuda")
    rc = layer.lib.vfmoe_route_noalloc(layer.handle, int(x.data_ptr()), T, int(idx.data_ptr()),
                                       int(w.data_ptr()), _stream())
    assert rc == 0, _lib.last_error()
    return idx, w


def test_noalloc_route_matches_workspace_route_on_two_calls(routing_layer):
    layer, x, cfg = routing_layer
    for T in (32, 7):                       # two calls in a row, sizes that differ
        xt = x[:T].contiguous()
        idx_ref, w_ref = layer.route(xt)    # existing entry point (workspace)
        idx, w = _route_noalloc(layer, xt, T)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(idx.cpu().numpy(), idx_ref.cpu().numpy())
        np.testing.assert_allclose(w.cpu().numpy(), w_ref.cpu().numpy(), rtol=0, atol=1e-6)
    layer.check_device_error()


def test_noalloc_route_prefill_path_two_calls(routing_layer):
    layer, x, cfg = routing_layer
    xt = x[:64].contiguous()                # T > 32 takes the tiled logits kernel
    idx_ref, w_ref = layer.route(xt)
    a = _route_noalloc(layer, xt, 64)
    b = _route_noalloc(layer, xt, 64)
    torch.cuda.synchronize()
    for idx, w in (a, b):
        np.testing.assert_array_equal(idx.cpu().numpy(), idx_ref.cpu().numpy())
        np.testing.assert_allclose(w.cpu().numpy(), w_ref.cpu().numpy(), rtol=0, atol=1e-6)


def test_noalloc_route_rejects_sizes_beyond_its_scratch(routing_layer):
    layer, x, cfg = routing_layer
    T = 8192                                 # 8192 x 256 fp32 logits > the 4 MiB scratch
    big = torch.zeros((T, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    idx = torch.empty((T, layer.k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, layer.k), dtype=torch.float32, device="cuda")
    rc = layer.lib.vfmoe_route_noalloc(layer.handle, int(big.data_ptr()), T, int(idx.data_ptr()),
                                       int(w.data_ptr()), _stream())
    assert rc == _lib.ERR_UNSUPPORTED
    assert "static scratch" in _lib.last_error()


def test_noalloc_route_limit_is_t127_at_c1_shapes(routing_layer):
    """The documented limit at E = 256, H = 6144: T = 127 fits the scratch and routes like
    vfmoe_route; T = 128 is rejected before anything is launched."""
    layer, x, cfg = routing_layer
    g = torch.Generator(device="cuda").manual_seed(127)
    x127 = torch.randn((127, cfg.hidden), generator=g, device="cuda").to(torch.bfloat16)
    idx_ref, w_ref = layer.route(x127)
    idx, w = _route_noalloc(layer, x127, 127)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx.cpu().numpy(), idx_ref.cpu().numpy())
    np.testing.assert_allclose(w.cpu().numpy(), w_ref.cpu().numpy(), rtol=0, atol=1e-6)
    x128 = torch.zeros((128, cfg.hidden), dtype=torch.bfloat16, device="cuda")
    idx = torch.empty((128, layer.k), dtype=torch.int32, device="cuda")
    w = torch.empty((128, layer.k), dtype=torch.float32, device="cuda")
    rc = layer.lib.vfmoe_route_noalloc(layer.handle, int(x128.data_ptr()), 128, int(idx.data_ptr()),
                                       int(w.data_ptr()), _stream())
    assert rc == _lib.ERR_UNSUPPORTED
    assert "static scratch" in _lib.last_error()


def test_noalloc_route_hidden_not_multiple_of_512():
    """H = 1280 is a multiple of 256 but of neither 768 nor 512, so even at T <= 32 the tiled
    logits kernel runs with its own K-slice count; the scratch sizing must use that count.
    Both entry points against the f64 oracle, two calls in a row."""
    from oracle import moe_oracle as orc
    init(0)
    rng = np.random.default_rng(1280)
    H, E, k, T = 1280, 256, 8, 24
    from vybforge_b200.quant import round_bf16
    x = round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    w_r = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    bias = rng.normal(0, 0.01, E).astype(np.float32)
    I = 256
    gu = torch.zeros((E, I, H // 32 * 34), dtype=torch.uint8, device="cuda")
    dn = torch.zeros((E, H, I // 32 * 34), dtype=torch.uint8, device="cuda")
    layer = MoELayer(hidden=H, inter=I, n_experts=E, topk=k, router_w=torch.from_numpy(w_r).cuda(),
                     router_bias=torch.from_numpy(bias).cuda(), gate=gu, up=gu, down=dn,
                     x_dtype=torch.bfloat16, out_dtype=torch.float32)
    xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
    ri, rw = orc.route(x, w_r, bias, k)
    for _ in range(2):
        idx_ws, w_ws = layer.route(xd)
        idx, w = _route_noalloc(layer, xd, T)
        torch.cuda.synchronize()
        for a, b in ((idx_ws, w_ws), (idx, w)):
            np.testing.assert_array_equal(a.cpu().numpy(), ri)
            np.testing.assert_allclose(b.cpu().numpy(), rw, rtol=0, atol=1e-6)
    layer.check_device_error()
    layer.close()
