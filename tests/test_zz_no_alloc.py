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
