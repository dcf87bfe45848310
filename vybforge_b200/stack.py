"""Pre-norm stack of MoE layers: x <- x + MoE_l(RMSNorm_l(x)) for l = 0..L-1.

This is the 4-layer expert-parallel workload built from GLM MoE layers.  The reference
engine (native/glm53/glm_engine.vyb) mixes layers through hyper-connections; this stack
uses the plain pre-norm residual instead.  The oracle's ``moe_stack`` mirrors it.

- ``MoEStack``: all layers on one GPU.
- ``EpStack``: one rank's share of the expert-parallel stack.  Tokens are sharded over
  ranks; each layer is an ``ep.EpLayer`` over this rank's experts (``vfmoe_ep_forward``).

Every step is a libvfmoe kernel:
- ``vfmoe_residual_rmsnorm`` fuses layer l's residual add with layer l+1's input norm.
- The layer itself is ``vfmoe_forward`` or the expert-parallel entry points.
"""

from __future__ import annotations

import numpy as np
import torch

from . import ep
from .moe import residual_rmsnorm


class MoEStack:
    def __init__(self, layers, norm_w, eps: float = 1e-5):
        """layers: list of MoELayer; norm_w: list of fp32 [H] device tensors (one per layer)."""
        assert len(layers) == len(norm_w) and layers
        self.layers, self.norm_w, self.eps = layers, norm_w, eps

    def forward(self, x: torch.Tensor, trace: bool = False):
        """x [T, H] (the layers' x dtype) -> residual stream after the last layer.
        trace=True also returns per layer (h, y, idx): normed input, layer output, expert ids."""
        L = len(self.layers)
        x, h = residual_rmsnorm(x, None, self.norm_w[0], self.eps)
        tr = []
        for l, layer in enumerate(self.layers):
            if trace:
                y, idx, _ = layer.moe_block(h)
                tr.append((h, y, idx))
            else:
                y = layer.forward(h)
            x, h = residual_rmsnorm(x, y, self.norm_w[l + 1] if l + 1 < L else None, self.eps)
        return (x, tr) if trace else x


class EpStack:
    def __init__(self, layers, norm_w, eps: float = 1e-5):
        """layers: list (one per layer) of ep.EpLayer of this process's rank."""
        assert len(layers) == len(norm_w) and layers
        self.layers, self.norm_w, self.eps = layers, norm_w, eps

    def forward(self, comm, x: torch.Tensor, mark=None) -> torch.Tensor:
        """This rank's tokens through all layers over the library's NCCL communicator `comm`
        (ep.EpComm); mark(name), if given, is called after each norm and each layer."""
        L = len(self.layers)
        x, h = residual_rmsnorm(x, None, self.norm_w[0], self.eps)
        if mark:
            mark("norm")
        for l, lay in enumerate(self.layers):
            y = lay.forward(comm, h)
            if mark:
                mark("layer")
            x, h = residual_rmsnorm(x, y, self.norm_w[l + 1] if l + 1 < L else None, self.eps)
            if mark:
                mark("norm")
        return x


def ep_stack_forward_virtual(stacks, xs):
    """N virtual ranks held by one process (see ep.ep_forward_virtual)."""
    L = len(stacks[0].layers)
    eps = stacks[0].eps
    state = [residual_rmsnorm(x, None, s.norm_w[0], eps) for s, x in zip(stacks, xs)]
    for l in range(L):
        ys = ep.ep_forward_virtual([s.layers[l] for s in stacks], [h for _, h in state])
        state = [residual_rmsnorm(x, y, s.norm_w[l + 1] if l + 1 < L else None, eps)
                 for s, (x, _), y in zip(stacks, state, ys)]
    return [x for x, _ in state]


def token_shards(T: int, world: int):
    """Contiguous token ranges per rank (sizes differ by at most one)."""
    return np.array_split(np.arange(T), world)
