"""Checkpoint access for GLM-5.3 MoE layers over libvfmoe (vfmoe_ckpt_*).

The reference resolves tensor names through its gx index (native/glm53/gx.vyb:41-99: index ->
shard -> safetensors header -> byte range; native/torchload/safetensors.vyb) and dequantizes
experts on demand (native/glm53/loader.py).  Here the library resolves and reads the bytes
(straight into device memory), and ``glm_moe_layer`` builds a ``MoELayer`` from one layer's
tensors as stored:

  mlp.gate.weight                      bf16 [E, H]   -> fp32 router weights (exact)
  mlp.gate.e_score_correction_bias     f32 [E]
  mlp.experts.<e>.<proj>.trellis       int16 [in/16, out/16, 16*bits]   EXL3, stacked over e
  mlp.experts.<e>.<proj>.suh / .svh    f16 [in] / [out]
  mlp.experts.<e>.<proj>.mcg           i32 [1]       (the mcg codebook; required)
  mlp.shared_experts.<proj>.weight     bf16 [out, in] -> shared_format "bf16"

No weight is dequantized at load: the kernels decode EXL3 trellis on the fly.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import check

_TORCH = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "F64": torch.float64,
          "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
          "BOOL": torch.bool}
_NUMPY = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "F64": np.float64, "I64": np.int64,
          "I32": np.int32, "I16": np.int16, "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_, "U16": np.uint16,
          "U32": np.uint32, "U64": np.uint64}

PROJS = ("gate_proj", "up_proj", "down_proj")


class Checkpoint:
    """A safetensors checkpoint directory (model.safetensors.index.json + shards, or one
    model.safetensors)."""

    def __init__(self, path: str):
        self.lib = _lib.load()
        self.path = path
        self.handle = check(self.lib.vfmoe_ckpt_open(path.encode()))

    def info(self, name: str) -> dict:
        t = _lib.TensorInfo()
        check(self.lib.vfmoe_ckpt_find(self.handle, name.encode(), C.byref(t)))
        return {"dtype": _lib.ST_NAMES[t.dtype], "shape": tuple(t.shape[:t.ndim]), "nbytes": t.nbytes,
                "offset": t.file_offset, "shard": t.shard}

    def has(self, name: str) -> bool:
        t = _lib.TensorInfo()
        return self.lib.vfmoe_ckpt_find(self.handle, name.encode(), C.byref(t)) == 0

    def read_into(self, name: str, dst: torch.Tensor) -> torch.Tensor:
        """The tensor's bytes into dst (CUDA or contiguous CPU tensor of at least its size)."""
        assert dst.is_contiguous()
        check(self.lib.vfmoe_ckpt_read(self.handle, name.encode(), int(dst.data_ptr()),
                                       dst.numel() * dst.element_size(), 1 if dst.is_cuda else 0))
        return dst

    def read(self, name: str, device="cuda") -> torch.Tensor:
        i = self.info(name)
        if i["dtype"] not in _TORCH:
            raise ValueError(f"{name}: dtype {i['dtype']} has no torch counterpart here")
        out = torch.empty(i["shape"], dtype=_TORCH[i["dtype"]], device=device)
        return self.read_into(name, out)

    def read_numpy(self, name: str) -> np.ndarray:
        """Host copy (BF16 as its uint16 bit patterns)."""
        i = self.info(name)
        out = np.empty(i["shape"], dtype=_NUMPY[i["dtype"]])
        check(self.lib.vfmoe_ckpt_read(self.handle, name.encode(), out.ctypes.data, out.nbytes, 0))
        return out

    def close(self):
        if getattr(self, "handle", 0) > 0:
            self.lib.vfmoe_ckpt_close(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def glm_moe_layer(ck: Checkpoint, layer: int, *, topk: int = 8, scale: float = 2.5, limit: float = 10.0,
                  x_dtype=torch.bfloat16, out_dtype=torch.bfloat16,
                  prefix: str = "model.language_model.layers."):
    """The MoE layer `layer` of a GLM-5.3 checkpoint as a MoELayer (EXL3 routed experts as stored,
    bf16 shared expert).  Returns (layer, info) with info = {H, I, E, bits}."""
    from .moe import MoELayer
    pre = f"{prefix}{layer}.mlp."
    gate_w = ck.read(pre + "gate.weight")
    E, H = gate_w.shape
    router_w = gate_w.float().contiguous()
    bias = ck.read(pre + "gate.e_score_correction_bias").float().contiguous()
    t0 = ck.info(pre + "experts.0.gate_proj.trellis")
    if t0["dtype"] != "I16" or len(t0["shape"]) != 3:
        raise ValueError(f"{pre}experts.0.gate_proj.trellis: expected int16 [in/16, out/16, words]")
    I, words = t0["shape"][1] * 16, t0["shape"][2]
    bits = words // 16
    if bits not in (3, 4):
        raise ValueError(f"EXL3 with {words} words per tile ({bits} bits) is not supported")
    dev = {}
    for p in PROJS:
        K, N = (H, I) if p != "down_proj" else (I, H)
        tr = torch.empty((E, K // 16, N // 16, words), dtype=torch.int16, device="cuda")
        suh = torch.empty((E, K), dtype=torch.float16, device="cuda")
        svh = torch.empty((E, N), dtype=torch.float16, device="cuda")
        for e in range(E):
            q = f"{pre}experts.{e}.{p}."
            if not ck.has(q + "mcg"):
                raise ValueError(f"{q}mcg missing: only the mcg codebook is supported")
            ck.read_into(q + "trellis", tr[e])
            ck.read_into(q + "suh", suh[e])
            ck.read_into(q + "svh", svh[e])
        dev[p] = (tr, suh, svh)
    shared = tuple(ck.read(f"{pre}shared_experts.{p}.weight").contiguous() for p in PROJS)
    lay = MoELayer(hidden=H, inter=I, n_experts=E, topk=topk, router_w=router_w, router_bias=bias,
                   gate=dev["gate_proj"], up=dev["up_proj"], down=dev["down_proj"], shared=shared, fmt="exl3",
                   exl3_bits=bits, x_dtype=x_dtype, out_dtype=out_dtype, scale=scale, limit=limit,
                   shared_format="bf16")
    return lay, {"H": H, "I": I, "E": E, "bits": bits}
