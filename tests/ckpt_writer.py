"""Writes safetensors checkpoints for the loader tests (test infrastructure).

The format (native/torchload/safetensors.vyb): u64 little-endian header length, a JSON header
{name: {"dtype", "shape", "data_offsets": [begin, end]}} with offsets relative to the data region
that follows it, then the raw tensor bytes.  A sharded checkpoint adds model.safetensors.index.json
with {"weight_map": {name: shard file}}.
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np


def write_safetensors(path, tensors):
    """tensors: {name: (dtype string, ndarray)} (BF16 given as uint16 bit patterns)."""
    header, blobs, off = {}, [], 0
    for name, (dt, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_sharded(dirpath, tensors, n_shards=2):
    """Split tensors over n_shards files model-0000i-of-0000n.safetensors plus the index."""
    os.makedirs(dirpath, exist_ok=True)
    names = list(tensors)
    weight_map = {}
    for s in range(n_shards):
        fname = f"model-{s + 1:05d}-of-{n_shards:05d}.safetensors"
        part = {n: tensors[n] for n in names[s::n_shards]}
        write_safetensors(os.path.join(dirpath, fname), part)
        weight_map.update({n: fname for n in part})
    with open(os.path.join(dirpath, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": 0}, "weight_map": weight_map}, f)


def glm_moe_tensors(rng, layer, H, I, E, bits=4):
    """One GLM-5.3-style MoE layer: bf16 router, f32 bias, EXL3 experts (trellis/suh/svh/mcg), bf16
    shared expert.  Returns {name: (dtype, array)}."""
    from vybforge_b200.quant import f32_to_bf16_bits
    pre = f"model.language_model.layers.{layer}.mlp."
    t = {pre + "gate.weight": ("BF16", f32_to_bf16_bits(rng.normal(0, 0.02, (E, H)).astype(np.float32))),
         pre + "gate.e_score_correction_bias": ("F32", rng.normal(0, 0.01, E).astype(np.float32))}
    for e in range(E):
        for p in ("gate_proj", "up_proj", "down_proj"):
            K, N = (H, I) if p != "down_proj" else (I, H)
            q = f"{pre}experts.{e}.{p}."
            t[q + "trellis"] = ("I16", rng.integers(-32768, 32768, (K // 16, N // 16, 16 * bits), dtype=np.int16))
            t[q + "suh"] = ("F16", np.where(rng.random(K) < 0.5, -1.0, 1.0).astype(np.float16))
            t[q + "svh"] = ("F16", (np.where(rng.random(N) < 0.5, -1.0, 1.0) * rng.uniform(0.01, 0.03, N)).astype(np.float16))
            t[q + "mcg"] = ("I32", np.array([1], dtype=np.int32))
    for p in ("gate_proj", "up_proj", "down_proj"):
        rows, cols = (I, H) if p != "down_proj" else (H, I)
        t[f"{pre}shared_experts.{p}.weight"] = ("BF16", f32_to_bf16_bits(rng.normal(0, 0.02, (rows, cols)).astype(np.float32)))
    return t
