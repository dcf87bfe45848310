"""Host-side weight packing for the MoE layer (numpy; no GPU needed).

* Q8_0 (GGUF ``block_q8_0``): 34-byte blocks, fp16 scale ``d`` then 32 int8
  quants; a matrix is stored as output rows, each row K/32 consecutive blocks
  (native/kernels/q8_0.vyb:6 and native/kernels/rgemv.vyb:12 of the reference).
  ``quantize_q8_0`` restates ggml's reference quantizer (``quantize_row_q8_0_ref``):
  d = amax/127 in float32, q = round-half-away-from-zero(x * (1/d)), d stored as
  fp16.  The reference never quantizes (it reads GGUF bytes), so the GPU path and
  the oracle simply consume the same bytes.
* EXL3 trellis tiles: ``uint16 [K/16][N/16][16*bits]`` (native/exl3/README.md:26-31).
* bf16 helpers: round-to-nearest-even float32 -> bf16 bits and back.
"""

from __future__ import annotations

import numpy as np

Q8_BLOCK = 32
Q8_BYTES = 34


def q8_0_row_bytes(k: int) -> int:
    if k % Q8_BLOCK:
        raise ValueError(f"Q8_0 needs K % 32 == 0, got {k}")
    return (k // Q8_BLOCK) * Q8_BYTES


def quantize_q8_0(w) -> np.ndarray:
    """float [rows, K] -> uint8 [rows, K/32*34] (ggml quantize_row_q8_0_ref)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, k = w.shape
    blocks = w.reshape(rows * (k // Q8_BLOCK), Q8_BLOCK)
    d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    v = blocks * inv
    a = np.abs(v)
    fl = np.floor(a)
    q = np.sign(v) * (fl + np.floor(np.float32(2) * (a - fl)))
    out = np.empty((blocks.shape[0], Q8_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = q.astype(np.int8).view(np.uint8)
    return out.reshape(rows, q8_0_row_bytes(k))


def f32_to_bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u                     # finite inputs: no uint32 wrap-around (max 0xFF807FFE)
    r >>= np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    """float -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def exl3_words(bits: int) -> int:
    if bits not in (3, 4):
        raise ValueError(f"EXL3 bits must be 3 or 4, got {bits}")
    return 16 * bits


def exl3_matrix_bytes(k: int, n: int, bits: int) -> int:
    """Trellis bytes of one [K, N] matrix."""
    if k % 128 or n % 128:
        raise ValueError("EXL3 needs K and N multiples of 128 (Hadamard blocks)")
    return (k // 16) * (n // 16) * exl3_words(bits) * 2
