"""Numpy restatement of the library's expert-parallel exchange protocol (test infrastructure).

The reference has no multi-GPU code, so there is no reference counterpart: this restates what
include/vfmoe.h specifies for vfmoe_ep_* (fixed-capacity blocks, token-level entries, lane
slots and weights, partial rows, combine in rank order) so that

* tests/test_ep_cpu.py can run the whole protocol on gloo ranks (CPU) against the single-device
  oracle, and
* tests/test_gpu_ep.py can compare the library's plan and pack outputs with it bit for bit.
"""

from __future__ import annotations

import numpy as np


def local_slots(owner):
    owner = np.asarray(owner)
    slot = np.empty_like(owner)
    for r in np.unique(owner):
        ids = np.nonzero(owner == r)[0]
        slot[ids] = np.arange(len(ids))
    return slot.astype(np.int32)


def virtual_ids(idx, n_experts, replica_of):
    """Lane (t, l) of expert replica_of[j] goes to virtual expert n_experts + j when t + l is odd."""
    idx = np.asarray(idx)
    v = idx.copy()
    if len(replica_of):
        copy_of = np.full(n_experts, -1, dtype=np.int64)
        copy_of[np.asarray(replica_of)] = n_experts + np.arange(len(replica_of))
        T, k = idx.shape
        odd = ((np.arange(T)[:, None] + np.arange(k)[None, :]) % 2) == 1
        c = copy_of[idx]
        v = np.where((c >= 0) & odd, c, idx)
    return v


def plan(idx, w, owner, replica_of, n_experts, world, cap):
    """Send blocks of one rank: counts [world], tok [world, cap] (-1 padding), slot [world, cap, k]
    (-1 = no lane), wt [world, cap, k], pos_of [T, world] (d * cap + i or -1)."""
    idx = np.asarray(idx)
    T, k = idx.shape
    v = virtual_ids(idx, n_experts, replica_of)
    own = np.asarray(owner)[v]
    ls = local_slots(owner)[v]
    counts = np.zeros(world, dtype=np.int32)
    tok = np.full((world, cap), -1, dtype=np.int32)
    slot = np.full((world, cap, k), -1, dtype=np.int32)
    wt = np.zeros((world, cap, k), dtype=np.float32)
    pos = np.full((T, world), -1, dtype=np.int32)
    for d in range(world):
        for t in range(T):
            mine = own[t] == d
            if mine.any():
                i = counts[d]
                tok[d, i] = t
                slot[d, i] = np.where(mine, ls[t], -1)
                wt[d, i] = np.where(mine, w[t], 0.0)
                pos[t, d] = d * cap + i
                counts[d] += 1
    return counts, tok, slot, wt, pos


def expert_partials(rows, slot, wt, ffn_of_slot):
    """Partial row per received entry: sum over lanes with slot >= 0 of wt * FFN_slot(row), lanes in
    order (f64).  rows [n, H], slot/wt [n, k]; ffn_of_slot(s, rows) -> [m, H]."""
    y = np.zeros(rows.shape, dtype=np.float64)
    for l in range(slot.shape[1]):
        for s in np.unique(slot[:, l]):
            if s < 0:
                continue
            sel = slot[:, l] == s
            y[sel] += wt[sel, l:l + 1].astype(np.float64) * ffn_of_slot(int(s), rows[sel])
    return y


def combine(y_back, pos, y_shared):
    """out[t] = sum over d (rank order) of y_back[pos[t, d]] + y_shared[t]."""
    out = np.array(y_shared, dtype=np.float64, copy=True)
    for t in range(pos.shape[0]):
        for d in range(pos.shape[1]):
            if pos[t, d] >= 0:
                out[t] += y_back[pos[t, d]]
    return out
