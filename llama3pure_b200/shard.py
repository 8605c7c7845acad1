"""Multi-GPU placement of the attention step: one process per GPU.

Attention is independent per KV-head group, so ranks first split the KV heads
(each rank owns n_kv/H consecutive KV heads and their kv_mul q heads).  When
there are more ranks than head groups (Gemma MQA has one KV head) or the
context is long, each head group is further split along the sequence axis;
the ranks sharing a head group then produce partial (m, l, o) triples that are
all-gathered over NCCL and combined by the LSE merge kernel.

The reference has no multi-device path (OpenMP over KV heads only,
llama3pure-c-engine.c:3327-3328); this module is new.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Shard:
    rank: int
    head_group: int      # index of the KV-head group
    seq_part: int        # index along the sequence axis
    kv_head_begin: int
    kv_head_count: int
    seq_begin: int
    seq_count: int


def plan_shards(n_kv_heads: int, seq_len: int, world: int, seq_parts: int | None = None) -> list[Shard]:
    """Split `world` ranks into head_groups x seq_parts.  By default the head
    axis takes as many ranks as it can (up to n_kv_heads, power-of-two
    friendly) and the sequence axis the rest."""
    if world <= 0:
        raise ValueError("world must be positive")
    if seq_parts is None:
        head_groups = np.gcd(world, n_kv_heads)
        seq_parts = world // head_groups
    if world % seq_parts != 0:
        raise ValueError(f"world {world} not divisible by seq_parts {seq_parts}")
    head_groups = world // seq_parts
    if n_kv_heads % head_groups != 0:
        raise ValueError(f"{n_kv_heads} KV heads do not split into {head_groups} groups")
    per_group = n_kv_heads // head_groups
    shards = []
    for r in range(world):
        g, s = divmod(r, seq_parts)
        b = seq_len * s // seq_parts
        e = seq_len * (s + 1) // seq_parts
        shards.append(Shard(r, g, s, g * per_group, per_group, b, e - b))
    return shards


def lse_merge_np(parts_o: np.ndarray, parts_ml: np.ndarray) -> np.ndarray:
    """numpy statement of the LSE merge: parts_o [P][rows][hd] normalised
    partial outputs, parts_ml [P][rows][2] with m in log2 units.  Used by the
    CPU tests of the sharded path."""
    m = parts_ml[..., 0].astype(np.float64)
    lsum = parts_ml[..., 1].astype(np.float64)
    mmax = np.max(m, axis=0)
    w = np.where(np.isneginf(m), 0.0, lsum * np.exp2(m - np.where(np.isneginf(mmax), 0.0, mmax)))
    tot = w.sum(axis=0)
    out = (parts_o.astype(np.float64) * w[..., None]).sum(axis=0) / np.where(tot > 0, tot, 1.0)[..., None]
    return out.astype(np.float32)


def partial_attention_np(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, lo: int, hi: int, kv_mul: int):
    """float64 partial attention of q [Hq][hd] over positions [lo, hi) of
    k, v [Hkv][ctx][hd], returned as the (o, (m, l)) triple of the C ABI."""
    hq, hd = q.shape
    o = np.zeros((hq, hd), np.float32)
    ml = np.zeros((hq, 2), np.float32)
    ml[:, 0] = -np.inf
    if hi <= lo:
        return o, ml
    for h in range(hq):
        kv = h // kv_mul
        s = (k[kv, lo:hi].astype(np.float64) @ (q[h].astype(np.float32) * np.float32(scale)).astype(np.float64))
        s2 = s * np.log2(np.e)
        m = s2.max()
        p = np.exp2(s2 - m)
        o[h] = (p @ v[kv, lo:hi].astype(np.float64)) / p.sum()
        ml[h] = (m, p.sum())
    return o, ml
