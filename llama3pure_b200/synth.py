"""Seeded synthetic attention inputs and the benchmark configurations.

The reference publishes no benchmark data set; its attention consumes
post-RoPE q/K/V produced by the model.  Every test and benchmark here uses
i.i.d. N(0, 1) fp32 draws from one documented generator so that the CUDA
path, the C oracle and the timed CPU baseline see byte-identical inputs:

    rng = numpy.random.Generator(PCG64(SeedSequence([seed, layer])))

Decode draw order per layer: K cache ``[n_kv][ctx][hd]``, V cache (same
shape), then q ``[n_heads][hd]``.  Prefill draw order per layer (token-major,
the layout the engines hand to attention, llama3pure-c-engine.c:3491-3493):
K ``[S][n_kv][hd]``, V ``[S][n_kv][hd]``, q ``[S][n_heads][hd]``.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field, replace

import numpy as np


@dataclass(frozen=True)
class AttnShape:
    """Geometry of one attention configuration (Config fields c:211-229)."""

    name: str
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    seq_len: int  # KV capacity in positions
    pos: int = 0  # decode position (query index); prefill: tokens = pos + 1
    seed: int = 0
    k_scale: float = 1.0  # multiplier applied to K rows after drawing
    is_gemma3: int = 0
    swa_window: int = 0
    swa_pattern: int = 0
    prefill: bool = False
    extra: dict = field(default_factory=dict, compare=False)

    @property
    def kv_mul(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def scale(self) -> float:
        # attn_scale = 1.0f / sqrtf((float)head_size), c:434 (float32 maths)
        return float(np.float32(1.0) / np.sqrt(np.float32(self.head_dim)))

    def start_t(self, layer: int, pos: int) -> int:
        """First attended position (SWA rule, c:3316-3321)."""
        swa_layer = self.swa_pattern > 0 and (layer % self.swa_pattern) < self.swa_pattern - 1
        if self.is_gemma3 and swa_layer and self.swa_window > 0:
            return max(0, pos - self.swa_window + 1)
        return 0

    def with_(self, **kw) -> "AttnShape":
        return replace(self, **kw)


# The five BASELINE.json configurations.
CONFIGS = {
    "llama32_1b_decode": AttnShape("llama32_1b_decode", 16, 32, 8, 64, 1024, pos=1023, seed=0),
    "llama31_8b_decode_8k": AttnShape("llama31_8b_decode_8k", 32, 32, 8, 128, 8192, pos=8191, seed=1),
    "llama31_8b_decode_128k": AttnShape(
        "llama31_8b_decode_128k", 32, 32, 8, 128, 131072, pos=131071, seed=2, k_scale=0.5
    ),
    "gemma_2b_decode": AttnShape("gemma_2b_decode", 18, 8, 1, 256, 4096, pos=4095, seed=3, is_gemma3=1),
    "llama31_8b_prefill_2k": AttnShape(
        "llama31_8b_prefill_2k", 32, 32, 8, 128, 2048, pos=2047, seed=4, prefill=True
    ),
}

# Windowed Gemma variant exercising the SWA start rule (window 512, pattern 6).
GEMMA_SWA = CONFIGS["gemma_2b_decode"].with_(name="gemma_2b_decode_swa512", swa_window=512, swa_pattern=6)


def rng_for(seed: int, layer: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, layer])))


def decode_inputs(shape: AttnShape, layer: int, ctx: int | None = None):
    """K, V ``[n_kv][ctx][hd]`` and q ``[n_heads][hd]`` for one decode layer."""
    ctx = shape.pos + 1 if ctx is None else ctx
    g = rng_for(shape.seed, layer)
    k = g.standard_normal((shape.n_kv_heads, ctx, shape.head_dim), dtype=np.float32)
    v = g.standard_normal((shape.n_kv_heads, ctx, shape.head_dim), dtype=np.float32)
    q = g.standard_normal((shape.n_heads, shape.head_dim), dtype=np.float32)
    if shape.k_scale != 1.0:
        k *= np.float32(shape.k_scale)
    return k, v, q


def prefill_inputs(shape: AttnShape, layer: int, n_tok: int | None = None):
    """Token-major K, V ``[S][n_kv][hd]`` and q ``[S][n_heads][hd]``."""
    s = shape.pos + 1 if n_tok is None else n_tok
    g = rng_for(shape.seed, layer)
    k = g.standard_normal((s, shape.n_kv_heads, shape.head_dim), dtype=np.float32)
    v = g.standard_normal((s, shape.n_kv_heads, shape.head_dim), dtype=np.float32)
    q = g.standard_normal((s, shape.n_heads, shape.head_dim), dtype=np.float32)
    if shape.k_scale != 1.0:
        k *= np.float32(shape.k_scale)
    return k, v, q


def raw_qkv_inputs(shape: AttnShape, layer: int, n_tok: int):
    """Projection outputs before QK-norm and RoPE, token-major: q
    ``[n_tok][n_heads*hd]``, k, v ``[n_tok][n_kv*hd]``, and QK-norm weights
    ``[n_layers][hd]`` for q and k drawn as 1 + 0.1*N(0, 1) (Gemma3 GGUF norm
    weights already carry the +1, c:3148).  Generator: rng_for(seed + 1000,
    layer); draw order k, v, q, q_norm, k_norm."""
    g = rng_for(shape.seed + 1000, layer)
    kvd, qd = shape.n_kv_heads * shape.head_dim, shape.n_heads * shape.head_dim
    k = g.standard_normal((n_tok, kvd), dtype=np.float32)
    v = g.standard_normal((n_tok, kvd), dtype=np.float32)
    q = g.standard_normal((n_tok, qd), dtype=np.float32)
    q_norm = (np.float32(1.0) + np.float32(0.1) * g.standard_normal((shape.n_layers, shape.head_dim),
                                                                     dtype=np.float32)).astype(np.float32)
    k_norm = (np.float32(1.0) + np.float32(0.1) * g.standard_normal((shape.n_layers, shape.head_dim),
                                                                     dtype=np.float32)).astype(np.float32)
    return q, k, v, q_norm, k_norm


# GGUF type -> (values, bytes) per block: F32, F16, Q4_0, Q4_1, Q5_0, Q5_1,
# Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ4_NL, BF16
W_BLOCK = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84),
           11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 20: (32, 18), 29: (1, 2)}


def wo_weights(wtype: int, rows: int, cols: int, seed: int, scale: float = 0.02) -> np.ndarray:
    """Random GGUF weight rows (uint8 [rows][cols/values*bytes]) of a Q8_0,
    Q2_K, Q3_K, Q4_K, Q5_K or Q6_K tensor whose values are ~N(0, scale): every
    quant byte drawn uniformly, every fp16 scale set so that the block spans
    about +-3 scale.
    Generator: rng_for(seed + 2000, wtype)."""
    n, nb = W_BLOCK[wtype]
    g = rng_for(seed + 2000, wtype)
    blocks = g.integers(0, 256, size=(rows, cols // n, nb), dtype=np.uint8)

    def f16(a):
        return np.ascontiguousarray(np.asarray(a, np.float16)).view(np.uint8).reshape(a.shape + (2,))

    shp = (rows, cols // n)
    if wtype in (0, 1, 29):
        # float rows: the values themselves, ~N(0, scale)
        v = g.standard_normal((rows, cols)).astype(np.float32) * np.float32(scale)
        if wtype == 0:
            return np.ascontiguousarray(v.view(np.uint8).reshape(rows, -1))
        if wtype == 1:
            return np.ascontiguousarray(v.astype(np.float16).view(np.uint8).reshape(rows, -1))
        return np.ascontiguousarray((v.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).reshape(rows, -1))
    if wtype in (2, 3, 6, 7, 20):
        # 32-value blocks: d (and m) first; q 4-bit (5 with qh), IQ4_NL table values up to 127
        qmax = {2: 8.0, 3: 15.0, 6: 16.0, 7: 31.0, 20: 127.0}[wtype]
        blocks[..., 0:2] = f16(g.uniform(0.5, 1.5, shp) * scale * 3.0 / qmax)
        if wtype in (3, 7):
            blocks[..., 2:4] = f16(-g.uniform(0.5, 1.5, shp) * scale * 3.0 / 2.0)
        return np.ascontiguousarray(blocks.reshape(rows, -1))
    if wtype == 8:
        blocks[..., 0:2] = f16(g.uniform(2.0, 4.0, shp) * scale / 127.0)
    elif wtype == 12:
        # value = d*sc*q - dmin*m, q in 0..15, sc and m 6-bit
        blocks[..., 0:2] = f16(g.uniform(0.5, 1.5, shp) * scale / 63.0 * 0.75)
        blocks[..., 2:4] = f16(g.uniform(0.5, 1.5, shp) * scale / 63.0 * 0.75 * 7.5)
    elif wtype == 13:
        # Q5_K: value = d*sc*q - dmin*m, q in 0..31, sc and m 6-bit
        blocks[..., 0:2] = f16(g.uniform(0.5, 1.5, shp) * scale / 63.0 * 0.375)
        blocks[..., 2:4] = f16(g.uniform(0.5, 1.5, shp) * scale / 63.0 * 0.375 * 15.5)
    elif wtype == 10:
        # Q2_K: value = d*sc*q - dmin*m, q in 0..3, sc and m 4-bit
        blocks[..., 80:82] = f16(g.uniform(0.5, 1.5, shp) * scale / 15.0 * 2.0)
        blocks[..., 82:84] = f16(g.uniform(0.5, 1.5, shp) * scale / 15.0 * 3.0)
    elif wtype == 11:
        # Q3_K: value = d*(sc-32)*q, q in -4..3, sc 6-bit
        blocks[..., 108:110] = f16(g.uniform(0.5, 1.5, shp) * scale * 3.0 / (32.0 * 4.0))
    else:
        # value = d*sc*(q-32), q 6-bit, sc int8
        blocks[..., 208:210] = f16(g.uniform(0.5, 1.5, shp) * scale * 3.0 / (32.0 * 127.0))
    return np.ascontiguousarray(blocks.reshape(rows, -1))


def wo_input(cols: int, seed: int) -> np.ndarray:
    """An attention output fed to wo: 0.3*N(0, 1) float32 [cols], generator
    PCG64(SeedSequence([seed, 3000]))."""
    g = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, 3000])))
    return (np.float32(0.3) * g.standard_normal(cols, dtype=np.float32)).astype(np.float32)


def sha256_arrays(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def decode_kv_bytes(shape: AttnShape, layer: int = 0) -> int:
    """Algorithmic fp32 bytes one decode layer must read: K and V rows of the
    attended window (2 * P * n_kv * hd * 4)."""
    p = shape.pos - shape.start_t(layer, shape.pos) + 1
    return 2 * p * shape.n_kv_heads * shape.head_dim * 4


def prefill_flops(shape: AttnShape, n_tok: int | None = None) -> int:
    """Algorithmic causal-attention FLOPs of one prefill layer:
    4 * Hq * hd * S(S+1)/2 (q.K^T and P.V, 2 flops per MAC, mask j <= i)."""
    s = shape.pos + 1 if n_tok is None else n_tok
    return 4 * shape.n_heads * shape.head_dim * s * (s + 1) // 2


def tolerance_ok(got: np.ndarray, want: np.ndarray, atol: float = 1e-4, rtol: float = 1e-4):
    """Element-wise |got - want| <= atol + rtol*|want|; returns (ok, max_abs, max_rel)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    diff = np.abs(got - want)
    max_abs = float(diff.max()) if diff.size else 0.0
    denom = np.maximum(np.abs(want), 1e-30)
    max_rel = float((diff / denom).max()) if diff.size else 0.0
    ok = bool(np.all(diff <= atol + rtol * np.abs(want))) and bool(np.all(np.isfinite(got)))
    return ok, max_abs, max_rel


__all__ = [
    "AttnShape",
    "CONFIGS",
    "GEMMA_SWA",
    "rng_for",
    "decode_inputs",
    "prefill_inputs",
    "raw_qkv_inputs",
    "wo_input",
    "wo_weights",
    "sha256_arrays",
    "decode_kv_bytes",
    "prefill_flops",
    "tolerance_ok",
]
