"""Generate tests/golden/attn_golden.npz from the REFERENCE's own code.

Run in a container that has the reference source (it needs oracle/_ref/,
built by `make -C oracle ref` from llama3pure-c-engine.c in place):

    python tests/golden/make_golden.py          # all three files
    python tests/golden/make_golden.py rope     # rope_golden.npz only
    python tests/golden/make_golden.py wo       # wo_golden.npz only

Each case records its geometry, the SHA-256 of its seeded inputs (so generator
drift is caught) and the reference's attention output in both oracle modes:
"f32" (the reference loop with an fp32 KV cache, the 1e-4 contract) and "q8"
(the reference as shipped, Q8_0 cache).  Large outputs are stored as a row
subsample plus float64 row sums.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
from llama3pure_b200.synth import (  # noqa: E402
    CONFIGS,
    GEMMA_SWA,
    AttnShape,
    decode_inputs,
    prefill_inputs,
    raw_qkv_inputs,
    sha256_arrays,
    wo_input,
    wo_weights,
)

PREFILL_ROWS = (0, 1, 2, 31, 32, 33, 1023, 2047)


def decode_cases():
    c = CONFIGS
    small = AttnShape("mha_hd32", 1, 4, 4, 32, 128, pos=100, seed=11)
    return [
        ("l1b_layer0", c["llama32_1b_decode"], 0, False),
        ("l1b_layer5", c["llama32_1b_decode"], 5, False),
        ("l8b_8k_layer0_append", c["llama31_8b_decode_8k"], 0, True),
        ("l8b_128k_layer0", c["llama31_8b_decode_128k"], 0, False),
        ("gemma_layer0", c["gemma_2b_decode"], 0, False),
        ("gemma_swa_layer0", GEMMA_SWA, 0, False),
        ("gemma_swa_layer5", GEMMA_SWA, 5, False),
        ("pos0", c["llama32_1b_decode"].with_(pos=0), 0, False),
        ("gemma_window1", GEMMA_SWA.with_(swa_window=1), 0, False),
        ("mha_hd32", small, 0, False),
        ("gqa2_hd256_odd", AttnShape("gqa2", 1, 4, 2, 256, 700, pos=612, seed=12), 0, True),
    ]


def prefill_cases():
    return [
        ("prefill_gqa_s48", AttnShape("pf_gqa", 1, 8, 2, 128, 48, pos=47, seed=4, prefill=True), 0),
        ("prefill_mqa_swa_s80", AttnShape("pf_swa", 1, 8, 1, 256, 80, pos=79, seed=5, prefill=True,
                                          is_gemma3=1, swa_window=16, swa_pattern=6), 0),
        ("prefill_8b_2k_layer0", CONFIGS["llama31_8b_prefill_2k"], 0),
    ]


def rope_cases():
    """(name, shape, layer, pos0, n_tok, rope_theta, rope_theta_swa, rms_norm_eps, qk_norm)"""
    c = CONFIGS
    return [
        ("l8b_pos8190", c["llama31_8b_decode_8k"], 0, 8190, 2, 0.0, 0.0, 0.0, False),
        ("l1b_pos0_l3", c["llama32_1b_decode"], 3, 0, 5, 500000.0, 0.0, 0.0, False),
        ("l8b_pos131071", c["llama31_8b_decode_128k"], 0, 131071, 1, 0.0, 0.0, 0.0, False),
        ("gemma_swa_l0_norm", GEMMA_SWA, 0, 4094, 2, 1000000.0, 10000.0, 1e-6, True),
        ("gemma_swa_l5_norm", GEMMA_SWA, 5, 4094, 2, 1000000.0, 10000.0, 1e-6, True),
        ("gemma_l2_plain", c["gemma_2b_decode"], 2, 77, 3, 0.0, 0.0, 0.0, False),
        ("gqa_hd64_theta1e4", AttnShape("gqa64", 2, 8, 2, 64, 512, pos=0, seed=21), 1, 100, 3,
         10000.0, 0.0, 0.0, False),
    ]


def write_rope_golden():
    """tests/golden/rope_golden.npz: the pre-attention step (QK-norm, RoPE) of
    raw_qkv_inputs through the reference's own tables and rmsnorm_per_head."""
    data = {}
    names = []
    for name, shape, layer, pos0, n_tok, th, th_swa, eps, norm in rope_cases():
        q, k, v, qn, kn = raw_qkv_inputs(shape, layer, n_tok)
        qr, kr = O.rope(shape, layer, pos0, q, k, th, th_swa, eps, qn if norm else None, kn if norm else None,
                        impl="ref", n_layers=shape.n_layers)
        data[f"{name}/q"] = qr
        data[f"{name}/k"] = kr
        data[f"{name}/sha256"] = np.array(sha256_arrays(q, k, v, qn, kn))
        data[f"{name}/geom"] = np.array([shape.n_layers, shape.n_heads, shape.n_kv_heads, shape.head_dim,
                                         shape.seq_len, shape.seed, layer, pos0, n_tok, shape.is_gemma3,
                                         shape.swa_window, shape.swa_pattern, int(norm)], np.int64)
        data[f"{name}/theta"] = np.array([th, th_swa, eps], np.float32)
        names.append(name)
        print("rope", name, "done", flush=True)
    data["cases"] = np.array(names)
    out_path = os.path.join(HERE, "rope_golden.npz")
    np.savez_compressed(out_path, **data)
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


def wo_cases():
    """(name, weight type, rows, cols, seed)"""
    return [
        ("q8_0_64x4096", O.W_Q8_0, 64, 4096, 1),
        ("q8_0_37x2048", O.W_Q8_0, 37, 2048, 2),
        ("q4_k_48x4096", O.W_Q4_K, 48, 4096, 3),
        ("q4_k_9x2048", O.W_Q4_K, 9, 2048, 4),
        ("q6_k_40x4096", O.W_Q6_K, 40, 4096, 5),
        ("q6_k_7x2048", O.W_Q6_K, 7, 2048, 6),
        ("q2_k_33x4096", O.W_Q2_K, 33, 4096, 7),
        ("q3_k_35x4096", O.W_Q3_K, 35, 4096, 8),
        ("q5_k_31x4096", O.W_Q5_K, 31, 4096, 9),
        ("q5_k_5x2048", O.W_Q5_K, 5, 2048, 10),
        ("q4_0_29x4096", O.W_Q4_0, 29, 4096, 11),
        ("q4_1_27x4096", O.W_Q4_1, 27, 4096, 12),
        ("q5_0_25x4096", O.W_Q5_0, 25, 4096, 13),
        ("q5_1_23x4096", O.W_Q5_1, 23, 4096, 14),
        ("iq4_nl_21x4096", O.W_IQ4_NL, 21, 4096, 15),
        ("q4_0_6x2048", O.W_Q4_0, 6, 2048, 16),
        ("f32_19x4096", O.W_F32, 19, 4096, 17),
        ("f16_17x4096", O.W_F16, 17, 4096, 18),
        ("bf16_15x4096", O.W_BF16, 15, 4096, 19),
    ]


def write_wo_golden():
    """tests/golden/wo_golden.npz: the wo projection through the reference's
    own matmul_quantized for every GGUF weight type it reads: dequantised rows
    and fp32 dots for Q8_0 and the K-quants (c:2063-2073), x quantised to Q8_0
    and integer block dots for Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL, fp32 dots for
    F32, F16, BF16 (c:2091-2132)."""
    data = {}
    names = []
    for name, wt, rows, cols, seed in wo_cases():
        w = wo_weights(wt, rows, cols, seed)
        x = wo_input(cols, seed)
        data[f"{name}/out"] = O.matvec(wt, w, rows, cols, x, impl="ref")
        data[f"{name}/sha256"] = np.array(sha256_arrays(w, x))
        data[f"{name}/geom"] = np.array([wt, rows, cols, seed], np.int64)
        names.append(name)
        print("wo", name, "done", flush=True)
    data["cases"] = np.array(names)
    out_path = os.path.join(HERE, "wo_golden.npz")
    np.savez_compressed(out_path, **data)
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


def run_decode(shape: AttnShape, layer: int, append: bool, mode: int):
    k, v, q = decode_inputs(shape, layer)
    o = O.Oracle(shape, mode, "ref", n_layers=layer + 1)
    if append:
        o.load_kv(layer, 0, k[:, : shape.pos], v[:, : shape.pos])
        out, sk = o.decode(layer, shape.pos, q, k[:, shape.pos].copy(), v[:, shape.pos].copy())
    else:
        o.load_kv(layer, 0, k, v)
        out, sk = o.decode(layer, shape.pos, q)
    o.close()
    return out, sk, sha256_arrays(k, v, q)


def run_prefill(shape: AttnShape, layer: int, mode: int):
    k, v, q = prefill_inputs(shape, layer)
    o = O.Oracle(shape, mode, "ref", n_layers=layer + 1)
    out, sk = o.prefill(layer, 0, q, k, v)
    o.close()
    return out, sk, sha256_arrays(k, v, q)


def main():
    if not O.ref_available():
        sys.exit("oracle/_ref/libl3p_ref.so missing: run `make -C oracle ref` where the reference source exists")
    data = {}
    names = []
    for name, shape, layer, append in decode_cases():
        for mode, tag in ((O.MODE_F32, "f32"), (O.MODE_Q8, "q8")):
            out, sk, sha = run_decode(shape, layer, append, mode)
            data[f"{name}/{tag}"] = out
            data[f"{name}/{tag}_skipped"] = np.int64(sk)
        data[f"{name}/sha256"] = np.array(sha)
        data[f"{name}/geom"] = np.array([shape.n_heads, shape.n_kv_heads, shape.head_dim, shape.seq_len,
                                         shape.pos, shape.seed, layer, int(append), shape.is_gemma3,
                                         shape.swa_window, shape.swa_pattern], np.int64)
        data[f"{name}/k_scale"] = np.float64(shape.k_scale)
        names.append(name)
        print("decode", name, "done", flush=True)
    for name, shape, layer in prefill_cases():
        for mode, tag in ((O.MODE_F32, "f32"), (O.MODE_Q8, "q8")):
            out, sk, sha = run_prefill(shape, layer, mode)
            s = out.shape[0]
            rows = np.array([r for r in PREFILL_ROWS if r < s] if s > 32 else list(range(s)), np.int64)
            data[f"{name}/{tag}_rows"] = rows
            data[f"{name}/{tag}"] = out[rows]
            data[f"{name}/{tag}_rowsum"] = out.astype(np.float64).sum(axis=(1, 2))
            data[f"{name}/{tag}_skipped"] = np.int64(sk)
        data[f"{name}/sha256"] = np.array(sha)
        data[f"{name}/geom"] = np.array([shape.n_heads, shape.n_kv_heads, shape.head_dim, shape.seq_len,
                                         shape.pos, shape.seed, layer, 0, shape.is_gemma3,
                                         shape.swa_window, shape.swa_pattern], np.int64)
        data[f"{name}/k_scale"] = np.float64(shape.k_scale)
        names.append(name)
        print("prefill", name, "done", flush=True)

    # codec known-answer vectors from the reference's own primitives
    prim = O.primitives("ref")
    table = np.array([prim["fp16_to_fp32"](h) for h in range(65536)], np.float32)
    data["kat/fp16_to_fp32_sha256"] = np.array(sha256_arrays(table))
    data["kat/fp16_to_fp32_sample"] = table[::257]
    rng = np.random.default_rng(7)
    xs = (rng.standard_normal(4096).astype(np.float32)
          * (np.float32(10.0) ** rng.integers(-9, 6, 4096).astype(np.float32))).astype(np.float32)
    data["kat/fp32_in"] = xs
    data["kat/fp32_to_fp16"] = np.array([prim["fp32_to_fp16"](float(x)) for x in xs], np.uint16)
    blk_in = rng.standard_normal(256).astype(np.float32) * np.float32(3.0)
    blk_in[32:64] = 0.0  # an all-zero block (d = 0 path, c:1550)
    qbuf = np.zeros(256 // 32 * 34, np.uint8)
    prim["q8_quantize"](O._fptr(blk_in), qbuf.ctypes.data, 256)
    data["kat/q8_in"] = blk_in
    data["kat/q8_blocks"] = qbuf
    data["cases"] = np.array(names)
    out_path = os.path.join(HERE, "attn_golden.npz")
    np.savez_compressed(out_path, **data)
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


if __name__ == "__main__":
    if not O.ref_available():
        sys.exit("oracle/_ref/libl3p_ref.so missing: run `make -C oracle ref` where the reference source exists")
    if sys.argv[1:] == ["rope"]:
        write_rope_golden()
    elif sys.argv[1:] == ["wo"]:
        write_wo_golden()
    else:
        main()
        write_rope_golden()
        write_wo_golden()
