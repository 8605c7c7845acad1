"""The CPU oracle against the reference's golden vectors (no GPU).

The golden file was produced by the reference's own functions compiled from
llama3pure-c-engine.c (tests/golden/make_golden.py); the plain-C restatement
must reproduce it bit for bit in both modes.
"""
import os

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.synth import AttnShape, decode_inputs, prefill_inputs, sha256_arrays


def _shape_from(g, name):
    hq, hkv, hd, cap, pos, seed, layer, append, gem, win, pat = [int(x) for x in g[f"{name}/geom"]]
    ks = float(g[f"{name}/k_scale"])
    return AttnShape(name, layer + 1, hq, hkv, hd, cap, pos=pos, seed=seed, k_scale=ks, is_gemma3=gem,
                     swa_window=win, swa_pattern=pat), layer, bool(append)


def _cases(kind):
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "attn_golden.npz"))
    names = [str(n) for n in g["cases"]]
    return [n for n in names if n.startswith("prefill") == (kind == "prefill")]


def test_fp16_decode_table_matches_reference(golden):
    prim = O.primitives("port")
    table = np.array([prim["fp16_to_fp32"](h) for h in range(65536)], np.float32)
    assert sha256_arrays(table) == str(golden["kat/fp16_to_fp32_sha256"])
    np.testing.assert_array_equal(table[::257].view(np.uint32), golden["kat/fp16_to_fp32_sample"].view(np.uint32))


def test_fp16_truncating_encode_matches_reference(golden):
    prim = O.primitives("port")
    got = np.array([prim["fp32_to_fp16"](float(x)) for x in golden["kat/fp32_in"]], np.uint16)
    np.testing.assert_array_equal(got, golden["kat/fp32_to_fp16"])


def test_q8_block_encode_matches_reference(golden):
    prim = O.primitives("port")
    x = np.ascontiguousarray(golden["kat/q8_in"])
    buf = np.zeros(x.size // 32 * 34, np.uint8)
    prim["q8_quantize"](O._fptr(x), buf.ctypes.data, x.size)
    np.testing.assert_array_equal(buf, golden["kat/q8_blocks"])


@pytest.mark.parametrize("name", _cases("decode"))
def test_decode_matches_golden(golden, name):
    shape, layer, append = _shape_from(golden, name)
    k, v, q = decode_inputs(shape, layer)
    assert sha256_arrays(k, v, q) == str(golden[f"{name}/sha256"]), "seeded generator drifted"
    for mode, tag in ((O.MODE_F32, "f32"), (O.MODE_Q8, "q8")):
        o = O.Oracle(shape, mode, "port", n_layers=layer + 1)
        if append:
            o.load_kv(layer, 0, k[:, : shape.pos], v[:, : shape.pos])
            out, sk = o.decode(layer, shape.pos, q, k[:, shape.pos].copy(), v[:, shape.pos].copy())
        else:
            o.load_kv(layer, 0, k, v)
            out, sk = o.decode(layer, shape.pos, q)
        o.close()
        np.testing.assert_array_equal(out.view(np.uint32), golden[f"{name}/{tag}"].view(np.uint32))
        assert sk == int(golden[f"{name}/{tag}_skipped"])


@pytest.mark.parametrize("name", _cases("prefill"))
def test_prefill_matches_golden(golden, name):
    shape, layer, _ = _shape_from(golden, name)
    k, v, q = prefill_inputs(shape, layer)
    assert sha256_arrays(k, v, q) == str(golden[f"{name}/sha256"]), "seeded generator drifted"
    modes = ((O.MODE_F32, "f32"), (O.MODE_Q8, "q8")) if shape.pos < 1000 else ((O.MODE_F32, "f32"),)
    for mode, tag in modes:
        o = O.Oracle(shape, mode, "port", n_layers=layer + 1)
        out, sk = o.prefill(layer, 0, q, k, v)
        o.close()
        rows = golden[f"{name}/{tag}_rows"]
        np.testing.assert_array_equal(out[rows].view(np.uint32), golden[f"{name}/{tag}"].view(np.uint32))
        np.testing.assert_array_equal(out.astype(np.float64).sum(axis=(1, 2)), golden[f"{name}/{tag}_rowsum"])
        assert sk == int(golden[f"{name}/{tag}_skipped"])


def test_baseline_configs_skip_no_weights(golden):
    """The reference skips V rows with |weight| < 1e-8 (c:1602); a one-pass
    device softmax cannot.  On every seeded configuration no row is skipped,
    so the two agree exactly on which rows contribute."""
    for name in _cases("decode") + _cases("prefill"):
        for tag in ("f32", "q8"):
            key = f"{name}/{tag}_skipped"
            if key in golden.files:
                assert int(golden[key]) == 0, key


@pytest.mark.skipif(not O.ref_available(), reason="reference harness not built (no reference source here)")
@pytest.mark.parametrize("seed", range(6))
def test_port_bit_identical_to_reference_harness(seed):
    rng = np.random.default_rng(100 + seed)
    hkv = int(rng.choice([1, 2, 4]))
    g = int(rng.choice([1, 2, 4, 8]))
    hd = int(rng.choice([32, 64, 128]))
    cap = int(rng.integers(8, 300))
    shape = AttnShape("rand", 7, hkv * g, hkv, hd, cap, pos=int(rng.integers(0, cap)), seed=seed,
                      is_gemma3=int(rng.integers(0, 2)), swa_window=int(rng.integers(0, 40)), swa_pattern=6)
    layer = int(rng.integers(0, 7))
    k, v, q = decode_inputs(shape, layer)
    pk, pv, pq = prefill_inputs(shape.with_(pos=min(cap - 1, 20)), layer)
    for mode in (O.MODE_F32, O.MODE_Q8):
        outs = []
        for impl in ("port", "ref"):
            o = O.Oracle(shape, mode, impl)
            o.load_kv(layer, 0, k, v)
            d, _ = o.decode(layer, shape.pos, q)
            p, _ = o.prefill(layer, 0, pq, pk, pv)
            outs.append((d, p))
            o.close()
        np.testing.assert_array_equal(outs[0][0].view(np.uint32), outs[1][0].view(np.uint32))
        np.testing.assert_array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))


def _tiny(pos=5, **kw):
    return AttnShape("tiny", 1, 4, 2, 64, 16, pos=pos, seed=9, **kw)


def test_known_answer_pos0_is_v_row():
    sh = _tiny(pos=0)
    k, v, q = decode_inputs(sh, 0)
    o = O.Oracle(sh)
    o.load_kv(0, 0, k, v)
    out, _ = o.decode(0, 0, q)
    for h in range(sh.n_heads):
        np.testing.assert_array_equal(out[h], v[h // sh.kv_mul, 0])


def test_known_answer_window1_is_current_v_row():
    sh = _tiny(pos=9, is_gemma3=1, swa_window=1, swa_pattern=6)
    k, v, q = decode_inputs(sh, 0, ctx=sh.seq_len)
    o = O.Oracle(sh)
    o.load_kv(0, 0, k, v)
    out, _ = o.decode(0, sh.pos, q)
    for h in range(sh.n_heads):
        np.testing.assert_array_equal(out[h], v[h // sh.kv_mul, sh.pos])


def test_known_answer_equal_keys_average_values():
    sh = _tiny(pos=11)
    k, v, q = decode_inputs(sh, 0)
    k[:] = k[:, :1]
    o = O.Oracle(sh)
    o.load_kv(0, 0, k, v)
    out, _ = o.decode(0, sh.pos, q)
    for h in range(sh.n_heads):
        np.testing.assert_allclose(out[h], v[h // sh.kv_mul].mean(axis=0), rtol=1e-5, atol=1e-6)


def test_known_answer_dominant_score_selects_row():
    sh = _tiny(pos=11)
    k, v, q = decode_inputs(sh, 0)
    k[:, 7] = q[:: sh.kv_mul] * 50.0
    o = O.Oracle(sh)
    o.load_kv(0, 0, k, v)
    out, _ = o.decode(0, sh.pos, q)
    for kv in range(sh.n_kv_heads):
        np.testing.assert_allclose(out[kv * sh.kv_mul], v[kv, 7], rtol=1e-4, atol=1e-5)


# ---- pre-attention step: QK-norm and RoPE -----------------------------------

_ROPE_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "rope_golden.npz")


def rope_case(g, name):
    """(shape, layer, pos0, n_tok, theta, theta_swa, eps, norm) of a rope_golden.npz case."""
    nl, hq, hkv, hd, cap, seed, layer, pos0, n_tok, gem, win, pat, norm = [int(x) for x in g[f"{name}/geom"]]
    th, th_swa, eps = [float(x) for x in g[f"{name}/theta"]]
    shape = AttnShape(name, nl, hq, hkv, hd, cap, pos=pos0, seed=seed, is_gemma3=gem, swa_window=win,
                      swa_pattern=pat)
    return shape, layer, pos0, n_tok, th, th_swa, eps, bool(norm)


def _rope_names():
    return [str(n) for n in np.load(_ROPE_GOLDEN)["cases"]]


@pytest.mark.parametrize("name", _rope_names())
def test_rope_matches_golden(name):
    """The restatement reproduces the reference's tables, rmsnorm_per_head and
    rotation loops bit for bit (golden from oracle/_ref)."""
    from llama3pure_b200.synth import raw_qkv_inputs

    g = np.load(_ROPE_GOLDEN)
    shape, layer, pos0, n_tok, th, th_swa, eps, norm = rope_case(g, name)
    q, k, v, qn, kn = raw_qkv_inputs(shape, layer, n_tok)
    assert sha256_arrays(q, k, v, qn, kn) == str(g[f"{name}/sha256"]), "seeded generator drifted"
    qr, kr = O.rope(shape, layer, pos0, q, k, th, th_swa, eps, qn if norm else None, kn if norm else None,
                    impl="port", n_layers=shape.n_layers)
    np.testing.assert_array_equal(qr.view(np.uint32), g[f"{name}/q"].view(np.uint32))
    np.testing.assert_array_equal(kr.view(np.uint32), g[f"{name}/k"].view(np.uint32))
    assert not np.array_equal(qr, q)  # something was rotated


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (needs the reference source)")
@pytest.mark.parametrize("gemma,norm,hd,layer", [(0, 0, 64, 0), (0, 0, 128, 3), (1, 1, 256, 0), (1, 1, 256, 5),
                                                 (1, 0, 128, 4), (1, 1, 64, 11)])
def test_rope_port_bit_identical_to_reference(gemma, norm, hd, layer):
    rng = np.random.default_rng(hd * 7 + layer)
    shape = AttnShape("r", 12, 8, 2, hd, 3000, is_gemma3=gemma, swa_window=128 if gemma else 0,
                      swa_pattern=6 if gemma else 0)
    n_tok, pos0 = 4, int(rng.integers(0, 2990))
    q = (3 * rng.standard_normal((n_tok, 8 * hd))).astype(np.float32)
    k = (3 * rng.standard_normal((n_tok, 2 * hd))).astype(np.float32)
    qn = (1 + 0.2 * rng.standard_normal((12, hd))).astype(np.float32)
    kn = (1 + 0.2 * rng.standard_normal((12, hd))).astype(np.float32)
    args = (shape, layer, pos0, q, k, 0.0, 0.0, 1e-6, qn if norm else None, kn if norm else None)
    a = O.rope(*args, impl="port", n_layers=12)
    b = O.rope(*args, impl="ref", n_layers=12)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x.view(np.uint32), y.view(np.uint32))


def test_rope_position0_is_identity_without_norm():
    """cos 0 = 1, sin 0 = 0: position 0 leaves q and k unchanged (c:402-404)."""
    shape = AttnShape("p0", 1, 4, 2, 128, 8)
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, 4 * 128)).astype(np.float32)
    k = rng.standard_normal((1, 2 * 128)).astype(np.float32)
    qr, kr = O.rope(shape, 0, 0, q, k, impl="port")
    np.testing.assert_array_equal(qr, q)
    np.testing.assert_array_equal(kr, k)


# ---- the wo projection -------------------------------------------------------

_WO_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "wo_golden.npz")


def _wo_names():
    return [str(n) for n in np.load(_WO_GOLDEN)["cases"]]


@pytest.mark.parametrize("name", _wo_names())
def test_wo_matvec_matches_golden(name):
    """The wo projection of every GGUF weight type the reference reads, bit for bit against the
    reference's own matmul_quantized (golden from oracle/_ref)."""
    from llama3pure_b200.synth import wo_input, wo_weights

    g = np.load(_WO_GOLDEN)
    wt, rows, cols, seed = [int(v) for v in g[f"{name}/geom"]]
    w = wo_weights(wt, rows, cols, seed)
    x = wo_input(cols, seed)
    assert sha256_arrays(w, x) == str(g[f"{name}/sha256"]), "seeded generator drifted"
    got = O.matvec(wt, w, rows, cols, x, impl="port")
    np.testing.assert_array_equal(got.view(np.uint32), g[f"{name}/out"].view(np.uint32))


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built (needs the reference source)")
@pytest.mark.parametrize("wt", [O.W_Q8_0, O.W_Q2_K, O.W_Q3_K, O.W_Q4_K, O.W_Q5_K, O.W_Q6_K, O.W_Q4_0, O.W_Q4_1,
                                O.W_Q5_0, O.W_Q5_1, O.W_IQ4_NL, O.W_F32, O.W_F16, O.W_BF16])
def test_wo_port_bit_identical_to_reference(wt):
    from llama3pure_b200.synth import wo_weights

    rng = np.random.default_rng(wt)
    for rows, cols in ((5, 256), (33, 1024), (4, 8192)):
        w = wo_weights(wt, rows, cols, seed=rows)
        x = rng.standard_normal(cols).astype(np.float32)
        a = O.matvec(wt, w, rows, cols, x, impl="port")
        b = O.matvec(wt, w, rows, cols, x, impl="ref")
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
