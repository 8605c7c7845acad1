"""The Q8_0 KV cache (kv_format = L3P_KV_Q8_0) on the GPU through the C ABI.

Bytes: the device quantiser must reproduce quantize_to_q8_0_cache
(llama3pure-c-engine.c:1535-1570) bit for bit -- checked against the
reference's own known-answer blocks in the golden file and against the
oracle's restatement on every geometry.

Attention: decode and prefill over the Q8_0 cache must match the reference as
shipped (the golden "q8" outputs, produced by the reference's own functions)
within |gpu - ref| <= 1e-4 + 1e-4*|ref|; the integer dot products are exact,
only fp32 summation order and exp differ.
"""
import os

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext, AttnError
from llama3pure_b200.synth import CONFIGS, AttnShape, decode_inputs, prefill_inputs, tolerance_ok

pytestmark = pytest.mark.gpu

Q8 = 1  # L3P_KV_Q8_0


def _check(got, want, what):
    ok, ma, mr = tolerance_ok(got, want)
    assert ok, f"{what}: max_abs={ma:.3e} max_rel={mr:.3e}"


def _golden_cases(golden, prefill):
    return [str(n) for n in golden["cases"] if str(n).startswith("prefill") == prefill]


def _shape_from(g, name):
    hq, hkv, hd, cap, pos, seed, layer, append, gem, win, pat = [int(x) for x in g[f"{name}/geom"]]
    return AttnShape(name, layer + 1, hq, hkv, hd, cap, pos=pos, seed=seed, k_scale=float(g[f"{name}/k_scale"]),
                     is_gemma3=gem, swa_window=win, swa_pattern=pat), layer, bool(append)


def _oracle_blocks(x):
    """Reference Q8_0 bytes of rows x[..., hd] (oracle restatement)."""
    prim = O.primitives("port")
    flat = np.ascontiguousarray(x.reshape(-1, x.shape[-1]), dtype=np.float32)
    hd = flat.shape[1]
    out = np.zeros((flat.shape[0], hd // 32 * 34), np.uint8)
    for r in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[r])
        prim["q8_quantize"](O._fptr(row), out[r].ctypes.data, hd)
    return out.reshape(x.shape[:-1] + (hd // 32 * 34,))


def test_quantiser_reproduces_reference_known_answer_blocks(golden):
    """The reference's own blocks for 256 values (one all-zero block, c:1550)."""
    x = np.ascontiguousarray(golden["kat/q8_in"], dtype=np.float32).reshape(1, 1, 256)
    with AttnContext(1, 1, 1, 256, 4, kv_format=Q8) as ctx:
        ctx.load_kv(0, 0, x, x)                       # bulk path
        ctx.kv_append(0, 1, x.reshape(256), x.reshape(256))  # token path
        kb, vb = ctx.read_kv_q8(0, 0, 2)
    want = golden["kat/q8_blocks"]
    for row in (kb[0, 0], vb[0, 0], kb[0, 1], vb[0, 1]):
        np.testing.assert_array_equal(row, want)


@pytest.mark.parametrize("hd,hkv", [(64, 8), (128, 8), (256, 1)])
def test_cache_bytes_match_the_reference_quantiser(hd, hkv):
    sh = AttnShape("bytes", 1, hkv * 4, hkv, hd, 300, pos=299, seed=40 + hd)
    k, v, _ = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1, kv_format=Q8) as ctx:
        ctx.load_kv(0, 0, k[:, :200].copy(), v[:, :200].copy())
        for p in range(200, 300):
            ctx.kv_append(0, p, k[:, p].copy(), v[:, p].copy())
        kb, vb = ctx.read_kv_q8(0, 0, 300)
        kd, vd = ctx.read_kv(0, 0, 300)
    np.testing.assert_array_equal(kb, _oracle_blocks(k))
    np.testing.assert_array_equal(vb, _oracle_blocks(v))
    # read_kv returns the dequantised values d * int8
    blk = kb.reshape(hkv, 300, hd // 32, 34)
    d = blk[..., :2].copy().view(np.float16).astype(np.float32)
    q = blk[..., 2:].view(np.int8).astype(np.float32)
    np.testing.assert_array_equal(kd, (q * d).reshape(hkv, 300, hd))


def test_load_kv_q8_round_trip_and_decode():
    sh = AttnShape("blocks", 1, 32, 8, 128, 513, pos=512, seed=44)
    k, v, q = decode_inputs(sh, 0)
    kb, vb = _oracle_blocks(k), _oracle_blocks(v)
    with AttnContext.for_shape(sh, n_layers=1, kv_format=Q8) as ctx:
        ctx.load_kv_q8(0, 0, kb, vb)
        rk, rv = ctx.read_kv_q8(0, 0, sh.seq_len)
        got = ctx.decode(0, sh.pos, q)
    np.testing.assert_array_equal(rk, kb)
    np.testing.assert_array_equal(rv, vb)
    o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=1)
    o.load_kv(0, 0, k, v)
    want, _ = o.decode(0, sh.pos, q)
    o.close()
    _check(got, want, "decode after load_kv_q8")


def _decode_case(golden, name):
    sh, layer, append = _shape_from(golden, name)
    k, v, q = decode_inputs(sh, layer)
    with AttnContext.for_shape(sh, n_layers=layer + 1, kv_format=Q8) as ctx:
        if append:
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            got = ctx.step(layer, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))
        else:
            ctx.load_kv(layer, 0, k, v)
            got = ctx.decode(layer, sh.pos, q)
    return got


def test_decode_matches_reference_as_shipped(golden):
    # head_dim 64, 128 and 256 have kernels (32 is rejected at create, as for fp32)
    names = [n for n in _golden_cases(golden, prefill=False) if int(golden[f"{n}/geom"][2]) in (64, 128, 256)]
    assert len(names) >= 10
    for name in names:
        got = _decode_case(golden, name)
        _check(got, golden[f"{name}/q8"], name)


def test_prefill_matches_reference_as_shipped(golden):
    names = [n for n in _golden_cases(golden, prefill=True) if f"{n}/q8" in golden.files]
    assert names
    for name in names:
        sh, layer, _ = _shape_from(golden, name)
        k, v, q = prefill_inputs(sh, layer)
        with AttnContext.for_shape(sh, n_layers=layer + 1, kv_format=Q8) as ctx:
            out = ctx.prefill(layer, 0, q, k, v)
        rows = golden[f"{name}/q8_rows"]
        _check(out[rows], golden[f"{name}/q8"], name)
        np.testing.assert_allclose(out.astype(np.float64).sum(axis=(1, 2)), golden[f"{name}/q8_rowsum"],
                                   rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("path", ["tc", "ffma"])
def test_prefill_paths_match_oracle(monkeypatch, path):
    """head_dim 128 prefill on the tensor cores (dequantised cache, q
    quantised to Q8_0 and back in the kernel) and on the decode kernel."""
    if path == "ffma":
        monkeypatch.setenv("L3P_PREFILL_PATH", "ffma")
    sh = AttnShape("pf_q8", 1, 32, 8, 128, 700, pos=699, seed=45)
    k, v, q = prefill_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1, kv_format=Q8) as ctx:
        first = ctx.prefill(0, 0, q[:300], k[:300], v[:300])
        second = ctx.prefill(0, 300, q[300:], k[300:], v[300:])
    o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=1)
    want, _ = o.prefill(0, 0, q, k, v)
    o.close()
    _check(np.concatenate([first, second]), want, f"q8 prefill {path}")


@pytest.mark.parametrize("name,layers", [
    ("llama32_1b_decode", [0, 7, 15]),
    ("llama31_8b_decode_8k", [0, 31]),
    ("gemma_2b_decode", [0, 17]),
])
def test_baseline_configs_match_oracle(name, layers):
    sh = CONFIGS[name]
    with AttnContext.for_shape(sh, n_layers=max(layers) + 1, seq_len=sh.pos + 1, kv_format=Q8) as ctx:
        for layer in layers:
            k, v, q = decode_inputs(sh, layer)
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            got = ctx.step(layer, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))
            o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=layer + 1, seq_len=sh.pos + 1)
            o.load_kv(layer, 0, k, v)
            want, _ = o.decode(layer, sh.pos, q)
            o.close()
            _check(got, want, f"{name} layer {layer}")


def test_device_entry_points_match_host():
    import torch

    sh = AttnShape("dev_q8", 4, 32, 8, 128, 1024, pos=1000, seed=46)
    with AttnContext.for_shape(sh, kv_format=Q8) as ctx:
        qs = []
        for layer in range(4):
            k, v, q = decode_inputs(sh, layer)
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            ctx.kv_append(layer, sh.pos, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))
            qs.append(q)
        host = np.stack([ctx.decode(layer, sh.pos, qs[layer]) for layer in range(4)])
        dq = torch.from_numpy(np.stack(qs)).cuda()
        out = torch.zeros_like(dq)
        ctx.decode_layers_dev(0, 4, sh.pos, dq, out)
        one = torch.zeros_like(dq[0])
        ctx.decode_dev(2, sh.pos, dq[2], one)
        # sequence partial of the whole range merged alone is the full result
        po = torch.zeros_like(dq[1])
        pml = torch.zeros((sh.n_heads, 2), device="cuda")
        ctx.decode_partial_dev(1, sh.pos, dq[1], po, pml)
        merged = torch.zeros_like(dq[1])
        ctx.lse_merge_dev(1, sh.n_heads, 0, sh.n_heads, po, pml, merged)
        torch.cuda.synchronize()
        ctx.check()
    np.testing.assert_allclose(out.cpu().numpy(), host, rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(one.cpu().numpy(), host[2], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(merged.cpu().numpy(), host[1], rtol=1e-5, atol=1e-6)


def test_step_dev_appends_then_attends():
    import torch

    sh = AttnShape("stepdev_q8", 1, 8, 2, 256, 600, pos=599, seed=47)
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1, kv_format=Q8) as ctx:
        ctx.load_kv(0, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
        dk = torch.from_numpy(np.ascontiguousarray(k[:, sh.pos])).cuda()
        dv = torch.from_numpy(np.ascontiguousarray(v[:, sh.pos])).cuda()
        dq = torch.from_numpy(q).cuda()
        out = torch.zeros_like(dq)
        ctx.step_dev(0, sh.pos, dq, dk, dv, out)
        torch.cuda.synchronize()
        ctx.check()
        kb, _ = ctx.read_kv_q8(0, sh.pos, 1)
    np.testing.assert_array_equal(kb[:, 0], _oracle_blocks(k[:, sh.pos]))
    o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=1)
    o.load_kv(0, 0, k, v)
    want, _ = o.decode(0, sh.pos, q)
    o.close()
    _check(out.cpu().numpy(), want, "q8 step_dev")


@pytest.mark.parametrize("plan", ["1:1", "7:1", "16:16", "32:8", "64:4"])
def test_every_merge_path(monkeypatch, plan):
    monkeypatch.setenv("L3P_DECODE_PLAN", plan)
    sh = CONFIGS["llama31_8b_decode_8k"]
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1, seq_len=sh.pos + 1, kv_format=Q8) as ctx:
        ctx.load_kv(0, 0, k, v)
        got = ctx.decode(0, sh.pos, q)
    o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=1, seq_len=sh.pos + 1)
    o.load_kv(0, 0, k, v)
    want, _ = o.decode(0, sh.pos, q)
    o.close()
    _check(got, want, f"plan {plan}")


def test_fp32_only_entry_points_refuse_a_q8_cache():
    with AttnContext(1, 8, 2, 128, 64, kv_format=Q8) as ctx:
        with pytest.raises(AttnError):
            ctx.kv_device_ptr(0)
    with AttnContext(1, 8, 2, 128, 64) as ctx:
        with pytest.raises(AttnError):
            ctx.read_kv_q8(0, 0, 4)


@pytest.mark.parametrize("overlap", [False, True])
def test_step_dev_layer_chain_in_a_graph(overlap):
    """Consecutive layers of step_dev (one launch each: the decode quantises
    and stores the new row itself) captured in a CUDA graph, with and without
    programmatic dependent launch between the layers."""
    import torch

    sh = CONFIGS["llama31_8b_decode_8k"].with_(seq_len=1024, pos=1023, n_layers=4)
    ks, vs, qs = [], [], []
    with AttnContext.for_shape(sh, kv_format=Q8) as ctx:
        for layer in range(sh.n_layers):
            k, v, q = decode_inputs(sh.with_(seed=60 + layer), layer)
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            ks.append(k)
            vs.append(v)
            qs.append(q)
        dq = torch.from_numpy(np.stack([q.reshape(-1) for q in qs])).cuda()
        dk = torch.from_numpy(np.stack([np.ascontiguousarray(k[:, sh.pos]).reshape(-1) for k in ks])).cuda()
        dv = torch.from_numpy(np.stack([np.ascontiguousarray(v[:, sh.pos]).reshape(-1) for v in vs])).cuda()
        out = torch.zeros_like(dq)
        ctx.set_overlap(overlap)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for layer in range(sh.n_layers):
                    ctx.step_dev(layer, sh.pos, dq[layer], dk[layer], dv[layer], out[layer], s)
            g.replay()
        torch.cuda.synchronize()
        ctx.check()
        got = out.cpu().numpy()
        del g
    for layer in range(sh.n_layers):
        o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=layer + 1)
        o.load_kv(layer, 0, ks[layer], vs[layer])
        want, _ = o.decode(layer, sh.pos, qs[layer])
        o.close()
        _check(got[layer].reshape(want.shape), want, f"q8 step_dev chain layer {layer} overlap={overlap}")


@pytest.mark.parametrize("kv_format", [0, Q8])
@pytest.mark.parametrize("plan", ["auto", "1:1", "3:1"])
def test_same_layer_consecutive_positions_under_overlap(monkeypatch, kv_format, plan):
    """One layer stepped at positions p, p+1, ... back to back in a CUDA graph
    with programmatic dependent launch, across tile boundaries (8 rows for
    fp32, 16 for Q8_0): each step's launch may start while the previous one
    still runs, and copies the cache row the previous one stored; that store
    must land first.  Every output matches the oracle and the cache holds the
    appended rows (Q8_0: the reference quantiser's bytes)."""
    import torch

    if plan != "auto":
        monkeypatch.setenv("L3P_DECODE_PLAN", plan)
    sh = AttnShape("samelayer", 1, 8, 2, 128, 64, pos=60, seed=71)
    p0, n = 13, 20  # positions 13..32 cross the boundaries at 16, 24 and 32
    k, v, q = decode_inputs(sh, 0)
    qs = np.random.default_rng(72).standard_normal((n, sh.n_heads, sh.head_dim)).astype(np.float32)
    with AttnContext.for_shape(sh, n_layers=1, kv_format=kv_format) as ctx:
        ctx.load_kv(0, 0, np.ascontiguousarray(k[:, :p0]), np.ascontiguousarray(v[:, :p0]))
        dq = torch.from_numpy(qs).cuda()
        dk = torch.from_numpy(np.ascontiguousarray(k[:, p0:p0 + n].transpose(1, 0, 2))).cuda()
        dv = torch.from_numpy(np.ascontiguousarray(v[:, p0:p0 + n].transpose(1, 0, 2))).cuda()
        out = torch.zeros_like(dq)
        ctx.set_overlap(True)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(n):
                    ctx.step_dev(0, p0 + i, dq[i], dk[i], dv[i], out[i], s)
            g.replay()
        torch.cuda.synchronize()
        ctx.check()
        got = out.cpu().numpy()
        if kv_format == Q8:
            kb, vb = ctx.read_kv_q8(0, p0, n)
        else:
            kc, vc = ctx.read_kv(0, p0, n)
        del g
    if kv_format == Q8:
        np.testing.assert_array_equal(kb, _oracle_blocks(k[:, p0:p0 + n]))
        np.testing.assert_array_equal(vb, _oracle_blocks(v[:, p0:p0 + n]))
    else:
        np.testing.assert_array_equal(kc, k[:, p0:p0 + n])
        np.testing.assert_array_equal(vc, v[:, p0:p0 + n])
    mode = O.MODE_Q8 if kv_format == Q8 else O.MODE_F32
    o = O.Oracle(sh, mode, "port", n_layers=1)
    o.load_kv(0, 0, k, v)
    for i in range(n):
        want, _ = o.decode(0, p0 + i, qs[i])
        _check(got[i], want, f"kv_format {kv_format} plan {plan} pos {p0 + i}")
    o.close()
