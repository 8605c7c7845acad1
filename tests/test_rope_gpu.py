"""The pre-attention step on the GPU (QK-norm, RoPE, cache write) through the C ABI.

Bits: l3p_attn_rope_dev must reproduce the reference's pre-attention
arithmetic exactly -- the golden rows of tests/golden/rope_golden.npz come
from the reference's own cos/sin tables (malloc_run_state,
llama3pure-c-engine.c:381-421) and rmsnorm_per_head (c:3150-3165) -- and the
K rows the raw entry points store must be the oracle's rotated rows bit for
bit (fp32 cache) or their Q8_0 bytes (Q8_0 cache).

Attention: step_raw / prefill_raw must equal the oracle's attention over the
oracle's rotated q and K within |gpu - ref| <= 1e-4 + 1e-4*|ref|.
"""
import os

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext, AttnError
from llama3pure_b200.synth import CONFIGS, GEMMA_SWA, AttnShape, raw_qkv_inputs, tolerance_ok
from test_oracle import rope_case

pytestmark = pytest.mark.gpu

Q8 = 1
ROPE_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "rope_golden.npz")


def _torch():
    import torch

    return torch


def _check(got, want, what):
    ok, ma, mr = tolerance_ok(got, want)
    assert ok, f"{what}: max_abs={ma:.3e} max_rel={mr:.3e}"


def _q8_blocks(x):
    prim = O.primitives("port")
    flat = np.ascontiguousarray(x.reshape(-1, x.shape[-1]), dtype=np.float32)
    hd = flat.shape[1]
    out = np.zeros((flat.shape[0], hd // 32 * 34), np.uint8)
    for r in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[r])
        prim["q8_quantize"](O._fptr(row), out[r].ctypes.data, hd)
    return out.reshape(x.shape[:-1] + (hd // 32 * 34,))


def _rope_kw(theta, theta_swa, eps, norm, qn, kn, n_layers):
    return dict(rope_theta=theta, rope_theta_swa=theta_swa, rms_norm_eps=eps,
                q_norm=qn[:n_layers] if norm else None, k_norm=kn[:n_layers] if norm else None)


@pytest.mark.parametrize("name", [str(n) for n in np.load(ROPE_GOLDEN)["cases"]])
def test_rope_dev_matches_reference_golden(name):
    torch = _torch()
    g = np.load(ROPE_GOLDEN)
    shape, layer, pos0, n_tok, th, th_swa, eps, norm = rope_case(g, name)
    q, k, v, qn, kn = raw_qkv_inputs(shape, layer, n_tok)
    nl = layer + 1
    with AttnContext.for_shape(shape, n_layers=nl, seq_len=max(shape.seq_len, pos0 + n_tok), kv_format=Q8) as ctx:
        ctx.set_rope(**_rope_kw(th, th_swa, eps, norm, qn, kn, nl))
        dq, dk = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
        oq, ok_ = torch.full_like(dq, float("nan")), torch.full_like(dk, float("nan"))
        ctx.rope_dev(layer, pos0, n_tok, dq, dk, oq, ok_)
        ctx.check()
        gq, gk = oq.cpu().numpy(), ok_.cpu().numpy()
    np.testing.assert_array_equal(gq.view(np.uint32), g[f"{name}/q"].view(np.uint32))
    np.testing.assert_array_equal(gk.view(np.uint32), g[f"{name}/k"].view(np.uint32))


RAW_SHAPES = {
    "l8b": (CONFIGS["llama31_8b_decode_8k"].with_(seq_len=600, n_layers=2), 1, False),
    "gemma_swa_norm_l0": (GEMMA_SWA.with_(seq_len=700, n_layers=6, swa_window=96), 0, True),
    "gemma_swa_norm_l5": (GEMMA_SWA.with_(seq_len=700, n_layers=6, swa_window=96), 5, True),
    "l1b_hd64": (CONFIGS["llama32_1b_decode"].with_(seq_len=400, n_layers=1), 0, False),
    "gqa3_hd128": (AttnShape("gqa3", 1, 6, 2, 128, 300, seed=31), 0, False),
}


def _expected_step(shape, layer, pos, hist_k, hist_v, qr, kr, v, mode):
    o = O.Oracle(shape, mode, "port", n_layers=layer + 1)
    if pos:
        o.load_kv(layer, 0, hist_k, hist_v)
    kd = shape.n_kv_heads * shape.head_dim
    out, _ = o.decode(layer, pos, qr.reshape(-1), kr.reshape(kd).copy(), v.reshape(kd).copy())
    o.close()
    return out


@pytest.mark.parametrize("kv_format", [0, Q8])
@pytest.mark.parametrize("entry", ["host", "dev", "dev_overlap"])
@pytest.mark.parametrize("case", list(RAW_SHAPES))
def test_step_raw_matches_oracle(case, entry, kv_format):
    torch = _torch()
    shape, layer, norm = RAW_SHAPES[case]
    pos = shape.seq_len - 3
    rng = np.random.default_rng(sum(case.encode()))
    hd, hkv = shape.head_dim, shape.n_kv_heads
    hist_k = rng.standard_normal((hkv, pos, hd)).astype(np.float32)
    hist_v = rng.standard_normal((hkv, pos, hd)).astype(np.float32)
    q, k, v, qn, kn = raw_qkv_inputs(shape, layer, 1)
    th, th_swa, eps = (1e6, 1e4, 1e-6) if shape.is_gemma3 else (5e5, 0.0, 0.0)
    qr, kr = O.rope(shape, layer, pos, q, k, th, th_swa, eps, qn if norm else None, kn if norm else None,
                    n_layers=shape.n_layers)
    mode = O.MODE_Q8 if kv_format == Q8 else O.MODE_F32
    want = _expected_step(shape, layer, pos, hist_k, hist_v, qr, kr, v, mode)
    with AttnContext.for_shape(shape, kv_format=kv_format) as ctx:
        ctx.set_rope(**_rope_kw(th, th_swa, eps, norm, qn, kn, shape.n_layers))
        ctx.load_kv(layer, 0, hist_k, hist_v)
        if entry == "host":
            got = ctx.step_raw(layer, pos, q[0].copy(), k[0].copy(), v[0].copy())
        else:
            ctx.set_overlap(entry == "dev_overlap")
            dq, dk, dv = (torch.from_numpy(a[0].copy()).cuda() for a in (q, k, v))
            dout = torch.zeros(shape.n_heads * hd, device="cuda")
            ctx.step_raw_dev(layer, pos, dq, dk, dv, dout)
            ctx.check()
            got = dout.cpu().numpy().reshape(shape.n_heads, hd)
        if kv_format == Q8:
            kb, vb = ctx.read_kv_q8(layer, pos, 1)
            np.testing.assert_array_equal(kb[:, 0], _q8_blocks(kr.reshape(hkv, hd)))
            np.testing.assert_array_equal(vb[:, 0], _q8_blocks(v.reshape(hkv, hd)))
        else:
            kc, vc = ctx.read_kv(layer, pos, 1)
            np.testing.assert_array_equal(kc[:, 0].view(np.uint32), kr.reshape(hkv, hd).view(np.uint32))
            np.testing.assert_array_equal(vc[:, 0].view(np.uint32), v.reshape(hkv, hd).view(np.uint32))
    _check(got, want, f"{case} {entry} kv_format={kv_format}")


PREFILL_SHAPES = {
    "l8b_tc": (CONFIGS["llama31_8b_prefill_2k"].with_(seq_len=320, n_layers=1), 0, False, 300),
    "gemma_swa_norm": (GEMMA_SWA.with_(seq_len=200, n_layers=6, swa_window=40), 5, True, 150),
    "gemma_swa_norm_l1": (GEMMA_SWA.with_(seq_len=200, n_layers=6, swa_window=40), 1, True, 150),
    "l1b_hd64": (CONFIGS["llama32_1b_decode"].with_(seq_len=160, n_layers=1), 0, False, 130),
}


@pytest.mark.parametrize("kv_format", [0, Q8])
@pytest.mark.parametrize("start", [0, 17])
@pytest.mark.parametrize("entry", ["host", "dev"])
@pytest.mark.parametrize("case", list(PREFILL_SHAPES))
def test_prefill_raw_matches_oracle(case, entry, start, kv_format):
    torch = _torch()
    shape, layer, norm, n_tok = PREFILL_SHAPES[case]
    hd, hkv, hq = shape.head_dim, shape.n_kv_heads, shape.n_heads
    rng = np.random.default_rng(7 + start)
    hist_k = rng.standard_normal((hkv, start, hd)).astype(np.float32)
    hist_v = rng.standard_normal((hkv, start, hd)).astype(np.float32)
    q, k, v, qn, kn = raw_qkv_inputs(shape, layer, n_tok)
    th, th_swa, eps = (1e6, 1e4, 1e-6) if shape.is_gemma3 else (5e5, 0.0, 0.0)
    qr, kr = O.rope(shape, layer, start, q, k, th, th_swa, eps, qn if norm else None, kn if norm else None,
                    n_layers=shape.n_layers)
    mode = O.MODE_Q8 if kv_format == Q8 else O.MODE_F32
    o = O.Oracle(shape, mode, "port", n_layers=layer + 1)
    if start:
        o.load_kv(layer, 0, hist_k, hist_v)
    want, _ = o.prefill(layer, start, qr.reshape(n_tok, hq, hd), kr.reshape(n_tok, hkv, hd),
                        v.reshape(n_tok, hkv, hd))
    o.close()
    with AttnContext.for_shape(shape, kv_format=kv_format) as ctx:
        ctx.set_rope(**_rope_kw(th, th_swa, eps, norm, qn, kn, shape.n_layers))
        if start:
            ctx.load_kv(layer, 0, hist_k, hist_v)
        if entry == "host":
            got = ctx.prefill_raw(layer, start, q, k, v)
        else:
            dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
            dout = torch.zeros(n_tok, hq * hd, device="cuda")
            ctx.prefill_raw_dev(layer, start, n_tok, dq, dk, dv, dout)
            ctx.check()
            got = dout.cpu().numpy().reshape(n_tok, hq, hd)
        if kv_format == Q8:
            kb, vb = ctx.read_kv_q8(layer, start, n_tok)
            np.testing.assert_array_equal(kb, _q8_blocks(kr.reshape(n_tok, hkv, hd).transpose(1, 0, 2)))
            np.testing.assert_array_equal(vb, _q8_blocks(v.reshape(n_tok, hkv, hd).transpose(1, 0, 2)))
        else:
            kc, vc = ctx.read_kv(layer, start, n_tok)
            np.testing.assert_array_equal(kc, kr.reshape(n_tok, hkv, hd).transpose(1, 0, 2))
            np.testing.assert_array_equal(vc, v.reshape(n_tok, hkv, hd).transpose(1, 0, 2))
    _check(got, want, f"{case} {entry} start={start} kv_format={kv_format}")


def test_step_raw_dev_layer_chain_with_overlap():
    """Consecutive layers through step_raw_dev with programmatic dependent
    launch: each layer's pre-attention kernel overlaps the previous decode."""
    torch = _torch()
    shape = GEMMA_SWA.with_(seq_len=520, n_layers=7, swa_window=64)
    pos = 515
    hd, hkv, hq = shape.head_dim, shape.n_kv_heads, shape.n_heads
    rng = np.random.default_rng(99)
    th, th_swa, eps = 1e6, 1e4, 1e-6
    qn, kn = raw_qkv_inputs(shape, 0, 1)[3:]
    with AttnContext.for_shape(shape) as ctx:
        ctx.set_rope(th, th_swa, eps, qn, kn)
        ins, wants = [], []
        for layer in range(shape.n_layers):
            hk = rng.standard_normal((hkv, pos, hd)).astype(np.float32)
            hv = rng.standard_normal((hkv, pos, hd)).astype(np.float32)
            ctx.load_kv(layer, 0, hk, hv)
            q, k, v = raw_qkv_inputs(shape, layer, 1)[:3]
            qr, kr = O.rope(shape, layer, pos, q, k, th, th_swa, eps, qn, kn, n_layers=shape.n_layers)
            wants.append(_expected_step(shape, layer, pos, hk, hv, qr, kr, v, O.MODE_F32))
            ins.append(tuple(torch.from_numpy(a[0].copy()).cuda() for a in (q, k, v)))
        ctx.set_overlap(True)
        outs = []
        for layer, (dq, dk, dv) in enumerate(ins):
            dout = torch.zeros(hq * hd, device="cuda")
            ctx.step_raw_dev(layer, pos, dq, dk, dv, dout)
            outs.append(dout)
        ctx.check()
        for layer in range(shape.n_layers):
            _check(outs[layer].cpu().numpy().reshape(hq, hd), wants[layer], f"layer {layer}")


def test_rope_dev_sharded_context_writes_owned_heads_only():
    torch = _torch()
    shape = CONFIGS["llama31_8b_decode_8k"].with_(seq_len=64, n_layers=1)
    q, k, _, _, _ = raw_qkv_inputs(shape, 0, 3)
    qr, kr = O.rope(shape, 0, 40, q, k)
    hd = shape.head_dim
    with AttnContext.for_shape(shape, kv_head_begin=2, kv_head_count=3) as ctx:
        ctx.set_rope()
        dq, dk = torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda()
        oq, ok_ = torch.full_like(dq, -7.0), torch.full_like(dk, -7.0)
        ctx.rope_dev(0, 40, 3, dq, dk, oq, ok_)
        ctx.check()
        gq, gk = oq.cpu().numpy(), ok_.cpu().numpy()
    G = shape.kv_mul
    qlo, qhi = 2 * G * hd, 5 * G * hd
    np.testing.assert_array_equal(gq[:, qlo:qhi], qr[:, qlo:qhi])
    assert np.all(gq[:, :qlo] == -7.0) and np.all(gq[:, qhi:] == -7.0)
    np.testing.assert_array_equal(gk[:, 2 * hd:5 * hd], kr[:, 2 * hd:5 * hd])
    assert np.all(gk[:, :2 * hd] == -7.0) and np.all(gk[:, 5 * hd:] == -7.0)


def test_raw_entry_points_need_set_rope():
    shape = CONFIGS["llama32_1b_decode"].with_(seq_len=16, n_layers=1)
    q, k, v, _, _ = raw_qkv_inputs(shape, 0, 1)
    with AttnContext.for_shape(shape) as ctx:
        with pytest.raises(AttnError) as e:
            ctx.step_raw(0, 3, q[0].copy(), k[0].copy(), v[0].copy())
        assert e.value.code == -1
        with pytest.raises(AttnError) as e:
            ctx.prefill_raw(0, 0, q, k, v)
        assert e.value.code == -1
