"""Causal prefill parity on the GPU through the C ABI against the oracle's
token-by-token loop (llama3pure-c-engine.c:3499-3613), tolerance
|gpu - oracle| <= 1e-4 + 1e-4*|oracle| element-wise."""
import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext
from llama3pure_b200.synth import CONFIGS, AttnShape, prefill_inputs, tolerance_ok

pytestmark = pytest.mark.gpu


def _oracle(sh, q, k, v, start=0):
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=1)
    if start:
        o.prefill(0, 0, q[:start], k[:start], v[:start])
    out, _ = o.prefill(0, start, q[start:], k[start:], v[start:])
    o.close()
    return out


def _check(got, want, what):
    ok, ma, mr = tolerance_ok(got, want)
    assert ok, f"{what}: max_abs={ma:.3e} max_rel={mr:.3e}"


@pytest.mark.parametrize("shape", [
    AttnShape("pf_gqa", 1, 8, 2, 128, 48, pos=47, seed=4),
    AttnShape("pf_mqa_swa", 1, 8, 1, 256, 80, pos=79, seed=5, is_gemma3=1, swa_window=16, swa_pattern=6),
    AttnShape("pf_hd64", 1, 32, 8, 64, 200, pos=199, seed=6),
    AttnShape("pf_one_token", 1, 8, 2, 128, 8, pos=0, seed=7),
    AttnShape("pf_swa_hd128", 1, 8, 2, 128, 300, pos=299, seed=10, is_gemma3=1, swa_window=50, swa_pattern=6),
    AttnShape("pf_ragged_hd128", 1, 12, 3, 128, 333, pos=332, seed=12),
    AttnShape("pf_odd_group_hd128", 1, 6, 2, 128, 290, pos=289, seed=14),
])
def test_prefill_small_matches_oracle(shape):
    k, v, q = prefill_inputs(shape, 0)
    with AttnContext.for_shape(shape, n_layers=1) as ctx:
        got = ctx.prefill(0, 0, q, k, v)
    _check(got, _oracle(shape, q, k, v), shape.name)


@pytest.mark.parametrize("path", ["tc_pair", "tc_single", "ffma"])
def test_prefill_paths_agree_with_oracle(monkeypatch, path):
    """head_dim 128 prefill runs on the tcgen05 tensor cores (3xTF32): CTA
    pairs (cta_group::2) for even GQA groups, single CTAs otherwise; the FFMA
    path (decode kernel, one slice per token) is kept for other head sizes.
    All must meet the same tolerance."""
    if path == "ffma":
        monkeypatch.setenv("L3P_PREFILL_PATH", "ffma")
    if path == "tc_pair":
        monkeypatch.setenv("L3P_PREFILL_CG", "2")
    sh = AttnShape("pf_path", 1, 32, 8, 128, 640, pos=639, seed=13)
    k, v, q = prefill_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        got = ctx.prefill(0, 0, q, k, v)
    _check(got, _oracle(sh, q, k, v), f"prefill path {path}")


def test_prefill_continues_an_existing_cache():
    sh = AttnShape("pf_cont", 1, 8, 2, 128, 96, pos=95, seed=8)
    k, v, q = prefill_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        first = ctx.prefill(0, 0, q[:40], k[:40], v[:40])
        second = ctx.prefill(0, 40, q[40:], k[40:], v[40:])
    want = _oracle(sh, q, k, v)
    _check(np.concatenate([first, second]), want, "split prefill")


def test_prefill_8b_2k_layer0_matches_oracle():
    sh = CONFIGS["llama31_8b_prefill_2k"]
    k, v, q = prefill_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        got = ctx.prefill(0, 0, q, k, v)
    _check(got, _oracle(sh, q, k, v), "8B prefill 2k")


def test_prefill_device_entry_point_matches_host():
    import torch

    sh = AttnShape("pf_dev", 2, 32, 8, 128, 256, pos=255, seed=9)
    k, v, q = prefill_inputs(sh, 1)
    with AttnContext.for_shape(sh) as ctx:
        host = ctx.prefill(1, 0, q, k, v)
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        out = torch.zeros_like(dq)
        ctx.prefill_dev(0, 0, q.shape[0], dq, dk, dv, out)
        torch.cuda.synchronize()
        ctx.check()
    np.testing.assert_allclose(out.cpu().numpy(), host, rtol=1e-6, atol=1e-7)


def test_prefill_image_growth_keeps_rope_tables_and_wo_weights():
    """A prefill longer than any before it regrows the tensor-core image
    buffer; the RoPE tables and wo weights set earlier must stay valid (a raw
    step and the projection after the growth match the oracle's chain)."""
    from llama3pure_b200.synth import raw_qkv_inputs, wo_weights

    sh = AttnShape("pf_grow", 1, 8, 2, 128, 520, pos=511, seed=15)
    k, v, q = prefill_inputs(sh, 0)
    qr, kr, vr, _, _ = raw_qkv_inputs(sh, 0, 1)
    pos, cols = 512, sh.n_heads * sh.head_dim
    w = wo_weights(8, 256, cols, seed=4)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        ctx.set_rope()
        ctx.set_wo(0, 8, w)
        ctx.prefill(0, 0, q[:64], k[:64], v[:64])      # image sized for 64 keys
        ctx.prefill(0, 64, q[64:], k[64:], v[64:])     # grows it to 512 keys
        att = ctx.step_raw(0, pos, qr[0].copy(), kr[0].copy(), vr[0].copy())
        xb2 = ctx.wo(0, att.reshape(-1).copy())
    q_rot, k_rot = O.rope(sh, 0, pos, qr, kr, n_layers=1)
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=1)
    o.load_kv(0, 0, np.ascontiguousarray(k.transpose(1, 0, 2)), np.ascontiguousarray(v.transpose(1, 0, 2)))
    want, _ = o.decode(0, pos, q_rot.reshape(-1), k_rot.reshape(-1).copy(), vr.reshape(-1).copy())
    o.close()
    _check(att.reshape(-1), want.reshape(-1), "raw step after image growth")
    _check(xb2, O.matvec(8, w, 256, cols, np.ascontiguousarray(att.reshape(-1))), "wo after image growth")


@pytest.mark.parametrize("name,shape", [
    # Llama-3.2-1B shapes (head_dim 64, tensor cores) and Gemma shapes (head_dim
    # 256, the decode kernel in token mode) at a 2048-token prompt
    ("l1b_2k_hd64", CONFIGS["llama32_1b_decode"].with_(n_layers=1, seq_len=2048, pos=2047, seed=16)),
    ("gemma_2k_hd256", CONFIGS["gemma_2b_decode"].with_(n_layers=1, seq_len=2048, pos=2047, seed=17)),
])
def test_prefill_2k_other_head_sizes_match_oracle(name, shape):
    k, v, q = prefill_inputs(shape, 0)
    with AttnContext.for_shape(shape, n_layers=1) as ctx:
        got = ctx.prefill(0, 0, q, k, v)
    _check(got, _oracle(shape, q, k, v), name)


@pytest.mark.parametrize("kv_format", [0, 1])
def test_prefill_hd64_continuation_and_q8_cache(kv_format):
    """head_dim 64 on the tensor cores: a prompt continued in a second call
    (keys of the first call's tiles), ragged lengths, both cache formats."""
    sh = AttnShape("pf_hd64_cont", 1, 16, 4, 64, 700, pos=699, seed=18)
    k, v, q = prefill_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1, kv_format=kv_format) as ctx:
        first = ctx.prefill(0, 0, q[:333], k[:333], v[:333])
        second = ctx.prefill(0, 333, q[333:], k[333:], v[333:])
    got = np.concatenate([first, second])
    if kv_format == 0:
        _check(got, _oracle(sh, q, k, v), "hd64 split prefill")
    else:
        o = O.Oracle(sh, O.MODE_Q8, "port", n_layers=1)
        want, _ = o.prefill(0, 0, q, k, v)
        o.close()
        _check(got, want, "hd64 split prefill, Q8_0 cache")
