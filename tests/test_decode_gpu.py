"""Decode parity on the GPU through the C ABI against the CPU oracle.

Contract (north star): max-abs 1e-4 / rel 1e-4 in fp32 against the
reference's attention loop with an fp32 KV cache ("f32" oracle mode), checked
element-wise as |gpu - oracle| <= 1e-4 + 1e-4*|oracle|.  The gap to the
reference as shipped (Q8_0 cache, "q8" mode) is reported, not asserted at
1e-4: it is the quantisation error of the reference itself.
"""
import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext
from llama3pure_b200.synth import CONFIGS, GEMMA_SWA, AttnShape, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu

ATOL = 1e-4
RTOL = 1e-4


def _oracle(sh, layer, k, v, q, mode=O.MODE_F32):
    o = O.Oracle(sh, mode, "port", n_layers=layer + 1, seq_len=k.shape[1])
    o.load_kv(layer, 0, k, v)
    out, skipped = o.decode(layer, sh.pos, q)
    o.close()
    return out, skipped


def _gpu_step(ctx, sh, layer, k, v, q):
    """Bulk-load positions [0, pos), then the engine's block: append row pos + decode."""
    ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
    return ctx.step(layer, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))


def _check(got, want, what):
    ok, ma, mr = tolerance_ok(got, want, ATOL, RTOL)
    assert ok, f"{what}: max_abs={ma:.3e} max_rel={mr:.3e}"
    return ma, mr


@pytest.mark.parametrize("name,layers", [
    ("llama32_1b_decode", list(range(16))),
    ("llama31_8b_decode_8k", [0, 1, 31]),
    ("gemma_2b_decode", list(range(18))),
])
def test_baseline_config_decode_matches_oracle(name, layers):
    sh = CONFIGS[name]
    with AttnContext.for_shape(sh, n_layers=max(layers) + 1, seq_len=sh.pos + 1) as ctx:
        for layer in layers:
            k, v, q = decode_inputs(sh, layer)
            got = _gpu_step(ctx, sh, layer, k, v, q)
            want, skipped = _oracle(sh, layer, k, v, q)
            assert skipped == 0
            _check(got, want, f"{name} layer {layer}")


def test_long_context_decode_layer0_matches_oracle():
    sh = CONFIGS["llama31_8b_decode_128k"]
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        got = _gpu_step(ctx, sh, 0, k, v, q)
    want, skipped = _oracle(sh, 0, k, v, q)
    assert skipped == 0
    _check(got, want, "128k layer 0")


def test_gemma_sliding_window_layers():
    sh = GEMMA_SWA
    with AttnContext.for_shape(sh, n_layers=12) as ctx:
        for layer in (0, 4, 5, 6, 11):  # SWA layers 0,4,6 (window 512); full layers 5, 11
            k, v, q = decode_inputs(sh, layer)
            got = _gpu_step(ctx, sh, layer, k, v, q)
            want, _ = _oracle(sh, layer, k, v, q)
            _check(got, want, f"swa layer {layer}")


@pytest.mark.parametrize("shape", [
    AttnShape("pos0", 1, 32, 8, 64, 64, pos=0, seed=31),
    AttnShape("mha_hd128", 1, 8, 8, 128, 777, pos=776, seed=32),
    AttnShape("gqa2_hd256", 1, 4, 2, 256, 700, pos=612, seed=33),
    AttnShape("gqa8_hd64", 1, 16, 2, 64, 333, pos=332, seed=34),
    AttnShape("gqa16_hd128", 1, 32, 2, 128, 129, pos=128, seed=35),
    AttnShape("gqa6_hd64", 1, 12, 2, 64, 95, pos=90, seed=36),
    AttnShape("mqa_hd128_odd", 1, 8, 1, 128, 1001, pos=1000, seed=37),
    AttnShape("window1", 1, 8, 1, 256, 40, pos=37, seed=38, is_gemma3=1, swa_window=1, swa_pattern=6),
    AttnShape("window_gt_pos", 1, 8, 2, 128, 100, pos=20, seed=39, is_gemma3=1, swa_window=64, swa_pattern=6),
])
def test_edge_geometries(shape):
    k, v, q = decode_inputs(shape, 0, ctx=shape.pos + 1)
    with AttnContext.for_shape(shape, n_layers=1) as ctx:
        got = _gpu_step(ctx, shape, 0, k, v, q)
    want, _ = _oracle(shape, 0, k, v, q)
    _check(got, want, shape.name)
    if shape.name == "window1":
        for h in range(shape.n_heads):  # a window of one attends only the current row
            np.testing.assert_allclose(got[h], v[h // shape.kv_mul, shape.pos], rtol=1e-6, atol=1e-6)


def test_append_writes_exact_rows():
    sh = AttnShape("append", 2, 8, 4, 128, 64, pos=17, seed=40)
    k, v, q = decode_inputs(sh, 1, ctx=64)
    with AttnContext.for_shape(sh) as ctx:
        ctx.kv_append(1, 17, np.ascontiguousarray(k[:, 17]), np.ascontiguousarray(v[:, 17]))
        rk, rv = ctx.read_kv(1, 17, 1)
        z, _ = ctx.read_kv(0, 17, 1)
    np.testing.assert_array_equal(rk[:, 0], k[:, 17])
    np.testing.assert_array_equal(rv[:, 0], v[:, 17])
    assert not z.any()


def test_q8_gap_is_the_reference_quantisation_error():
    sh = CONFIGS["llama31_8b_decode_8k"]
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        got = _gpu_step(ctx, sh, 0, k, v, q)
    want_q8, _ = _oracle(sh, 0, k, v, q, O.MODE_Q8)
    _, ma, mr = tolerance_ok(got, want_q8)
    print(f"fp32 kernel vs shipped Q8_0 reference: max_abs={ma:.3e}")
    assert ma < 5e-2


def test_device_entry_points_match_host_entry_points():
    import torch

    sh = CONFIGS["llama32_1b_decode"]
    n_layers = 4
    with AttnContext.for_shape(sh, n_layers=n_layers) as ctx:
        qs, outs_host = [], []
        for layer in range(n_layers):
            k, v, q = decode_inputs(sh, layer)
            outs_host.append(_gpu_step(ctx, sh, layer, k, v, q))
            qs.append(q)
        dq = torch.from_numpy(np.stack(qs)).cuda()
        dout = torch.zeros_like(dq)
        ctx.decode_layers_dev(0, n_layers, sh.pos, dq, dout)
        one = torch.zeros_like(dq[0])
        ctx.decode_dev(2, sh.pos, dq[2].contiguous(), one)
        torch.cuda.synchronize()
        ctx.check()
    got = dout.cpu().numpy()
    for layer in range(n_layers):
        np.testing.assert_allclose(got[layer], outs_host[layer], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(one.cpu().numpy(), outs_host[2], rtol=1e-6, atol=1e-7)


def test_errors_are_reported_not_fatal():
    from llama3pure_b200.attn import AttnError

    sh = AttnShape("err", 2, 8, 2, 128, 32, pos=3, seed=41)
    with AttnContext.for_shape(sh) as ctx:
        q = np.zeros((8, 128), np.float32)
        with pytest.raises(AttnError) as e:
            ctx.decode(0, 32, q)
        assert e.value.code == -2
        with pytest.raises(AttnError) as e:
            ctx.decode(2, 3, q)
        assert e.value.code == -2
        ctx.decode(1, 3, q)  # the context stays usable


@pytest.mark.parametrize("plan", ["1:1", "5:1", "16:1", "16:16", "32:16", "24:8", "8:2", "64:4", "48:1", "79:1",
                                  "128:1"])
@pytest.mark.parametrize("name", ["llama31_8b_decode_8k", "gemma_2b_decode"])
@pytest.mark.parametrize("merge", ["designated", "ticket"])
def test_every_merge_path(monkeypatch, plan, name, merge):
    """Pin the split-K decomposition (single CTA, global merge by designated
    mergers or by the last arriver, cluster merge, cluster + global merge) and
    check each against the oracle."""
    monkeypatch.setenv("L3P_DECODE_PLAN", plan)
    if merge == "ticket":
        monkeypatch.setenv("L3P_DECODE_MERGE", "ticket")
    sh = CONFIGS[name].with_(pos=2047, seq_len=2048)
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        assert ctx.decode_plan(sh.pos) == tuple(int(x) for x in plan.split(":")), "plan not applied"
        got = _gpu_step(ctx, sh, 0, k, v, q)
    want, _ = _oracle(sh, 0, k, v, q)
    _check(got, want, f"{name} plan {plan}")


@pytest.mark.parametrize("plan", ["79:1", "128:1"])
@pytest.mark.parametrize("merge", ["designated", "ticket"])
def test_several_mergers_across_launches(monkeypatch, plan, merge):
    """One KV head split 79 or 128 ways fits one wave: designated mergers
    (two at head_dim 256 with 8 q heads) or the last four parts to finish
    each merge a slice of the output; the unit's flags or ticket must be back
    at zero for every following launch (several positions in a row)."""
    monkeypatch.setenv("L3P_DECODE_PLAN", plan)
    if merge == "ticket":
        monkeypatch.setenv("L3P_DECODE_MERGE", "ticket")
    sh = CONFIGS["gemma_2b_decode"].with_(pos=2047, seq_len=2048)
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1) as ctx:
        ctx.load_kv(0, 0, k, v)
        for pos in (2047, 1500, 2047, 1024):
            got = ctx.decode(0, pos, q)
            want, _ = _oracle(sh.with_(pos=pos), 0, k, v, q)
            _check(got, want, f"plan {plan} pos {pos}")
        ctx.check()


def test_default_plans_are_reported():
    for name in ("llama31_8b_decode_8k", "gemma_2b_decode", "llama32_1b_decode"):
        sh = CONFIGS[name]
        with AttnContext.for_shape(sh, n_layers=1) as ctx:
            ns, cs = ctx.decode_plan(sh.pos)
            print(f"{name}: nsplit={ns} cluster={cs}")
            assert ns >= 1 and cs >= 1 and ns % cs == 0


@pytest.mark.parametrize("use_graph", [False, True])
def test_overlap_mode_consecutive_layers(use_graph):
    """Programmatic dependent launch between the layers of one decode step
    (each launch's predecessor is another layer's attention): same results."""
    import torch

    sh = CONFIGS["llama31_8b_decode_8k"].with_(pos=3000, seq_len=4096)
    n_layers = 6
    stream = torch.cuda.Stream()
    with AttnContext.for_shape(sh, n_layers=n_layers) as ctx:
        qs, ks, vs, wants = [], [], [], []
        for layer in range(n_layers):
            k, v, q = decode_inputs(sh, layer)
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            qs.append(q)
            ks.append(np.ascontiguousarray(k[:, sh.pos]))
            vs.append(np.ascontiguousarray(v[:, sh.pos]))
            wants.append(_oracle(sh, layer, k, v, q)[0])
        dq = torch.from_numpy(np.stack(qs)).cuda()
        dk = torch.from_numpy(np.stack(ks)).cuda()
        dv = torch.from_numpy(np.stack(vs)).cuda()
        out = torch.zeros_like(dq)
        ctx.set_overlap(True)
        torch.cuda.synchronize()

        def run():
            for layer in range(n_layers):
                ctx.step_dev(layer, sh.pos, dq[layer], dk[layer], dv[layer], out[layer], stream)

        if use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run()
            for _ in range(3):
                g.replay()
        else:
            for _ in range(3):
                run()
        torch.cuda.synchronize()
        ctx.check()
    got = out.cpu().numpy()
    for layer in range(n_layers):
        _check(got[layer], wants[layer], f"overlap layer {layer}")

