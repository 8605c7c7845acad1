"""The host-call server (l3p_attn_set_host_server) against the CPU oracle.

With the server on, l3p_attn_step / l3p_attn_decode hand their rows to a
resident decode grid (one copy of tagged packets into a device inbox) and
poll the mergers' flags in mapped pinned memory for the output.  The contract is the launched path's: |gpu - oracle| <=
1e-4 + 1e-4*|oracle| element-wise, against the reference's attention loop
over an fp32 cache (llama3pure-c-engine.c:3299-3359).  The cases cover the
BASELINE shapes, a KV-head shard (unowned rows untouched), decode without an
append, a run of positions whose split-K plan changes (the server restarts
with the new split), an idle spell long enough for the grid to leave, and the
other entry points of the context stopping and restarting it.
"""
import time

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext, AttnError
from llama3pure_b200.synth import CONFIGS, GEMMA_SWA, AttnShape, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu

ATOL = 1e-4
RTOL = 1e-4


def _check(got, want, what):
    ok, ma, mr = tolerance_ok(got, want, ATOL, RTOL)
    assert ok, f"{what}: max_abs={ma:.3e} max_rel={mr:.3e}"


def _oracle(sh, layer, pos, k, v, q):
    """Reference attention of q at `pos` over rows [0, pos] of k, v ([kvh][seq][hd])."""
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=layer + 1, seq_len=pos + 1)
    o.load_kv(layer, 0, np.ascontiguousarray(k[:, : pos + 1]), np.ascontiguousarray(v[:, : pos + 1]))
    out, skipped = o.decode(layer, pos, q)
    o.close()
    assert skipped == 0
    return out


@pytest.mark.parametrize("name,layers", [
    ("llama32_1b_decode", list(range(16))),
    ("llama31_8b_decode_8k", [0, 1, 31]),
    ("gemma_2b_decode", list(range(18))),
])
def test_server_steps_match_oracle(name, layers):
    """Every layer's cache loaded first, then the steps back to back: one
    resident grid serves them all."""
    sh = CONFIGS[name]
    inputs = {layer: decode_inputs(sh, layer) for layer in layers}
    with AttnContext.for_shape(sh, n_layers=max(layers) + 1, seq_len=sh.pos + 1) as ctx:
        for layer, (k, v, q) in inputs.items():
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
        ctx.set_host_server(True)
        n0 = ctx.launch_count()
        got = {layer: ctx.step(layer, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))
               for layer, (k, v, q) in inputs.items()}
        launches = ctx.launch_count() - n0
        ctx.set_host_server(False)
        # the cache holds the appended rows
        for layer, (k, v, q) in inputs.items():
            kk, vv = ctx.read_kv(layer, sh.pos, 1)
            np.testing.assert_array_equal(kk[:, 0], k[:, sh.pos])
            np.testing.assert_array_equal(vv[:, 0], v[:, sh.pos])
    assert launches == 1, f"{launches} launches for {len(layers)} served calls"
    for layer, (k, v, q) in inputs.items():
        _check(got[layer], _oracle(sh, layer, sh.pos, k, v, q), f"{name} layer {layer}")


def test_server_matches_launched_path():
    """Same calls with and without the server: equal within the summation-order noise."""
    sh = CONFIGS["llama31_8b_decode_8k"]
    k, v, q = decode_inputs(sh, 0)
    outs = []
    for server in (False, True):
        with AttnContext.for_shape(sh, n_layers=1, seq_len=sh.pos + 1) as ctx:
            ctx.load_kv(0, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            if server:
                ctx.set_host_server(True)
            outs.append(ctx.step(0, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos])))
    np.testing.assert_allclose(outs[1], outs[0], rtol=1e-5, atol=1e-6)


def test_server_kv_head_shard_writes_owned_rows_only():
    sh = CONFIGS["llama31_8b_decode_8k"]
    k, v, q = decode_inputs(sh, 2)
    begin, count = 2, 3
    with AttnContext.for_shape(sh, n_layers=3, seq_len=sh.pos + 1, kv_head_begin=begin, kv_head_count=count) as ctx:
        ctx.load_kv(2, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
        ctx.set_host_server(True)
        out = np.full((sh.n_heads, sh.head_dim), np.nan, np.float32)
        ctx.step(2, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]), out=out)
    want = _oracle(sh, 2, sh.pos, k, v, q)
    r0, r1 = begin * sh.kv_mul, (begin + count) * sh.kv_mul
    _check(out[r0:r1], want[r0:r1], "kv shard rows")
    assert np.isnan(out[:r0]).all() and np.isnan(out[r1:]).all()


def test_server_decode_without_append():
    sh = GEMMA_SWA
    with AttnContext.for_shape(sh, n_layers=6) as ctx:
        cases = []
        for layer in (0, 5):  # a sliding-window layer and a full one
            k, v, q = decode_inputs(sh, layer)
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos + 1]), np.ascontiguousarray(v[:, : sh.pos + 1]))
            cases.append((layer, k, v, q))
        ctx.set_host_server(True)
        got = [ctx.decode(layer, sh.pos, q) for layer, k, v, q in cases]
    for (layer, k, v, q), g in zip(cases, got):
        _check(g, _oracle(sh, layer, sh.pos, k, v, q), f"swa decode layer {layer}")


def test_server_position_run_replans():
    """Steps at positions 0 .. 600 on one layer, the cache built by the steps
    themselves: the split-K plan grows with the range and the server restarts
    with each new split."""
    sh = AttnShape("run", 1, 32, 8, 128, 601, pos=600, seed=77)
    k, v, q = decode_inputs(sh, 0)
    checks = {0, 1, 7, 8, 63, 255, 600}
    got = {}
    with AttnContext.for_shape(sh, n_layers=1, seq_len=601) as ctx:
        ctx.set_host_server(True)
        n0 = ctx.launch_count()
        for p in range(601):
            o = ctx.step(0, p, q, np.ascontiguousarray(k[:, p]), np.ascontiguousarray(v[:, p]))
            if p in checks:
                got[p] = o
        restarts = ctx.launch_count() - n0
        plans = [ctx.decode_plan(p)[0] for p in range(601)]
    for p in sorted(checks):
        _check(got[p], _oracle(sh, 0, p, k, v, q), f"position {p}")
    # a new grid only where the split changes (the server's split is the
    # plan's, capped so that the grid is resident at once)
    changes = sum(a != b for a, b in zip(plans, plans[1:]))
    assert 1 < restarts <= changes + 1


def test_server_leaves_when_idle_and_comes_back():
    sh = CONFIGS["llama32_1b_decode"]
    with AttnContext.for_shape(sh, n_layers=2, seq_len=sh.pos + 1) as ctx:
        ctx.set_host_server(True, idle_us=2000)
        outs = []
        for layer in (0, 1, 0):
            k, v, q = decode_inputs(sh, layer)
            ctx.load_kv(layer, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
            n0 = ctx.launch_count()
            time.sleep(0.02)  # ten idle limits: the grid started by the last call has left
            outs.append((layer, k, v, q, ctx.step(layer, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]),
                                                 np.ascontiguousarray(v[:, sh.pos])), ctx.launch_count() - n0))
            time.sleep(0.02)
            # a call after the grid left on its own: started again, same result
            again = ctx.step(layer, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))
            np.testing.assert_array_equal(again, outs[-1][4])
        ctx.check()
    for layer, k, v, q, out, launches in outs:
        assert launches == 1
        _check(out, _oracle(sh, layer, sh.pos, k, v, q), f"idle layer {layer}")


def test_other_entry_points_stop_the_server():
    """A device-side entry point between served calls: the grid is ended
    first, the call runs, the next host call starts a new grid."""
    sh = CONFIGS["llama31_8b_decode_8k"]
    k0, v0, q0 = decode_inputs(sh, 0)
    k1, v1, q1 = decode_inputs(sh, 1)
    with AttnContext.for_shape(sh, n_layers=2, seq_len=sh.pos + 1) as ctx:
        ctx.load_kv(0, 0, np.ascontiguousarray(k0[:, : sh.pos]), np.ascontiguousarray(v0[:, : sh.pos]))
        ctx.set_host_server(True)
        a = ctx.step(0, sh.pos, q0, np.ascontiguousarray(k0[:, sh.pos]), np.ascontiguousarray(v0[:, sh.pos]))
        # launched entry points while the server is on
        ctx.load_kv(1, 0, np.ascontiguousarray(k1[:, : sh.pos]), np.ascontiguousarray(v1[:, : sh.pos]))
        b_launched = ctx.prefill(1, sh.pos, np.ascontiguousarray(q1[None]), np.ascontiguousarray(k1[:, sh.pos][None]),
                                 np.ascontiguousarray(v1[:, sh.pos][None]))[0]
        b = ctx.decode(1, sh.pos, q1)  # served again
        ctx.set_host_server(False)
        c = ctx.decode(0, sh.pos, q0)  # launched
    _check(a, _oracle(sh, 0, sh.pos, k0, v0, q0), "served step")
    want1 = _oracle(sh, 1, sh.pos, k1, v1, q1)
    _check(b_launched, want1, "prefill between served calls")
    _check(b, want1, "served decode after a prefill")
    _check(c, a, "launched decode after the server")


def test_server_refuses_q8_cache_and_sequence_shards():
    sh = CONFIGS["llama32_1b_decode"]
    with AttnContext.for_shape(sh, n_layers=1, seq_len=sh.pos + 1, kv_format=1) as ctx:
        with pytest.raises(AttnError):
            ctx.set_host_server(True)
    with AttnContext.for_shape(sh, n_layers=1, seq_len=sh.pos + 1, seq_begin=512, seq_count=512) as ctx:
        with pytest.raises(AttnError):
            ctx.set_host_server(True)
