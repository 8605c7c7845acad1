"""The wo projection on the GPU (the attention output's consumer) through the C ABI.

wo_gemv_kernel must equal the reference's matmul_quantized
(llama3pure-c-engine.c:2091-2176: dequantised weight rows, fp32 dots) for
Q8_0, Q4_K and Q6_K weights within |gpu - ref| <= 1e-4 + 1e-4*|ref|: the
products are the reference's, only the summation order differs.  The oracle's
matvec is pinned bit for bit to the reference by tests/golden/wo_golden.npz.
"""
import os

import numpy as np
import pytest

import oracle as O
from llama3pure_b200.attn import AttnContext, AttnError
from llama3pure_b200.synth import CONFIGS, GEMMA_SWA, raw_qkv_inputs, tolerance_ok, wo_input, wo_weights

pytestmark = pytest.mark.gpu

WO_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "wo_golden.npz")
TYPES = {"q8_0": O.W_Q8_0, "q2_k": O.W_Q2_K, "q3_k": O.W_Q3_K, "q4_k": O.W_Q4_K, "q5_k": O.W_Q5_K,
         "q6_k": O.W_Q6_K, "q4_0": O.W_Q4_0, "q4_1": O.W_Q4_1, "q5_0": O.W_Q5_0, "q5_1": O.W_Q5_1,
         "iq4_nl": O.W_IQ4_NL, "f32": O.W_F32, "f16": O.W_F16, "bf16": O.W_BF16}
SHAPES = {
    "l8b": CONFIGS["llama31_8b_decode_8k"].with_(seq_len=64, n_layers=2),       # 4096 x 4096
    "l1b": CONFIGS["llama32_1b_decode"].with_(seq_len=64, n_layers=2),          # 2048 x 2048
    "gemma": CONFIGS["gemma_2b_decode"].with_(seq_len=64, n_layers=2),          # 2048 x 2048 (hd 256)
}
DIMS = {"l8b": 4096, "l1b": 2048, "gemma": 2048}


def _torch():
    import torch

    return torch


def _check(got, want, what):
    ok, ma, mr = tolerance_ok(got, want)
    assert ok, f"{what}: max_abs={ma:.3e} max_rel={mr:.3e}"


@pytest.mark.parametrize("name", [str(n) for n in np.load(WO_GOLDEN)["cases"]])
def test_wo_matches_reference_golden(name):
    """Against the reference's own outputs: a context whose q_dim is the
    case's column count (heads of 128), dim = the case's rows."""
    torch = _torch()
    g = np.load(WO_GOLDEN)
    wt, rows, cols, seed = [int(v) for v in g[f"{name}/geom"]]
    w = wo_weights(wt, rows, cols, seed)
    x = wo_input(cols, seed)
    with AttnContext(1, cols // 128, cols // 128, 128, 16) as ctx:
        ctx.set_wo(0, wt, w)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full((rows,), float("nan"), device="cuda")
        ctx.wo_dev(0, dx, dy)
        ctx.check()
        got = dy.cpu().numpy()
        _check(got, g[f"{name}/out"], name)
        _check(ctx.wo(0, x), g[f"{name}/out"], name + " host")


@pytest.mark.parametrize("tname", list(TYPES))
@pytest.mark.parametrize("sname", list(SHAPES))
def test_wo_model_shapes(sname, tname):
    torch = _torch()
    sh, dim, wt = SHAPES[sname], DIMS[sname], TYPES[tname]
    cols = sh.n_heads * sh.head_dim
    w = wo_weights(wt, dim, cols, seed=11)
    x = wo_input(cols, seed=12)
    want = O.matvec(wt, w, dim, cols, x)
    with AttnContext.for_shape(sh) as ctx:
        ctx.set_wo(1, wt, w)
        dx = torch.from_numpy(x).cuda()
        dy = torch.zeros(dim, device="cuda")
        ctx.wo_dev(1, dx, dy)
        ctx.check()
        _check(dy.cpu().numpy(), want, f"{sname} {tname}")


@pytest.mark.parametrize("tname", list(TYPES))
@pytest.mark.parametrize("n_shards", [2, 4, 8])
def test_wo_head_shards_sum_to_the_whole(n_shards, tname):
    """Tensor parallelism by head: each context holds the columns of its q
    heads; the partial outputs add up to the full projection."""
    torch = _torch()
    sh, dim, wt = SHAPES["l8b"], DIMS["l8b"], TYPES[tname]
    cols = sh.n_heads * sh.head_dim
    w = wo_weights(wt, dim, cols, seed=21)
    x = wo_input(cols, seed=22)
    want = O.matvec(wt, w, dim, cols, x)
    per = sh.n_kv_heads // n_shards
    total = np.zeros(dim, np.float64)
    for r in range(n_shards):
        with AttnContext.for_shape(sh, kv_head_begin=r * per, kv_head_count=per) as ctx:
            ctx.set_wo(0, wt, w)
            dx = torch.from_numpy(x).cuda()
            dy = torch.zeros(dim, device="cuda")
            ctx.wo_dev(0, dx, dy)
            ctx.check()
            total += dy.cpu().numpy()
            # the shard's own columns only
            c0, c1 = r * per * sh.kv_mul * sh.head_dim, (r + 1) * per * sh.kv_mul * sh.head_dim
            xs = np.zeros_like(x)
            xs[c0:c1] = x[c0:c1]
            _check(dy.cpu().numpy(), O.matvec(wt, w, dim, cols, xs), f"shard {r}/{n_shards}")
    _check(total, want, f"sum of {n_shards} shards")


@pytest.mark.parametrize("n_kv,G,hd", [(3, 4, 64), (1, 4, 64), (5, 2, 128), (3, 8, 128)])
def test_wo_q8_0_owned_columns_not_a_slice_multiple(n_kv, G, hd):
    """Owned column counts that end inside a 1024-value slice (768, 256,
    1280, 3072): the lanes past the end read nothing."""
    torch = _torch()
    cols, dim = n_kv * G * hd, 384
    w = wo_weights(O.W_Q8_0, dim, cols, seed=cols)
    x = wo_input(cols, seed=7)
    with AttnContext(1, n_kv * G, n_kv, hd, 16) as ctx:
        ctx.set_wo(0, O.W_Q8_0, w)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full((dim,), float("nan"), device="cuda")
        ctx.wo_dev(0, dx, dy)
        ctx.check()
        _check(dy.cpu().numpy(), O.matvec(O.W_Q8_0, w, dim, cols, x), f"{cols} columns")


@pytest.mark.parametrize("tname", list(TYPES))
def test_wo_wide_rows_use_eight_column_groups(tname):
    """8192 owned columns (64 heads of 128): eight slices of Q8_0/Q4_K, four
    of Q6_K, i.e. the 8-warp CTAs."""
    torch = _torch()
    cols, dim, wt = 8192, 300, TYPES[tname]
    w = wo_weights(wt, dim, cols, seed=77)
    x = wo_input(cols, seed=78)
    with AttnContext(1, 64, 8, 128, 16) as ctx:
        ctx.set_wo(0, wt, w)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full((dim,), float("nan"), device="cuda")
        ctx.wo_dev(0, dx, dy)
        ctx.check()
        _check(dy.cpu().numpy(), O.matvec(wt, w, dim, cols, x), f"{tname} 8192 columns")


@pytest.mark.parametrize("tname", ["q8_0", "q6_k"])
@pytest.mark.parametrize("sname", ["l8b", "gemma"])
def test_step_raw_wo_is_the_engines_block(sname, tname):
    """QK-norm/RoPE, cache write, attention and wo in one host call against the
    oracle's chain (rope -> attention -> matvec)."""
    sh = SHAPES[sname].with_(seq_len=300) if sname == "l8b" else GEMMA_SWA.with_(seq_len=300, n_layers=6,
                                                                                    swa_window=64)
    layer = 1 if sname == "l8b" else 5
    dim, wt = DIMS[sname], TYPES[tname]
    hd, hkv = sh.head_dim, sh.n_kv_heads
    cols = sh.n_heads * hd
    pos = 290
    rng = np.random.default_rng(5)
    hk = rng.standard_normal((hkv, pos, hd)).astype(np.float32)
    hv = rng.standard_normal((hkv, pos, hd)).astype(np.float32)
    q, k, v, qn, kn = raw_qkv_inputs(sh, layer, 1)
    norm = bool(sh.is_gemma3)
    th, th_swa, eps = (1e6, 1e4, 1e-6) if norm else (5e5, 0.0, 0.0)
    qr, kr = O.rope(sh, layer, pos, q, k, th, th_swa, eps, qn if norm else None, kn if norm else None,
                    n_layers=sh.n_layers)
    o = O.Oracle(sh, O.MODE_F32, "port", n_layers=layer + 1)
    o.load_kv(layer, 0, hk, hv)
    att, _ = o.decode(layer, pos, qr.reshape(-1), kr.reshape(-1).copy(), v.reshape(-1).copy())
    o.close()
    w = wo_weights(wt, dim, cols, seed=31)
    want = O.matvec(wt, w, dim, cols, np.ascontiguousarray(att.reshape(-1)))
    with AttnContext.for_shape(sh) as ctx:
        ctx.set_rope(th, th_swa, eps, qn if norm else None, kn if norm else None)
        ctx.set_wo(layer, wt, w)
        ctx.load_kv(layer, 0, hk, hv)
        got = ctx.step_raw_wo(layer, pos, q[0].copy(), k[0].copy(), v[0].copy())
    _check(got, want, f"{sname} {tname}")


def test_wo_after_decode_in_a_graph_with_overlap():
    """decode -> wo with programmatic dependent launch inside a CUDA graph: the
    wo kernel prefetches weights before its wait and reads x after it."""
    torch = _torch()
    sh = CONFIGS["llama31_8b_decode_8k"].with_(seq_len=2048, n_layers=4)
    dim, wt = 4096, O.W_Q8_0
    cols = sh.n_heads * sh.head_dim
    pos = 2047
    rng = np.random.default_rng(8)
    with AttnContext.for_shape(sh) as ctx:
        ws = []
        for layer in range(sh.n_layers):
            hk = rng.standard_normal((sh.n_kv_heads, pos + 1, sh.head_dim)).astype(np.float32)
            hv = rng.standard_normal((sh.n_kv_heads, pos + 1, sh.head_dim)).astype(np.float32)
            ctx.load_kv(layer, 0, hk, hv)
            w = wo_weights(wt, dim, cols, seed=40 + layer)
            ctx.set_wo(layer, wt, w)
            ws.append(w)
        q = torch.randn(sh.n_layers, cols, device="cuda")
        att = torch.zeros(sh.n_layers, cols, device="cuda")
        y = torch.zeros(sh.n_layers, dim, device="cuda")
        ctx.set_overlap(True)
        s = torch.cuda.Stream()
        ctx.set_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for layer in range(sh.n_layers):
                    ctx.decode_dev(layer, pos, q[layer], att[layer], s)
                    ctx.wo_dev(layer, att[layer], y[layer], s)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        ctx.check()
        a, yy = att.cpu().numpy(), y.cpu().numpy()
        for layer in range(sh.n_layers):
            _check(yy[layer], O.matvec(wt, ws[layer], dim, cols, np.ascontiguousarray(a[layer])), f"layer {layer}")
        del g


def test_wo_errors():
    sh = CONFIGS["llama32_1b_decode"].with_(seq_len=16, n_layers=1)
    with AttnContext.for_shape(sh) as ctx:
        with pytest.raises(AttnError) as e:
            ctx.wo(0, np.zeros(2048, np.float32))
        assert e.value.code == -1  # set_wo not called
        with pytest.raises(AttnError) as e:
            ctx.set_wo(0, 9, np.zeros((4, 2048 // 32 * 36), np.uint8))  # Q8_1: no matmul path in the reference
        assert e.value.code == -6
    # hd 64, one KV head of 4 q heads owns columns [256, 512): whole Q4_K blocks
    with AttnContext.for_shape(sh, kv_head_begin=1, kv_head_count=1) as ctx:
        ctx.set_wo(0, O.W_Q4_K, wo_weights(O.W_Q4_K, 8, 2048, seed=1))
    # 2 heads of 64 = 128 columns: not a whole 256-value Q4_K block
    with AttnContext(1, 2, 2, 64, 16) as ctx:
        with pytest.raises(AttnError) as e:
            ctx.set_wo(0, O.W_Q4_K, np.zeros((8, 144), np.uint8))
        assert e.value.code == -6
