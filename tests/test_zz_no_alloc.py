"""l3p_attn_decode_noalloc: the decode entry point that allocates nothing.

It exists for callers that own all device memory (one arena planned at model
load) and cannot let a library allocate while generating.  This test calls it
through the C ABI on a cache owned by an ordinary context and checks two
consecutive calls against the existing entry point and against the oracle,
within the decode tests' tolerance (|a - b| <= 1e-4 + 1e-4*|b|).  The cases:
  * 8B at 8K and Gemma MQA at 4K, where the kernel splits every KV head's
    range over many CTAs, so the fixed scratch array (partials and tickets)
    carries the result;
  * a Gemma sliding-window layer (the host computes the window for the split
    plan);
  * a KV-head shard (kv_head_begin > 0, fewer KV heads than the model): the
    cache is indexed by the shard's own heads, q and out by absolute head.

Collected last (file name) so a run that stops at the first failure has
already run every other test.
"""
import numpy as np
import pytest

from llama3pure_b200.attn import AttnContext, decode_noalloc, load_library
from llama3pure_b200.synth import CONFIGS, GEMMA_SWA, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu

CASES = {
    # name: (shape, layer, kv_head_begin, kv_head_count, must split)
    "llama31_8b_decode_8k": (CONFIGS["llama31_8b_decode_8k"], 0, 0, 0, True),
    "gemma_2b_decode": (CONFIGS["gemma_2b_decode"], 0, 0, 0, True),
    "gemma_swa_layer": (GEMMA_SWA, 0, 0, 0, False),  # layer 0 of pattern 6: window of 512 rows
    "llama31_8b_kv_shard": (CONFIGS["llama31_8b_decode_8k"], 0, 2, 3, True),
}


@pytest.mark.parametrize("name", list(CASES))
def test_noalloc_decode_matches_context_decode_and_oracle_twice(name):
    import torch

    import oracle as O

    sh, layer, hb, hc, must_split = CASES[name]
    k, v, q = decode_inputs(sh, layer)
    ref = O.Oracle(sh, O.MODE_F32, "port", n_layers=layer + 1)
    ref.load_kv(layer, 0, k, v)
    want_oracle, _ = ref.decode(layer, sh.pos, q)
    ref.close()
    with AttnContext.for_shape(sh, n_layers=layer + 1, seq_len=sh.pos + 1, kv_head_begin=hb,
                               kv_head_count=hc) as ctx:
        ctx.load_kv(layer, 0, k, v)
        if must_split:
            ns, _ = ctx.decode_plan(sh.pos)
            assert ns > 1, "geometry must split the range (exercises the scratch array)"
        r0, r1 = ctx.owned_rows
        dq = torch.from_numpy(q).cuda()
        want_ctx = torch.zeros_like(dq)
        ctx.decode_dev(layer, sh.pos, dq, want_ctx)
        torch.cuda.synchronize()
        ctx.check()
        kp, vp = ctx.kv_device_ptr(layer)
        outs = []
        for _ in range(2):
            out = torch.full_like(dq, float("nan"))
            decode_noalloc(ctx.cfg, layer, sh.pos, kp, vp, dq, out, lib=load_library())
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
    want_ctx = want_ctx.cpu().numpy()[r0:r1]
    want_oracle = want_oracle.reshape(sh.n_heads, sh.head_dim)[r0:r1]
    for i, got in enumerate(outs):
        got = got[r0:r1]
        ok, ma, mr = tolerance_ok(got, want_ctx)
        assert ok, f"call {i} vs the context decode: max_abs={ma:.3e} max_rel={mr:.3e}"
        ok, ma, mr = tolerance_ok(got, want_oracle)
        assert ok, f"call {i} vs the oracle: max_abs={ma:.3e} max_rel={mr:.3e}"
        assert np.isfinite(got).all()
    if (r0, r1) != (0, sh.n_heads):  # rows of heads the shard does not own stay untouched
        assert np.isnan(np.delete(outs[1], np.s_[r0:r1], axis=0)).all()


def test_noalloc_rejects_oversized_geometry_and_bad_layer():
    from llama3pure_b200.attn import AttnConfig, AttnError

    import torch

    # 2048 (KV head, q-head group) units exceed the 1024 tickets of the array
    cfg = AttnConfig(1, 2048, 2048, 64, 16, 0.0, 0, 0, 0, 0, 0, 0, 0, 0, 0)
    buf = torch.zeros(2048 * 16 * 64, device="cuda")
    q = torch.zeros(2048 * 64, device="cuda")
    with pytest.raises(AttnError) as e:
        decode_noalloc(cfg, 0, 15, buf, buf, q, q)
    assert e.value.code == -2
    # a layer outside [0, n_layers) is rejected like the context entry points do
    cfg = AttnConfig(2, 8, 1, 256, 16, 0.0, 1, 8, 6, 0, 0, 0, 0, 0, 0)
    for layer in (-1, 2):
        with pytest.raises(AttnError) as e:
            decode_noalloc(cfg, layer, 15, buf, buf, q, q)
        assert e.value.code == -2
