"""l3p_attn_decode_noalloc: the decode entry point that allocates nothing.

It exists for callers that own all device memory (one arena planned at model
load) and cannot let a library allocate while generating.  This test calls it
through the C ABI on a cache owned by an ordinary context and checks two
consecutive calls against the existing entry point, within the decode tests'
tolerance (|a - b| <= 1e-4 + 1e-4*|b|).  The geometries chosen make the
kernel split every KV head's range over many CTAs, so the fixed scratch array
(partials and tickets) is what carries the result.

Collected last (file name) so a run that stops at the first failure has
already run every other test.
"""
import numpy as np
import pytest

from llama3pure_b200.attn import AttnContext, decode_noalloc, load_library
from llama3pure_b200.synth import CONFIGS, decode_inputs, tolerance_ok

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["llama31_8b_decode_8k", "gemma_2b_decode"])
def test_noalloc_decode_matches_context_decode_twice(name):
    import torch

    sh = CONFIGS[name]
    k, v, q = decode_inputs(sh, 0)
    with AttnContext.for_shape(sh, n_layers=1, seq_len=sh.pos + 1) as ctx:
        ctx.load_kv(0, 0, k, v)
        ns, _ = ctx.decode_plan(sh.pos)
        assert ns > 1, "geometry must split the range (exercises the scratch array)"
        dq = torch.from_numpy(q).cuda()
        ref = torch.zeros_like(dq)
        ctx.decode_dev(0, sh.pos, dq, ref)
        torch.cuda.synchronize()
        ctx.check()
        kp, vp = ctx.kv_device_ptr(0)
        outs = []
        for _ in range(2):
            out = torch.full_like(dq, float("nan"))
            decode_noalloc(ctx.cfg, 0, sh.pos, kp, vp, dq, out, lib=load_library())
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
    want = ref.cpu().numpy()
    for i, got in enumerate(outs):
        ok, ma, mr = tolerance_ok(got, want)
        assert ok, f"call {i}: max_abs={ma:.3e} max_rel={mr:.3e}"
    assert np.isfinite(outs[1]).all()


def test_noalloc_rejects_oversized_geometry():
    from llama3pure_b200.attn import AttnConfig, AttnError

    import torch

    # 2048 (KV head, q-head group) units exceed the 1024 tickets of the array
    cfg = AttnConfig(1, 2048, 2048, 64, 16, 0.0, 0, 0, 0, 0, 0, 0, 0, 0, 0)
    buf = torch.zeros(2048 * 16 * 64, device="cuda")
    q = torch.zeros(2048 * 64, device="cuda")
    with pytest.raises(AttnError) as e:
        decode_noalloc(cfg, 0, 15, buf, buf, q, q)
    assert e.value.code == -2
