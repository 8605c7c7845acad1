"""The reference C engine wired to libllama3pure_attn.so (the engine
maintainer's integration, built by tests/engine/Makefile where the reference
source is).

The reference engine's own forward pass (transformer_prefill + transformer,
llama3pure-c-engine.c:3190, c:3439) runs twice on the same synthetic Q8_0
model: once as shipped, once with its attention blocks (c:3232-3359,
c:3495-3613) replaced by l3p_attn_step_raw / l3p_attn_prefill_raw on the
GPU.  Greedy generations must be identical and every position's logits equal
within 2e-3 of the largest logit: the attention inputs are bit-identical
(the library's RoPE, QK-norm and Q8_0 quantiser are the reference's bits);
only the attention's float summation order and exp differ, and their
last-bit differences grow a little through the later layers.
"""
import numpy as np
import pytest

import engines as E


@pytest.mark.skipif(not E.available(False), reason="engine build absent (needs the reference source where built)")
def test_reference_engine_harness_runs_deterministically():
    e = E.Engine(False)
    a = e.run("llama_hd64", E.prompt_for("llama_hd64", 40), 4)
    b = e.run("llama_hd64", E.prompt_for("llama_hd64", 40), 4)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    assert np.all(np.isfinite(a[1])) and float(a[1].std()) > 0.1


@pytest.mark.gpu
@pytest.mark.skipif(not (E.available(False) and E.available(True)),
                    reason="engine builds absent (need the reference source where built)")
@pytest.mark.parametrize("model", list(E.MODELS))
def test_wired_engine_generates_what_the_reference_engine_generates(model):
    prompt = E.prompt_for(model, 70)
    want_tok, want = E.Engine(False).run(model, prompt, 8)
    got_tok, got = E.Engine(True).run(model, prompt, 8)
    err = float(np.abs(got - want).max())
    scale = float(np.abs(want).max())
    assert err <= 2e-3 * scale, f"{model}: max |logit diff| {err:.3e} (largest logit {scale:.3f})"
    np.testing.assert_array_equal(got_tok, want_tok)
