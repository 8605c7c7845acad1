"""Wire libllama3pure_attn.so into the reference C engine (test infrastructure).

Reads llama3pure-c-engine.c where it lies and writes a copy in which the
engine's attention blocks call the library, the integration an engine
maintainer makes:

  transformer()          c:3232-3359 (QK-norm, RoPE, cache write, attention)
                         -> l3p_attn_step_raw
  transformer_prefill()  c:3495-3613 (the same, token by token)
                         -> l3p_attn_prefill_raw

plus a few helper functions inserted before transformer() (c:3188).  Nothing
of the reference is stored in this repository: the copy is written into
oracle/_ref/ (git-ignored) at build time, and the line numbers are guarded by
the SHA-256 of the source they apply to.

    python tests/engine/wire_engine.py <llama3pure-c-engine.c> <out.c>
"""
from __future__ import annotations

import hashlib
import sys

REF_SHA256 = "7991d405df63b8e2fc07637bd39ccd0044d208a2e86004f9d3b7ef8523d9cd7d"

HELPERS = r"""
/* ---- libllama3pure_attn wiring (inserted before transformer()) ---- */
#include "llama3pure_attn.h"

static l3p_attn_ctx* l3p_wired_ctx = NULL;

/* The context for this model, created on first use: the engine's geometry
 * (Config, RunState), its RoPE parameters and Gemma3 QK-norm weights.  The
 * cache format follows L3P_WIRED_KV_FORMAT (default the engine's own Q8_0). */
static l3p_attn_ctx* l3p_wired_get(Config* p, RunState* s, TransformerWeights* w) {
    if (l3p_wired_ctx) return l3p_wired_ctx;
    l3p_attn_config c;
    memset(&c, 0, sizeof(c));
    c.n_layers = p->n_layers;
    c.n_heads = p->n_heads;
    c.n_kv_heads = p->n_kv_heads;
    c.head_dim = s->head_size;
    c.seq_len = p->seq_len;
    c.scale = 0.0f; /* the library's 1/sqrtf(head_dim), the engine's attn_scale */
    c.is_gemma3 = p->is_gemma3;
    c.swa_window = p->swa_window;
    c.swa_pattern = p->swa_pattern;
    c.device = 0;
    c.kv_format = L3P_KV_Q8_0;
    const char* fmt = getenv("L3P_WIRED_KV_FORMAT");
    if (fmt && strcmp(fmt, "f32") == 0) c.kv_format = L3P_KV_F32;
    if (l3p_attn_create(&c, &l3p_wired_ctx) != L3P_OK) {
        fprintf(stderr, "l3p_attn_create failed\n");
        exit(1);
    }
    l3p_attn_rope_config r;
    memset(&r, 0, sizeof(r));
    r.rope_theta = p->rope_theta;
    r.rope_theta_swa = p->rope_theta_swa;
    r.rms_norm_eps = p->rms_norm_eps;
    r.q_norm = w->attn_q_norm;
    r.k_norm = w->attn_k_norm;
    if (l3p_attn_set_rope(l3p_wired_ctx, &r) != L3P_OK) {
        fprintf(stderr, "l3p_attn_set_rope: %s\n", l3p_attn_last_error(l3p_wired_ctx));
        exit(1);
    }
    return l3p_wired_ctx;
}

void l3p_wired_reset(void) {
    l3p_attn_destroy(l3p_wired_ctx);
    l3p_wired_ctx = NULL;
}

/* c:3232-3359 of transformer(): s->q, s->k, s->v -> s->xb */
static void l3p_wired_step(Config* p, RunState* s, TransformerWeights* w, int l, int pos) {
    l3p_attn_ctx* ctx = l3p_wired_get(p, s, w);
    if (l3p_attn_step_raw(ctx, l, pos, s->q, s->k, s->v, s->xb) != L3P_OK) {
        fprintf(stderr, "l3p_attn_step_raw: %s\n", l3p_attn_last_error(ctx));
        exit(1);
    }
}

/* c:3495-3613 of transformer_prefill(): bq, bk, bv -> bxb (row stride max_dim) */
static void l3p_wired_prefill(Config* p, RunState* s, TransformerWeights* w, int l, int start_pos, int n,
                              float* bq, float* bk, float* bv, float* bxb) {
    l3p_attn_ctx* ctx = l3p_wired_get(p, s, w);
    float* out = bxb;
    if (s->max_dim != s->q_dim) out = (float*)malloc((size_t)n * s->q_dim * sizeof(float));
    if (!out || l3p_attn_prefill_raw(ctx, l, start_pos, n, bq, bk, bv, out) != L3P_OK) {
        fprintf(stderr, "l3p_attn_prefill_raw: %s\n", out ? l3p_attn_last_error(ctx) : "out of memory");
        exit(1);
    }
    if (out != bxb) {
        for (int b = 0; b < n; b++) memcpy(bxb + (size_t)b * s->max_dim, out + (size_t)b * s->q_dim, s->q_dim * sizeof(float));
        free(out);
    }
}
/* ---- end of wiring helpers ---- */

"""

DECODE = "        l3p_wired_step(p, s, w, l, pos);  /* libllama3pure_attn: c:3232-3359 */\n"
PREFILL = ("        l3p_wired_prefill(p, s, w, l, start_pos, batch_size, bq, bk, bv, bxb);"
           "  /* libllama3pure_attn: c:3495-3613 */\n")


def wire(src: str, out: str) -> None:
    data = open(src, "rb").read()
    digest = hashlib.sha256(data).hexdigest()
    if digest != REF_SHA256:
        sys.exit(f"{src}: SHA-256 {digest} is not the engine these line numbers were taken from")
    lines = data.decode("utf-8").splitlines(keepends=True)
    # edits from the bottom up so earlier line numbers stay valid (1-based, inclusive)
    lines[3495 - 1:3613] = [PREFILL]
    lines[3232 - 1:3359] = [DECODE]
    lines[3188 - 1:3188 - 1] = [HELPERS]
    with open(out, "w") as f:
        f.write("".join(lines))


if __name__ == "__main__":
    if len(sys.argv) != 3:
        sys.exit(__doc__)
    wire(sys.argv[1], sys.argv[2])
