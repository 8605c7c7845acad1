/*
 * ref_harness.c -- drives the REFERENCE's own attention primitives.
 *
 * TEST INFRASTRUCTURE ONLY.  This file compiles llama3pure-c-engine.c from
 * where it lies (path passed as -DL3P_REF_ENGINE=... by oracle/Makefile; the
 * engine source is never copied into this repository) with its main()
 * renamed, and exposes the l3pref_* interface of l3p_oracle.h.  The output
 * goes to oracle/_ref/ (git-ignored).  It serves two purposes:
 *   1. it pins the plain-C restatement (l3p_oracle.c) bit-for-bit and
 *      generates the golden vectors in tests/golden/;
 *   2. built with the reference's own OpenMP flags (Makefile:33) it is the
 *      timed CPU baseline ("kind": "reference") of bench.py.
 *
 * The reference has no attention function (attention is inlined in
 * transformer() and transformer_prefill()), so the loop below re-creates only
 * the control flow of c:3299-3359 (decode) and c:3562-3612 (prefill) and
 * calls the reference's own static functions for every arithmetic step:
 *   quantize_to_q8_0_cache (c:1535), dot_q8_0_q8_0_cache (c:1574),
 *   accum_q8_0_cache (c:1600), softmax (c:3167), vec_dot_f32 (c:1487),
 *   init_fp16_table / fp16_to_fp32 / fp32_to_fp16 (c:545-599),
 *   malloc_run_state (c:346) for the Q8_0 cache, attn_scale and GQA tables.
 * RoPE is outside the boundary: q arrives post-RoPE and is multiplied by
 * attn_scale exactly where the reference's RoPE loop would (c:3264, c:3288).
 */
#define main llama3pure_main
#include L3P_REF_ENGINE
#undef main

#include "l3p_oracle.h"

#define L3P_EXPORT __attribute__((visibility("default")))

typedef struct {
    Config p;
    RunState s;
    int mode;
    float scale;
    float** kf; /* fp32 caches [Hkv][seq_len][hd] per layer (f32 mode only) */
    float** vf;
} rctx;

static int g_fp16_ready = 0;

static void ensure_fp16(void) {
    if (!g_fp16_ready) {
        init_fp16_table();
        g_fp16_ready = 1;
    }
}

L3P_EXPORT void* l3pref_create(const l3p_oracle_cfg* cfg, int mode) {
    if (!cfg || cfg->head_dim % QK8_0 != 0 || cfg->n_heads % cfg->n_kv_heads != 0) return NULL;
    ensure_fp16();
    rctx* r = (rctx*)calloc(1, sizeof(rctx));
    r->mode = mode;
    Config* p = &r->p;
    p->n_layers = cfg->n_layers;
    p->n_heads = cfg->n_heads;
    p->n_kv_heads = cfg->n_kv_heads;
    p->head_dim = cfg->head_dim;
    p->dim = cfg->n_heads * cfg->head_dim;
    p->hidden_dim = 32;
    p->vocab_size = 1;
    p->seq_len = cfg->seq_len;
    p->rope_theta = 500000.0f;
    p->is_gemma3 = cfg->is_gemma3;
    p->swa_window = cfg->swa_window;
    p->swa_pattern = cfg->swa_pattern;
    p->rope_theta_swa = 10000.0f;
    malloc_run_state(&r->s, p);
    r->scale = cfg->scale != 0.0f ? cfg->scale : r->s.attn_scale;
    if (mode == L3P_MODE_F32) {
        r->kf = (float**)calloc((size_t)p->n_layers, sizeof(float*));
        r->vf = (float**)calloc((size_t)p->n_layers, sizeof(float*));
    }
    return r;
}

L3P_EXPORT void l3pref_destroy(void* ctx) {
    rctx* r = (rctx*)ctx;
    if (!r) return;
    if (r->kf)
        for (int l = 0; l < r->p.n_layers; ++l) {
            free(r->kf[l]);
            free(r->vf[l]);
        }
    free(r->kf);
    free(r->vf);
    free_run_state(&r->s);
    free(r);
}

static int ensure_f32_layer(rctx* r, int l) {
    size_t n = (size_t)r->p.n_kv_heads * r->p.seq_len * r->s.head_size;
    if (!r->kf[l]) r->kf[l] = (float*)calloc(n, sizeof(float));
    if (!r->vf[l]) r->vf[l] = (float*)calloc(n, sizeof(float));
    return r->kf[l] && r->vf[l];
}

/* One head row into the cache at (layer, kv head, pos): the Q8_0 write of
 * c:3302-3308, or a plain copy into the fp32 cache. */
static void put_row(rctx* r, int l, int kh, int pos, const float* kr, const float* vr) {
    RunState* s = &r->s;
    int hs = s->head_size;
    if (r->mode == L3P_MODE_F32) {
        size_t off = ((size_t)kh * r->p.seq_len + pos) * hs;
        memcpy(r->kf[l] + off, kr, hs * sizeof(float));
        memcpy(r->vf[l] + off, vr, hs * sizeof(float));
    } else {
        size_t off = (size_t)l * s->kv_cache_layer_size + kh * s->head_seq_bytes +
                     (size_t)pos * s->head_q8_bytes;
        quantize_to_q8_0_cache(kr, s->key_cache + off, hs);
        quantize_to_q8_0_cache(vr, s->value_cache + off, hs);
    }
}

L3P_EXPORT int l3pref_load_kv(void* ctx, int layer, int pos0, int n_pos, const float* k,
                              const float* v) {
    rctx* r = (rctx*)ctx;
    if (!r || layer < 0 || layer >= r->p.n_layers || pos0 < 0 || pos0 + n_pos > r->p.seq_len)
        return -2;
    if (r->mode == L3P_MODE_F32 && !ensure_f32_layer(r, layer)) return -4;
    int hs = r->s.head_size;
    for (int h = 0; h < r->p.n_kv_heads; ++h)
        for (int t = 0; t < n_pos; ++t) {
            size_t src = ((size_t)h * n_pos + t) * hs;
            put_row(r, layer, h, pos0 + t, k + src, v + src);
        }
    return 0;
}

static inline void accum_f32_ref(float* out, const float* v, float w, int n) {
    /* fp32 form of accum_q8_0_cache: same |w| < 1e-8 skip (c:1602) */
    if (w > -1e-8f && w < 1e-8f) return;
    for (int i = 0; i < n; ++i) out[i] += w * v[i];
}

/* Attention for one token: c:3310-3359 (parallel=1, the decode path with its
 * `omp parallel for` over KV heads at c:3327-3328) or c:3569-3612
 * (parallel=0, the serial prefill loop at c:3583). */
static long long attend(rctx* r, int l, int pos, const float* q, float* out, int parallel) {
    Config* p = &r->p;
    RunState* s = &r->s;
    int head_size = s->head_size;
    int q_dim = s->q_dim;
    for (int i = 0; i < q_dim; ++i) s->q[i] = q[i] * r->scale;
    if (r->mode == L3P_MODE_Q8) quantize_to_q8_0_cache(s->q, s->qQ8, q_dim);
    memset(out, 0, q_dim * sizeof(float));

    int is_swa_layer = (p->swa_pattern > 0) && (l % p->swa_pattern < p->swa_pattern - 1);
    int start_t = 0;
    if (p->is_gemma3 && is_swa_layer && p->swa_window > 0) {
        start_t = pos - p->swa_window + 1;
        if (start_t < 0) start_t = 0;
    }
    int att_size = pos - start_t + 1;
    int kv_mul = s->kv_mul;
    int head_q8_bytes = s->head_q8_bytes;
    size_t head_seq_bytes = s->head_seq_bytes;
    size_t loff = (size_t)l * s->kv_cache_layer_size;
    long long skipped = 0;
    int kvH;
#pragma omp parallel for private(kvH) reduction(+ : skipped) if (parallel)
    for (kvH = 0; kvH < p->n_kv_heads; kvH++) {
        size_t kBase = loff + kvH * head_seq_bytes;
        size_t fBase = (size_t)kvH * p->seq_len;
        for (int t = start_t; t <= pos; t++) {
            for (int mh = 0; mh < kv_mul; mh++) {
                int h = kvH * kv_mul + mh;
                float sc;
                if (r->mode == L3P_MODE_Q8) {
                    int qOff = h * head_q8_bytes;
                    const uint8_t* kQ8 = s->key_cache + kBase + (size_t)t * head_q8_bytes;
                    sc = dot_q8_0_q8_0_cache(s->qQ8 + qOff, s->qQ8i8 + qOff, kQ8,
                                             (const int8_t*)kQ8, head_size);
                } else {
                    sc = vec_dot_f32(s->q + s->head_q_offsets[h],
                                     r->kf[l] + (fBase + t) * head_size, head_size);
                }
                s->att[s->head_att_offsets[h] + t - start_t] = sc;
            }
        }
        for (int mh = 0; mh < kv_mul; mh++) {
            int h = kvH * kv_mul + mh;
            float* att = s->att + s->head_att_offsets[h];
            softmax(att, att_size);
            float* xb = out + s->head_q_offsets[h];
            for (int t = start_t; t <= pos; t++) {
                float w = att[t - start_t];
                if (w > -1e-8f && w < 1e-8f) ++skipped;
                if (r->mode == L3P_MODE_Q8)
                    accum_q8_0_cache(xb, s->value_cache + kBase + (size_t)t * head_q8_bytes, w,
                                     head_size);
                else
                    accum_f32_ref(xb, r->vf[l] + (fBase + t) * head_size, w, head_size);
            }
        }
    }
    return skipped;
}

L3P_EXPORT int l3pref_decode(void* ctx, int layer, int pos, const float* q, const float* k_row,
                             const float* v_row, float* out, long long* skipped) {
    rctx* r = (rctx*)ctx;
    if (!r || layer < 0 || layer >= r->p.n_layers || pos < 0 || pos >= r->p.seq_len) return -2;
    if (r->mode == L3P_MODE_F32 && !ensure_f32_layer(r, layer)) return -4;
    int hs = r->s.head_size;
    if (k_row && v_row)
        for (int kh = 0; kh < r->p.n_kv_heads; ++kh)
            put_row(r, layer, kh, pos, k_row + (size_t)kh * hs, v_row + (size_t)kh * hs);
    long long sk = attend(r, layer, pos, q, out, 1);
    if (skipped) *skipped = sk;
    return 0;
}

L3P_EXPORT int l3pref_prefill(void* ctx, int layer, int start_pos, int n_tok, const float* q,
                              const float* k, const float* v, float* out, long long* skipped) {
    rctx* r = (rctx*)ctx;
    if (!r || layer < 0 || layer >= r->p.n_layers || start_pos < 0 ||
        start_pos + n_tok > r->p.seq_len)
        return -2;
    if (r->mode == L3P_MODE_F32 && !ensure_f32_layer(r, layer)) return -4;
    int hs = r->s.head_size;
    size_t q_dim = (size_t)r->s.q_dim, kv_dim = (size_t)r->s.kv_dim;
    long long total = 0;
    for (int b = 0; b < n_tok; ++b) {
        int pos = start_pos + b;
        if (k && v)
            for (int kh = 0; kh < r->p.n_kv_heads; ++kh)
                put_row(r, layer, kh, pos, k + b * kv_dim + (size_t)kh * hs,
                        v + b * kv_dim + (size_t)kh * hs);
        total += attend(r, layer, pos, q + b * q_dim, out + b * q_dim, 0);
    }
    if (skipped) *skipped = total;
    return 0;
}

L3P_EXPORT float l3pref_fp16_to_fp32(uint16_t h) {
    ensure_fp16();
    return fp16_to_fp32(h);
}
L3P_EXPORT uint16_t l3pref_fp32_to_fp16(float f) { return fp32_to_fp16(f); }
L3P_EXPORT void l3pref_q8_quantize(const float* src, uint8_t* dst, int count) {
    quantize_to_q8_0_cache(src, dst, count);
}
L3P_EXPORT float l3pref_q8_dot(const uint8_t* a, const uint8_t* b, int count) {
    ensure_fp16();
    return dot_q8_0_q8_0_cache(a, (const int8_t*)a, b, (const int8_t*)b, count);
}
L3P_EXPORT void l3pref_q8_accum(float* out, const uint8_t* v, float w, int count) {
    ensure_fp16();
    accum_q8_0_cache(out, v, w, count);
}
L3P_EXPORT void l3pref_softmax(float* x, int n) { softmax(x, n); }
L3P_EXPORT int l3pref_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Pre-attention step of c:3233-3296 (decode) / c:3507-3560 (prefill) for
 * n_tok tokens: the reference's own rmsnorm_per_head (c:3150) and the cos/sin
 * tables its malloc_run_state builds (c:381-421, per-layer choice c:456-468);
 * the rotation loops are re-created without the attn_scale factor, which the
 * attention applies afterwards. */
L3P_EXPORT int l3pref_rope(const l3p_oracle_cfg* cfg, const l3p_oracle_rope* rope, int layer, int pos0,
                           int n_tok, float* q, float* k) {
    if (!cfg || !rope || !q || !k || n_tok < 0 || pos0 < 0 || layer < 0 || layer >= cfg->n_layers)
        return -1;
    Config p;
    memset(&p, 0, sizeof(p));
    p.n_layers = layer + 1;
    p.n_heads = cfg->n_heads;
    p.n_kv_heads = cfg->n_kv_heads;
    p.head_dim = cfg->head_dim;
    p.dim = cfg->n_heads * cfg->head_dim;
    p.hidden_dim = 32;
    p.vocab_size = 1;
    p.seq_len = pos0 + n_tok > 1 ? pos0 + n_tok : 1;
    p.is_gemma3 = cfg->is_gemma3;
    p.swa_window = cfg->swa_window;
    p.swa_pattern = cfg->swa_pattern;
    p.rope_theta = rope->rope_theta > 0.0f ? rope->rope_theta : (cfg->is_gemma3 ? 1000000.0f : 500000.0f);
    p.rope_theta_swa = rope->rope_theta_swa;
    p.rms_norm_eps = rope->rms_norm_eps;
    RunState s;
    memset(&s, 0, sizeof(s));
    malloc_run_state(&s, &p);
    float eps = p.rms_norm_eps > 0 ? p.rms_norm_eps : 1e-5f; /* c:3198 */
    int head_size = s.head_size, half = head_size / 2;
    int q_dim = s.q_dim, kv_dim = s.kv_dim;
    for (int b = 0; b < n_tok; ++b) {
        int pos = pos0 + b;
        float* q_arr = q + (size_t)b * q_dim;
        float* k_arr = k + (size_t)b * kv_dim;
        if (p.is_gemma3 && rope->q_norm && rope->k_norm) {
            rmsnorm_per_head(q_arr, q_arr, (float*)rope->q_norm + layer * head_size, p.n_heads, head_size,
                             s.inv_head_size, eps);
            rmsnorm_per_head(k_arr, k_arr, (float*)rope->k_norm + layer * head_size, p.n_kv_heads, head_size,
                             s.inv_head_size, eps);
        }
        float* rope_cos = s.rope_cos_layer[layer] + pos * half;
        float* rope_sin = s.rope_sin_layer[layer] + pos * half;
        if (p.is_gemma3) {
            for (int h = 0; h < p.n_heads + p.n_kv_heads; h++) {
                float* x = h < p.n_heads ? q_arr + h * head_size : k_arr + (h - p.n_heads) * head_size;
                for (int i = 0; i < half; i++) {
                    float v0 = x[i], v1 = x[i + half];
                    x[i] = v0 * rope_cos[i] - v1 * rope_sin[i];
                    x[i + half] = v0 * rope_sin[i] + v1 * rope_cos[i];
                }
            }
        } else {
            for (int i = 0; i < q_dim; i += 2) {
                int j = (i % head_size) / 2;
                float v0 = q_arr[i], v1 = q_arr[i + 1];
                q_arr[i] = v0 * rope_cos[j] - v1 * rope_sin[j];
                q_arr[i + 1] = v0 * rope_sin[j] + v1 * rope_cos[j];
                if (i < kv_dim) {
                    float k0 = k_arr[i], k1 = k_arr[i + 1];
                    k_arr[i] = k0 * rope_cos[j] - k1 * rope_sin[j];
                    k_arr[i + 1] = k0 * rope_sin[j] + k1 * rope_cos[j];
                }
            }
        }
    }
    free_run_state(&s);
    return 0;
}

/* The wo projection through the reference's own matmul_quantized (c:2091)
 * with a QuantizedTensor set up as load_quantized_tensor does (c:2912-2920)
 * and the dequantisation / Q8_0 scratch main() allocates (c:5190-5200). */
L3P_EXPORT int l3pref_matvec(int type, const void* w, int rows, int cols, const float* x, float* out) {
    if (!w || !x || !out || rows <= 0 || cols <= 0) return -1;
    ensure_fp16();
    static int scratch_cols = 0;
    if (cols > scratch_cols) {
        free(q8_buf);
        free(deq_buf);
        q8_buf = (block_q8_0*)calloc((size_t)(cols + QK8_0 - 1) / QK8_0, sizeof(block_q8_0));
        deq_buf_stride = 4 * cols;
        deq_buf = (float*)calloc((size_t)omp_get_max_threads() * deq_buf_stride, sizeof(float));
        if (!q8_buf || !deq_buf) return -4;
        scratch_cols = cols;
    }
    QuantizedTensor qt;
    memset(&qt, 0, sizeof(qt));
    qt.data = (void*)w;
    qt.type = (enum ggml_type)type;
    qt.n_elements = rows * cols;
    qt.rows = rows;
    qt.cols = cols;
    qt.row_size = get_row_size(cols, qt.type);
    qt.q8_func = get_vec_dot_q8_func(qt.type);
    qt.dot_func = get_vec_dot_func(qt.type);
    qt.deq_func = get_deq_row_func(qt.type);
    matmul_quantized(out, x, &qt);
    return 0;
}
