/*
 * l3p_oracle.c -- plain-C restatement of llama3pure's attention step.
 *
 * TEST INFRASTRUCTURE ONLY (see l3p_oracle.h).  The shipped library never
 * links or calls this file; it is the checker for the CUDA kernels and the
 * "port" CPU baseline when the reference harness is not built.
 *
 * Every function restates one piece of llama3pure-c-engine.c (cited as
 * c:<line>) in this repository's own code.  Summation order, rounding points
 * and the skip rule follow the reference so that, built without fast-math and
 * without FMA contraction, the results are bit-identical to the reference's
 * own functions (tests/test_oracle.py checks this against oracle/_ref/ and
 * against the committed golden vectors in tests/golden/).
 *
 * Parity is pinned: golden vectors were produced by the reference's own code
 * compiled from llama3pure-c-engine.c (oracle/ref_harness.c,
 * tests/golden/make_golden.py).
 */
#include "l3p_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 32          /* values per Q8_0 block (c:120 QK8_0) */
#define QBLOCK 34      /* bytes per Q8_0 block: fp16 scale + 32 int8 (c:123) */
#define SKIP_EPS 1e-8f /* near-zero weight skip threshold (c:1602) */

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32, as the Q8_0 KV codec stores its block scale.               */

/* fp16 bits -> fp32.  Same values as the reference's 65536-entry table built
 * by init_fp16_table (c:545-578): exact for normals and subnormals, inf/nan
 * keep their payload shifted into the fp32 mantissa. */
float l3po_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ff;
    uint32_t bits;
    if (e == 0x1f) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        /* subnormal half: value = m * 2^-24, renormalise */
        int shift = 0;
        while ((m & 0x400) == 0) {
            m <<= 1;
            ++shift;
        }
        bits = sign | ((uint32_t)(113 - shift) << 23) | ((m & 0x3ff) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* fp32 -> fp16 by TRUNCATION of the mantissa (no round-to-nearest), with
 * values below half's subnormal range flushed to signed zero and anything at
 * or above 2^16 (including nan) mapped to signed inf -- fp32_to_fp16,
 * c:585-599. */
uint16_t l3po_fp32_to_fp16(float f) {
    uint32_t b;
    memcpy(&b, &f, sizeof b);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
    int e = (int)((b >> 23) & 0xff) - 112; /* rebias 127 -> 15 */
    uint32_t sig = (b & 0x7fffffu) | 0x800000u; /* 24-bit significand */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e > 0) return (uint16_t)(sign | (uint16_t)(e << 10) | (uint16_t)((b >> 13) & 0x3ffu));
    if (e < -10) return sign;
    /* subnormal result: drop 13 mantissa bits plus (1 - e) more */
    return (uint16_t)(sign | (uint16_t)(sig >> (14 - e)));
}

/* ------------------------------------------------------------------------ */
/* Q8_0 KV codec                                                             */

/* One Q8_0 encode of `count` floats (multiple of 32): per block, the scale
 * d = amax/127 stored as truncated fp16, and q = round-half-away(x*127/amax)
 * clamped to int8 -- quantize_to_q8_0_cache, c:1535-1570. */
void l3po_q8_quantize(const float* src, uint8_t* dst, int count) {
    for (int b = 0; b < count / QK; ++b) {
        const float* x = src + b * QK;
        uint8_t* blk = dst + b * QBLOCK;
        float amax = 0.0f;
        for (int j = 0; j < QK; ++j) {
            float a = fabsf(x[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float inv = (d > 0.0f) ? 127.0f / amax : 0.0f;
        uint16_t dh = l3po_fp32_to_fp16(d);
        blk[0] = (uint8_t)(dh & 0xff);
        blk[1] = (uint8_t)(dh >> 8);
        for (int j = 0; j < QK; ++j) {
            int qv = (int)roundf(x[j] * inv);
            qv = qv > 127 ? 127 : (qv < -128 ? -128 : qv);
            blk[2 + j] = (uint8_t)(int8_t)qv;
        }
    }
}

static inline float block_scale(const uint8_t* blk) {
    return l3po_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8)));
}

/* Q8_0 x Q8_0 dot: sum over blocks of (d_a*d_b)*int32(sum of int8 products),
 * accumulated in fp32 in block order -- dot_q8_0_q8_0_cache, c:1574-1597. */
float l3po_q8_dot(const uint8_t* a, const uint8_t* b, int count) {
    float acc = 0.0f;
    for (int blkno = 0; blkno < count / QK; ++blkno) {
        const uint8_t* ba = a + blkno * QBLOCK;
        const uint8_t* bb = b + blkno * QBLOCK;
        int32_t isum = 0;
        for (int j = 0; j < QK; ++j) isum += (int32_t)(int8_t)ba[2 + j] * (int32_t)(int8_t)bb[2 + j];
        float dd = block_scale(ba) * block_scale(bb);
        acc += dd * (float)isum;
    }
    return acc;
}

/* out += w * dequant(V row), skipped entirely when |w| < 1e-8; the product is
 * formed as int8 * (d*w) -- accum_q8_0_cache, c:1600-1622. */
void l3po_q8_accum(float* out, const uint8_t* v, float w, int count) {
    if (w > -SKIP_EPS && w < SKIP_EPS) return;
    for (int blkno = 0; blkno < count / QK; ++blkno) {
        const uint8_t* blk = v + blkno * QBLOCK;
        float sw = block_scale(blk) * w;
        float* o = out + blkno * QK;
        for (int j = 0; j < QK; ++j) o[j] += (float)(int8_t)blk[2 + j] * sw;
    }
}

/* ------------------------------------------------------------------------ */
/* softmax and the fp32 forms                                                */

/* In-place softmax: running max (first element seeds it, strict >), expf of
 * the shifted values summed in order, then scaled by the reciprocal of the
 * sum -- softmax, c:3167-3186. */
void l3po_softmax(float* x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; ++i)
        if (x[i] > mx) mx = x[i];
    float total = 0.0f;
    for (int i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        total += x[i];
    }
    float r = 1.0f / total;
    for (int i = 0; i < n; ++i) x[i] *= r;
}

/* Sequential fp32 dot -- vec_dot_f32, c:1487-1494. */
static inline float dot_f32(const float* x, const float* w, int n) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) acc += x[i] * w[i];
    return acc;
}

/* fp32 form of accum_q8_0_cache (c:1600-1622): same skip rule, out += w*v. */
static inline void accum_f32(float* out, const float* v, float w, int n) {
    if (w > -SKIP_EPS && w < SKIP_EPS) return;
    for (int i = 0; i < n; ++i) out[i] += w * v[i];
}

/* ------------------------------------------------------------------------ */
/* Attention step                                                            */

typedef struct {
    l3p_oracle_cfg c;
    int mode;
    float scale;
    int kv_mul;
    int hd;
    int row_q8; /* bytes of one Q8_0 head row */
    float** kf; /* per layer [Hkv][cap][hd] (f32 mode), lazily allocated */
    float** vf;
    uint8_t** kq; /* per layer [Hkv][cap][row_q8] (q8 mode) */
    uint8_t** vq;
    float* att;   /* [Hq][cap] scores / weights (c:290, c:363) */
    float* qs;    /* scaled query [Hq*hd] */
    uint8_t* qq;  /* Q8_0 query [Hq][row_q8] (c:321-322) */
} octx;

/* Sliding-window start: only Gemma-3 SWA layers (l % pattern < pattern-1)
 * with a positive window start at pos-window+1 (clamped at 0) -- c:3246 and
 * c:3316-3321 (decode), c:3496 and c:3574-3580 (prefill). */
int l3po_start_t(const l3p_oracle_cfg* c, int layer, int pos) {
    int swa_layer = c->swa_pattern > 0 && (layer % c->swa_pattern) < c->swa_pattern - 1;
    if (c->is_gemma3 && swa_layer && c->swa_window > 0) {
        int s = pos - c->swa_window + 1;
        return s < 0 ? 0 : s;
    }
    return 0;
}

void* l3po_create(const l3p_oracle_cfg* cfg, int mode) {
    if (!cfg || cfg->n_layers <= 0 || cfg->n_heads <= 0 || cfg->n_kv_heads <= 0 ||
        cfg->head_dim <= 0 || cfg->head_dim % QK != 0 || cfg->seq_len <= 0 ||
        cfg->n_heads % cfg->n_kv_heads != 0)
        return NULL;
    octx* o = (octx*)calloc(1, sizeof(octx));
    if (!o) return NULL;
    o->c = *cfg;
    o->mode = mode;
    o->hd = cfg->head_dim;
    /* attn_scale = 1/sqrtf(head_size), c:434 */
    o->scale = cfg->scale != 0.0f ? cfg->scale : 1.0f / sqrtf((float)cfg->head_dim);
    o->kv_mul = cfg->n_heads / cfg->n_kv_heads; /* c:428 */
    o->row_q8 = cfg->head_dim / QK * QBLOCK;    /* c:365 head_q8_bytes */
    o->kf = (float**)calloc((size_t)cfg->n_layers, sizeof(float*));
    o->vf = (float**)calloc((size_t)cfg->n_layers, sizeof(float*));
    o->kq = (uint8_t**)calloc((size_t)cfg->n_layers, sizeof(uint8_t*));
    o->vq = (uint8_t**)calloc((size_t)cfg->n_layers, sizeof(uint8_t*));
    o->att = (float*)calloc((size_t)cfg->n_heads * cfg->seq_len, sizeof(float));
    o->qs = (float*)calloc((size_t)cfg->n_heads * cfg->head_dim, sizeof(float));
    o->qq = (uint8_t*)calloc((size_t)cfg->n_heads * o->row_q8, 1);
    if (!o->kf || !o->vf || !o->kq || !o->vq || !o->att || !o->qs || !o->qq) {
        l3po_destroy(o);
        return NULL;
    }
    return o;
}

void l3po_destroy(void* ctx) {
    octx* o = (octx*)ctx;
    if (!o) return;
    for (int l = 0; l < o->c.n_layers; ++l) {
        if (o->kf) free(o->kf[l]);
        if (o->vf) free(o->vf[l]);
        if (o->kq) free(o->kq[l]);
        if (o->vq) free(o->vq[l]);
    }
    free(o->kf);
    free(o->vf);
    free(o->kq);
    free(o->vq);
    free(o->att);
    free(o->qs);
    free(o->qq);
    free(o);
}

/* Make sure the cache of `layer` exists (the reference preallocates all
 * layers at c:365-379; this oracle allocates on first use so that a test can
 * hold one layer of a long-context configuration). */
static int ensure_layer(octx* o, int layer) {
    size_t rows = (size_t)o->c.n_kv_heads * o->c.seq_len;
    if (o->mode == L3P_MODE_F32) {
        if (!o->kf[layer]) o->kf[layer] = (float*)calloc(rows * o->hd, sizeof(float));
        if (!o->vf[layer]) o->vf[layer] = (float*)calloc(rows * o->hd, sizeof(float));
        return o->kf[layer] && o->vf[layer];
    }
    if (!o->kq[layer]) o->kq[layer] = (uint8_t*)calloc(rows * o->row_q8, 1);
    if (!o->vq[layer]) o->vq[layer] = (uint8_t*)calloc(rows * o->row_q8, 1);
    return o->kq[layer] && o->vq[layer];
}

/* Write one head row of K and V at `pos` -- the per-head cache write of
 * c:3299-3308 (decode) / c:3562-3567 (prefill); Q8_0-encoded in q8 mode. */
static void put_row(octx* o, int layer, int kvh, int pos, const float* krow, const float* vrow) {
    size_t r = (size_t)kvh * o->c.seq_len + (size_t)pos;
    if (o->mode == L3P_MODE_F32) {
        memcpy(o->kf[layer] + r * o->hd, krow, (size_t)o->hd * sizeof(float));
        memcpy(o->vf[layer] + r * o->hd, vrow, (size_t)o->hd * sizeof(float));
    } else {
        l3po_q8_quantize(krow, o->kq[layer] + r * o->row_q8, o->hd);
        l3po_q8_quantize(vrow, o->vq[layer] + r * o->row_q8, o->hd);
    }
}

int l3po_load_kv(void* ctx, int layer, int pos0, int n_pos, const float* k, const float* v) {
    octx* o = (octx*)ctx;
    if (!o || layer < 0 || layer >= o->c.n_layers || pos0 < 0 || n_pos < 0 ||
        pos0 + n_pos > o->c.seq_len)
        return -2;
    if (!ensure_layer(o, layer)) return -4;
    for (int h = 0; h < o->c.n_kv_heads; ++h)
        for (int t = 0; t < n_pos; ++t) {
            size_t src = ((size_t)h * n_pos + t) * o->hd;
            put_row(o, layer, h, pos0 + t, k + src, v + src);
        }
    return 0;
}

/* Attention of one token at `pos` over cached positions [start_t, pos],
 * writing out[Hq*hd].  Body of c:3310-3359 (decode) and c:3569-3612
 * (prefill, which runs the KV-head loop without OpenMP). */
static long long attend(octx* o, int layer, int pos, const float* q, float* out, int parallel) {
    const int hd = o->hd, g = o->kv_mul, cap = o->c.seq_len;
    const int qdim = o->c.n_heads * hd;
    /* q arrives post-RoPE; the reference multiplies by attn_scale inside its
     * RoPE loop (c:3264-3265, c:3288-3289), so scale each element once. */
    for (int i = 0; i < qdim; ++i) o->qs[i] = q[i] * o->scale;
    if (o->mode == L3P_MODE_Q8) l3po_q8_quantize(o->qs, o->qq, qdim); /* c:3312 */
    memset(out, 0, (size_t)qdim * sizeof(float));                      /* c:3314 */
    const int start = l3po_start_t(&o->c, layer, pos);
    const int n = pos - start + 1;
    long long skipped = 0;
    int kvh;
#pragma omp parallel for reduction(+ : skipped) if (parallel)
    for (kvh = 0; kvh < o->c.n_kv_heads; ++kvh) {
        const size_t base = (size_t)kvh * cap;
        /* scores, position-first over the GQA group (c:3333-3344) */
        for (int t = start; t <= pos; ++t) {
            for (int j = 0; j < g; ++j) {
                int h = kvh * g + j;
                float s;
                if (o->mode == L3P_MODE_F32)
                    s = dot_f32(o->qs + (size_t)h * hd, o->kf[layer] + (base + t) * hd, hd);
                else
                    s = l3po_q8_dot(o->qq + (size_t)h * o->row_q8,
                                    o->kq[layer] + (base + t) * o->row_q8, hd);
                o->att[(size_t)h * cap + (t - start)] = s;
            }
        }
        /* per-head softmax then weighted V sum in position order (c:3347-3358) */
        for (int j = 0; j < g; ++j) {
            int h = kvh * g + j;
            float* w = o->att + (size_t)h * cap;
            l3po_softmax(w, n);
            float* oh = out + (size_t)h * hd;
            for (int t = start; t <= pos; ++t) {
                float wt = w[t - start];
                if (wt > -SKIP_EPS && wt < SKIP_EPS) ++skipped;
                if (o->mode == L3P_MODE_F32)
                    accum_f32(oh, o->vf[layer] + (base + t) * hd, wt, hd);
                else
                    l3po_q8_accum(oh, o->vq[layer] + (base + t) * o->row_q8, wt, hd);
            }
        }
    }
    return skipped;
}

int l3po_decode(void* ctx, int layer, int pos, const float* q, const float* k_row,
                const float* v_row, float* out, long long* skipped) {
    octx* o = (octx*)ctx;
    if (!o || !q || !out || layer < 0 || layer >= o->c.n_layers || pos < 0 || pos >= o->c.seq_len)
        return -2;
    if (!ensure_layer(o, layer)) return -4;
    if (k_row && v_row)
        for (int h = 0; h < o->c.n_kv_heads; ++h)
            put_row(o, layer, h, pos, k_row + (size_t)h * o->hd, v_row + (size_t)h * o->hd);
    long long s = attend(o, layer, pos, q, out, 1);
    if (skipped) *skipped = s;
    return 0;
}

/* Token-by-token causal prefill: token b (pos = start_pos+b) first appends
 * its own K/V row, then attends to [start_t, pos] -- c:3499-3613.  The
 * attention loop there carries no OpenMP pragma (c:3583), so neither does
 * this one. */
int l3po_prefill(void* ctx, int layer, int start_pos, int n_tok, const float* q,
                 const float* k, const float* v, float* out, long long* skipped) {
    octx* o = (octx*)ctx;
    if (!o || !q || !out || layer < 0 || layer >= o->c.n_layers || start_pos < 0 || n_tok < 0 ||
        start_pos + n_tok > o->c.seq_len)
        return -2;
    if (!ensure_layer(o, layer)) return -4;
    const size_t qdim = (size_t)o->c.n_heads * o->hd, kvdim = (size_t)o->c.n_kv_heads * o->hd;
    long long total = 0;
    for (int b = 0; b < n_tok; ++b) {
        int pos = start_pos + b;
        if (k && v)
            for (int h = 0; h < o->c.n_kv_heads; ++h)
                put_row(o, layer, h, pos, k + b * kvdim + (size_t)h * o->hd,
                        v + b * kvdim + (size_t)h * o->hd);
        total += attend(o, layer, pos, q + b * qdim, out + b * qdim, 0);
    }
    if (skipped) *skipped = total;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Pre-attention step: Gemma3 QK-RMSNorm and RoPE.                          */

/* Per-head RMS norm in place: the sum of squares accumulated in index order,
 * r = 1/sqrtf(mean + eps), x = w * (r * x)  (rmsnorm_per_head, c:3150-3165). */
static void head_rmsnorm(float* x, const float* w, int hd, float inv_hd, float eps) {
    float ss = 0.0f;
    for (int j = 0; j < hd; ++j) ss += x[j] * x[j];
    float r = 1.0f / sqrtf(ss * inv_hd + eps);
    for (int j = 0; j < hd; ++j) x[j] = w[j] * (r * x[j]);
}

/* Rotate one head row by the (cos, sin) pairs of its position: NEOX pairs
 * (i, i + hd/2) for Gemma3 (c:3254-3278), consecutive pairs (2i, 2i+1)
 * otherwise (c:3279-3296).  No attention scale (applied by the attention). */
static void head_rotate(float* x, const float* c, const float* s, int hd, int neox) {
    int half = hd / 2;
    for (int i = 0; i < half; ++i) {
        int a = neox ? i : 2 * i;
        int b = neox ? i + half : 2 * i + 1;
        float v0 = x[a], v1 = x[b];
        x[a] = v0 * c[i] - v1 * s[i];
        x[b] = v0 * s[i] + v1 * c[i];
    }
}

int l3po_rope(const l3p_oracle_cfg* cfg, const l3p_oracle_rope* rope, int layer, int pos0, int n_tok,
              float* q, float* k) {
    if (!cfg || !rope || !q || !k || n_tok < 0 || pos0 < 0 || layer < 0 || layer >= cfg->n_layers)
        return -1;
    int hd = cfg->head_dim, half = hd / 2, gemma = cfg->is_gemma3 != 0;
    /* per-layer table choice (c:456-468) and the theta defaults (c:390, c:5127) */
    int pat = cfg->swa_pattern;
    int swa_layer = pat > 0 && layer % pat < pat - 1;
    float theta;
    if (gemma && swa_layer)
        theta = rope->rope_theta_swa > 0.0f ? rope->rope_theta_swa : 10000.0f;
    else
        theta = rope->rope_theta > 0.0f ? rope->rope_theta : (gemma ? 1000000.0f : 500000.0f);
    float eps = rope->rms_norm_eps > 0.0f ? rope->rms_norm_eps : 1e-5f;
    float inv_hd = 1.0f / (float)hd;
    int norm = gemma && rope->q_norm && rope->k_norm;
    float* freq = (float*)malloc(sizeof(float) * 3 * (size_t)half);
    if (!freq) return -4;
    float* c = freq + half;
    float* s = c + half;
    /* inverse frequencies and angles as c:384-405 */
    for (int i = 0; i < half; ++i) freq[i] = 1.0f / powf(theta, (float)(i * 2) / (float)hd);
    size_t qd = (size_t)cfg->n_heads * hd, kvd = (size_t)cfg->n_kv_heads * hd;
    for (int t = 0; t < n_tok; ++t) {
        int pos = pos0 + t;
        for (int i = 0; i < half; ++i) {
            float ang = pos * freq[i];
            c[i] = cosf(ang);
            s[i] = sinf(ang);
        }
        for (int h = 0; h < cfg->n_heads; ++h) {
            float* x = q + t * qd + (size_t)h * hd;
            if (norm) head_rmsnorm(x, rope->q_norm + (size_t)layer * hd, hd, inv_hd, eps);
            head_rotate(x, c, s, hd, gemma);
        }
        for (int h = 0; h < cfg->n_kv_heads; ++h) {
            float* x = k + t * kvd + (size_t)h * hd;
            if (norm) head_rmsnorm(x, rope->k_norm + (size_t)layer * hd, hd, inv_hd, eps);
            head_rotate(x, c, s, hd, gemma);
        }
    }
    free(freq);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* The wo projection: weight rows dequantised, then fp32 dot products.      */

#define QK_SUPER 256 /* values per K-quant super-block (c:121 QK_K) */

long long l3po_w_row_bytes(int type, int cols) {
    switch (type) {
        case L3P_W_F32: return (long long)cols * 4;
        case L3P_W_F16:
        case L3P_W_BF16: return (long long)cols * 2;
        case L3P_W_Q4_0:
        case L3P_W_IQ4_NL: return (long long)(cols / 32) * 18;
        case L3P_W_Q4_1: return (long long)(cols / 32) * 20;
        case L3P_W_Q5_0: return (long long)(cols / 32) * 22;
        case L3P_W_Q5_1: return (long long)(cols / 32) * 24;
        case L3P_W_Q8_0: return (long long)(cols / 32) * 34;
        case L3P_W_Q2_K: return (long long)(cols / QK_SUPER) * 84;
        case L3P_W_Q3_K: return (long long)(cols / QK_SUPER) * 110;
        case L3P_W_Q4_K: return (long long)(cols / QK_SUPER) * 144;
        case L3P_W_Q5_K: return (long long)(cols / QK_SUPER) * 176;
        case L3P_W_Q6_K: return (long long)(cols / QK_SUPER) * 210;
        default: return 0;
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Q8_0: value = int8 * d (dequantize_row_q8_0, c:691-702). */
static void deq_q8_0(const uint8_t* src, float* dst, int cols) {
    for (int b = 0; b < cols / 32; ++b) {
        const uint8_t* blk = src + (size_t)b * 34;
        float d = l3po_fp16_to_fp32(rd16(blk));
        for (int j = 0; j < 32; ++j) dst[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
    }
}

/* 6-bit scale and min number j (0..7) of a Q4_K block's 12 packed bytes:
 * j < 4 in the low 6 bits of bytes j and j+4; j >= 4 split between the
 * nibbles of byte j+4 and the top 2 bits of bytes j-4 and j (c:705-713). */
static void k4_scale_min(const uint8_t* sc, int j, int* scale, int* min) {
    if (j < 4) {
        *scale = sc[j] & 63;
        *min = sc[j + 4] & 63;
    } else {
        *scale = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4);
        *min = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

/* Q4_K: 8 sub-blocks of 32; sub-block j value = (d*scale_j) * nibble - dmin*min_j.
 * Sub-blocks 2p and 2p+1 share 32 bytes: low nibbles, then high (c:715-746). */
static void deq_q4_k(const uint8_t* src, float* dst, int cols) {
    for (int b = 0; b < cols / QK_SUPER; ++b) {
        const uint8_t* blk = src + (size_t)b * 144;
        float d = l3po_fp16_to_fp32(rd16(blk)), dmin = l3po_fp16_to_fp32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* qs = blk + 16;
        float* y = dst + (size_t)b * QK_SUPER;
        for (int p = 0; p < 4; ++p) {
            int s0, m0, s1, m1;
            k4_scale_min(sc, 2 * p, &s0, &m0);
            k4_scale_min(sc, 2 * p + 1, &s1, &m1);
            float dl = d * s0, ml = dmin * m0, dh = d * s1, mh = dmin * m1;
            for (int l = 0; l < 32; ++l) y[64 * p + l] = dl * (qs[32 * p + l] & 15) - ml;
            for (int l = 0; l < 32; ++l) y[64 * p + 32 + l] = dh * (qs[32 * p + l] >> 4) - mh;
        }
    }
}

/* Q5_K: Q4_K's layout with a fifth bit per value: sub-block 2p (low nibbles
 * of qs[32p..32p+32)) takes bit 2p of qh[l], sub-block 2p+1 (high nibbles)
 * bit 2p+1, each worth 16 (c:834-871). */
static void deq_q5_k(const uint8_t* src, float* dst, int cols) {
    for (int b = 0; b < cols / QK_SUPER; ++b) {
        const uint8_t* blk = src + (size_t)b * 176;
        float d = l3po_fp16_to_fp32(rd16(blk)), dmin = l3po_fp16_to_fp32(rd16(blk + 2));
        const uint8_t* sc = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* qs = blk + 48;
        float* y = dst + (size_t)b * QK_SUPER;
        for (int p = 0; p < 4; ++p) {
            int s0, m0, s1, m1;
            k4_scale_min(sc, 2 * p, &s0, &m0);
            k4_scale_min(sc, 2 * p + 1, &s1, &m1);
            float dl = d * s0, ml = dmin * m0, dh = d * s1, mh = dmin * m1;
            for (int l = 0; l < 32; ++l) {
                int lo = (qs[32 * p + l] & 15) + (((qh[l] >> (2 * p)) & 1) ? 16 : 0);
                int hi = (qs[32 * p + l] >> 4) + (((qh[l] >> (2 * p + 1)) & 1) ? 16 : 0);
                y[64 * p + l] = dl * lo - ml;
                y[64 * p + 32 + l] = dh * hi - mh;
            }
        }
    }
}

/* Q2_K: two halves of 128 values, each from 32 quant bytes; within a half,
 * bit pair j (shift 2j) of bytes 0..15 and 16..31 gives two sub-blocks of
 * 16, scale byte s = scales[8h + 2j (+1)]: value = (d * (s & 15)) * q -
 * dmin * (s >> 4) (c:748-784). */
static void deq_q2_k(const uint8_t* src, float* dst, int cols) {
    for (int b = 0; b < cols / QK_SUPER; ++b) {
        const uint8_t* blk = src + (size_t)b * 84;
        const uint8_t* sc = blk;
        const uint8_t* qs = blk + 16;
        float d = l3po_fp16_to_fp32(rd16(blk + 80)), dmin = l3po_fp16_to_fp32(rd16(blk + 82));
        float* y = dst + (size_t)b * QK_SUPER;
        for (int h = 0; h < 2; ++h)
            for (int j = 0; j < 4; ++j)
                for (int g = 0; g < 2; ++g) {
                    int s = sc[8 * h + 2 * j + g];
                    float dl = d * (s & 15), ml = dmin * (s >> 4);
                    for (int l = 0; l < 16; ++l)
                        y[128 * h + 32 * j + 16 * g + l] = dl * ((qs[32 * h + 16 * g + l] >> (2 * j)) & 3) - ml;
                }
    }
}

/* Q3_K: Q2_K's quant layout with a third bit from hmask (set: +0, clear:
 * -4, bit 4h + j of hmask[l]) and 16 signed 6-bit scales (stored - 32):
 * the low nibbles of bytes 0..7 and, above them, bit pairs of bytes 8..11
 * (c:786-832). */
static int q3_scale(const uint8_t* sc, int k) {
    int low = k < 8 ? (sc[k] & 15) : (sc[k - 8] >> 4);
    int high = (sc[8 + (k & 3)] >> (2 * (k >> 2))) & 3;
    return (low | (high << 4)) - 32;
}

static void deq_q3_k(const uint8_t* src, float* dst, int cols) {
    for (int b = 0; b < cols / QK_SUPER; ++b) {
        const uint8_t* blk = src + (size_t)b * 110;
        const uint8_t* hm = blk;
        const uint8_t* qs = blk + 32;
        const uint8_t* sc = blk + 96;
        float d = l3po_fp16_to_fp32(rd16(blk + 108));
        float* y = dst + (size_t)b * QK_SUPER;
        for (int h = 0; h < 2; ++h)
            for (int j = 0; j < 4; ++j)
                for (int g = 0; g < 2; ++g) {
                    float dl = d * q3_scale(sc, 8 * h + 2 * j + g);
                    int bit = 4 * h + j;
                    for (int l = 0; l < 16; ++l) {
                        int i = 16 * g + l;
                        int q = ((qs[32 * h + i] >> (2 * j)) & 3) - (((hm[i] >> bit) & 1) ? 0 : 4);
                        y[128 * h + 32 * j + i] = dl * q;
                    }
                }
    }
}

/* Q6_K: two halves of 128 values; value = d * scale * (6-bit q - 32), the 6
 * bits from a nibble of ql and two bits of qh (c:873-902). */
static void deq_q6_k(const uint8_t* src, float* dst, int cols) {
    for (int b = 0; b < cols / QK_SUPER; ++b) {
        const uint8_t* blk = src + (size_t)b * 210;
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        float d = l3po_fp16_to_fp32(rd16(blk + 208));
        float* y = dst + (size_t)b * QK_SUPER;
        for (int h = 0; h < 2; ++h) {
            const uint8_t* l8 = ql + 64 * h;
            const uint8_t* h8 = qh + 32 * h;
            const int8_t* s8 = sc + 8 * h;
            float* yh = y + 128 * h;
            for (int l = 0; l < 32; ++l) {
                int g = l / 16;
                int v0 = ((l8[l] & 15) | (((h8[l] >> 0) & 3) << 4)) - 32;
                int v1 = ((l8[l + 32] & 15) | (((h8[l] >> 2) & 3) << 4)) - 32;
                int v2 = ((l8[l] >> 4) | (((h8[l] >> 4) & 3) << 4)) - 32;
                int v3 = ((l8[l + 32] >> 4) | (((h8[l] >> 6) & 3) << 4)) - 32;
                yh[l] = d * s8[g] * v0;
                yh[l + 32] = d * s8[g + 2] * v1;
                yh[l + 64] = d * s8[g + 4] * v2;
                yh[l + 96] = d * s8[g + 6] * v3;
            }
        }
    }
}

/* The types without a row dequantiser take the reference's other two paths
 * of matmul_quantized (c:2102-2132): */

/* IQ4_NL's 16 non-linear values (the format's table, c:204-206). */
static const int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* Q4_0 / Q4_1 / Q5_0 / Q5_1 / IQ4_NL: x quantised to Q8_0 once
 * (quantize_row_q8_0, c:1508-1529: the cache quantiser's steps), then per
 * row and 32-value block an exact int32 sum of products, accumulated in fp32
 * in block order as dw*dx*isum (+ mw*dx*xsum with a min), as
 * vec_dot_{q4_0,q4_1,q5_0,q5_1,iq4_nl}_q8_0 (c:1625-1717, c:1994-2013). */
static float q8x_row_dot(int type, const uint8_t* row, const uint8_t* xq, int cols) {
    float sum = 0.0f;
    for (int b = 0; b < cols / 32; ++b) {
        const uint8_t* xb = xq + (size_t)b * QBLOCK;
        const int8_t* xs = (const int8_t*)(xb + 2);
        float dx = block_scale(xb);
        const uint8_t* blk;
        float dw, mw = 0.0f;
        uint32_t qh = 0;
        const uint8_t* qs;
        switch (type) {
            case L3P_W_Q4_0:
            case L3P_W_IQ4_NL: blk = row + (size_t)b * 18; qs = blk + 2; break;
            case L3P_W_Q4_1: blk = row + (size_t)b * 20; qs = blk + 4; mw = l3po_fp16_to_fp32(rd16(blk + 2)); break;
            case L3P_W_Q5_0:
                blk = row + (size_t)b * 22;
                qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
                qs = blk + 6;
                break;
            default: /* Q5_1 */
                blk = row + (size_t)b * 24;
                mw = l3po_fp16_to_fp32(rd16(blk + 2));
                qh = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) | ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
                qs = blk + 8;
                break;
        }
        dw = l3po_fp16_to_fp32(rd16(blk));
        int isum = 0, xsum = 0;
        for (int j = 0; j < 16; ++j) {
            int lo = qs[j] & 15, hi = qs[j] >> 4;
            switch (type) {
                case L3P_W_Q4_0: lo -= 8; hi -= 8; break;
                case L3P_W_IQ4_NL: lo = kIq4nl[lo]; hi = kIq4nl[hi]; break;
                case L3P_W_Q5_0: lo = (lo | (((qh >> j) & 1) << 4)) - 16; hi = (hi | (((qh >> (j + 16)) & 1) << 4)) - 16; break;
                case L3P_W_Q5_1: lo |= ((qh >> j) & 1) << 4; hi |= ((qh >> (j + 16)) & 1) << 4; break;
                default: break; /* Q4_1 */
            }
            isum += xs[j] * lo + xs[j + 16] * hi;
            xsum += xs[j] + xs[j + 16];
        }
        if (type == L3P_W_Q4_1 || type == L3P_W_Q5_1)
            sum += dw * dx * (float)isum + mw * dx * (float)xsum;
        else
            sum += dw * dx * (float)isum;
    }
    return sum;
}

/* F32 / F16 / BF16: fp32 products of x and the converted weight, summed in
 * index order (vec_dot_f16 / vec_dot_bf16 / vec_dot_f32, c:1467-1494). */
static float float_row_dot(int type, const uint8_t* row, const float* x, int cols) {
    float sum = 0.0f;
    for (int i = 0; i < cols; ++i) {
        float w;
        if (type == L3P_W_F32) {
            memcpy(&w, row + (size_t)i * 4, 4);
        } else if (type == L3P_W_F16) {
            w = l3po_fp16_to_fp32(rd16(row + (size_t)i * 2));
        } else {
            uint32_t u = (uint32_t)rd16(row + (size_t)i * 2) << 16;
            memcpy(&w, &u, 4);
        }
        sum += x[i] * w;
    }
    return sum;
}

int l3po_matvec(int type, const void* w, int rows, int cols, const float* x, float* out) {
    long long rb = l3po_w_row_bytes(type, cols);
    if (rb <= 0 || !w || !x || !out || rows < 0) return -1;
    if (type == L3P_W_F32 || type == L3P_W_F16 || type == L3P_W_BF16) {
        for (int r = 0; r < rows; ++r) out[r] = float_row_dot(type, (const uint8_t*)w + (size_t)r * rb, x, cols);
        return 0;
    }
    if (type == L3P_W_Q4_0 || type == L3P_W_Q4_1 || type == L3P_W_Q5_0 || type == L3P_W_Q5_1 || type == L3P_W_IQ4_NL) {
        uint8_t* xq = (uint8_t*)malloc((size_t)(cols / 32) * QBLOCK);
        if (!xq) return -4;
        l3po_q8_quantize(x, xq, cols);
        for (int r = 0; r < rows; ++r) out[r] = q8x_row_dot(type, (const uint8_t*)w + (size_t)r * rb, xq, cols);
        free(xq);
        return 0;
    }
    float* buf = (float*)malloc(sizeof(float) * (size_t)cols);
    if (!buf) return -4;
    for (int r = 0; r < rows; ++r) {
        const uint8_t* row = (const uint8_t*)w + (size_t)r * rb;
        if (type == L3P_W_Q8_0) deq_q8_0(row, buf, cols);
        else if (type == L3P_W_Q2_K) deq_q2_k(row, buf, cols);
        else if (type == L3P_W_Q3_K) deq_q3_k(row, buf, cols);
        else if (type == L3P_W_Q4_K) deq_q4_k(row, buf, cols);
        else if (type == L3P_W_Q5_K) deq_q5_k(row, buf, cols);
        else deq_q6_k(row, buf, cols);
        float s = 0.0f;
        for (int j = 0; j < cols; ++j) s += buf[j] * x[j];
        out[r] = s;
    }
    free(buf);
    return 0;
}
