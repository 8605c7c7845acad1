/*
 * l3p_oracle.h -- CPU parity oracle for llama3pure's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, and only as the checker / the timed CPU reference.
 *
 * Two implementations share this interface:
 *   - l3po_*   : a plain-C restatement of the reference's attention step
 *                (oracle/l3p_oracle.c), written for this repository;
 *   - l3pref_* : a harness (oracle/ref_harness.c) that compiles the
 *                reference's own llama3pure-c-engine.c in place and drives
 *                the reference's own static primitives
 *                (quantize_to_q8_0_cache, dot_q8_0_q8_0_cache,
 *                accum_q8_0_cache, softmax, vec_dot_f32, malloc_run_state).
 *                It is built into oracle/_ref/ (git-ignored) and pins the
 *                restatement bit-for-bit.
 *
 * Modes:
 *   L3P_MODE_F32 : the reference loop with an fp32 KV cache (the 1e-4 parity
 *                  contract for the fp32 device kernels);
 *   L3P_MODE_Q8  : the reference exactly as shipped (Q8_0 KV cache and Q8_0
 *                  query, int8*int8 block dots).
 *
 * Layouts (all fp32, row-major):
 *   q      [n_heads][head_dim]          post-RoPE, NOT yet scaled
 *   k, v   head-major bulk loads        [n_kv_heads][n_pos][head_dim]
 *   k_row  one token's K or V           [n_kv_heads][head_dim]
 *   out    [n_heads][head_dim]
 */
#ifndef L3P_ORACLE_H
#define L3P_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define L3P_MODE_F32 0
#define L3P_MODE_Q8 1

typedef struct {
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int seq_len;     /* KV capacity in positions */
    float scale;     /* 0 => 1/sqrtf(head_dim) */
    int is_gemma3;
    int swa_window;  /* 0 => no sliding window */
    int swa_pattern; /* 0 => no SWA layers */
} l3p_oracle_cfg;

/* Pre-attention step (the engines' code between the q/k projections and the
 * cache write): Gemma3 QK-RMSNorm then RoPE, q left unscaled.  Fields as the
 * library's l3p_attn_rope_config. */
typedef struct {
    float rope_theta;     /* <= 0 => 1e6 for Gemma3, 5e5 otherwise */
    float rope_theta_swa; /* <= 0 => 10000 */
    float rms_norm_eps;   /* <= 0 => 1e-5f */
    const float* q_norm;  /* [n_layers][head_dim] or NULL */
    const float* k_norm;  /* [n_layers][head_dim] or NULL */
} l3p_oracle_rope;

/* Weight types of the wo projection (GGUF tensor types, ggml numbering). */
#define L3P_W_F32 0     /* float rows */
#define L3P_W_F16 1     /* fp16 rows */
#define L3P_W_Q4_0 2    /* 18-byte blocks of 32: fp16 d, 16 nibble bytes (q - 8) */
#define L3P_W_Q4_1 3    /* 20-byte blocks of 32: fp16 d, m, 16 nibble bytes */
#define L3P_W_Q5_0 6    /* 22-byte blocks of 32: fp16 d, 4 high-bit bytes, 16 nibble bytes (q - 16) */
#define L3P_W_Q5_1 7    /* 24-byte blocks of 32: fp16 d, m, 4 high-bit bytes, 16 nibble bytes */
#define L3P_W_IQ4_NL 20 /* 18-byte blocks of 32: fp16 d, 16 nibble bytes indexing a 16-value table */
#define L3P_W_BF16 29   /* bfloat16 rows */
#define L3P_W_Q8_0 8  /* 34-byte blocks of 32: fp16 d, 32 int8 */
#define L3P_W_Q2_K 10 /* 84-byte blocks of 256: 16 scale|min bytes, 64 bytes of 2-bit quants, fp16 d, dmin */
#define L3P_W_Q3_K 11 /* 110-byte blocks of 256: 32 high-bit bytes, 64 bytes of 2-bit quants, 12 scale bytes, fp16 d */
#define L3P_W_Q4_K 12 /* 144-byte blocks of 256: fp16 d, dmin, 12 scale bytes, 128 nibble bytes */
#define L3P_W_Q5_K 13 /* 176-byte blocks of 256: fp16 d, dmin, 12 scale bytes, 32 high-bit bytes, 128 nibble bytes */
#define L3P_W_Q6_K 14 /* 210-byte blocks of 256: 128 low-nibble, 64 high-bit, 16 int8 scales, fp16 d */

/* ---- restatement (oracle/l3p_oracle.c) ---- */
void* l3po_create(const l3p_oracle_cfg* cfg, int mode);
void l3po_destroy(void* ctx);
int l3po_load_kv(void* ctx, int layer, int pos0, int n_pos, const float* k, const float* v);
int l3po_decode(void* ctx, int layer, int pos, const float* q, const float* k_row,
                const float* v_row, float* out, long long* skipped);
int l3po_prefill(void* ctx, int layer, int start_pos, int n_tok, const float* q,
                 const float* k, const float* v, float* out, long long* skipped);
int l3po_start_t(const l3p_oracle_cfg* cfg, int layer, int pos);
float l3po_fp16_to_fp32(uint16_t h);
uint16_t l3po_fp32_to_fp16(float f);
void l3po_q8_quantize(const float* src, uint8_t* dst, int count);
float l3po_q8_dot(const uint8_t* a, const uint8_t* b, int count);
void l3po_q8_accum(float* out, const uint8_t* v, float w, int count);
void l3po_softmax(float* x, int n);
/* In place on q [n_tok][n_heads*head_dim] and k [n_tok][n_kv_heads*head_dim]
 * of tokens at positions pos0, pos0+1, ... of `layer`. */
int l3po_rope(const l3p_oracle_cfg* cfg, const l3p_oracle_rope* rope, int layer, int pos0, int n_tok,
              float* q, float* k);
/* Bytes of one weight row of `cols` values (0 for an unknown type). */
long long l3po_w_row_bytes(int type, int cols);
/* out[rows] = W x: each row dequantised to fp32, then summed in column order
 * (matmul_deq_4row, c:2136-2176).  W: rows of l3po_w_row_bytes bytes. */
int l3po_matvec(int type, const void* w, int rows, int cols, const float* x, float* out);

/* ---- reference harness (oracle/ref_harness.c -> oracle/_ref/) ---- */
void* l3pref_create(const l3p_oracle_cfg* cfg, int mode);
void l3pref_destroy(void* ctx);
int l3pref_load_kv(void* ctx, int layer, int pos0, int n_pos, const float* k, const float* v);
int l3pref_decode(void* ctx, int layer, int pos, const float* q, const float* k_row,
                  const float* v_row, float* out, long long* skipped);
int l3pref_prefill(void* ctx, int layer, int start_pos, int n_tok, const float* q,
                   const float* k, const float* v, float* out, long long* skipped);
float l3pref_fp16_to_fp32(uint16_t h);
uint16_t l3pref_fp32_to_fp16(float f);
void l3pref_q8_quantize(const float* src, uint8_t* dst, int count);
float l3pref_q8_dot(const uint8_t* a, const uint8_t* b, int count);
void l3pref_q8_accum(float* out, const uint8_t* v, float w, int count);
void l3pref_softmax(float* x, int n);
int l3pref_rope(const l3p_oracle_cfg* cfg, const l3p_oracle_rope* rope, int layer, int pos0, int n_tok,
                float* q, float* k);
int l3pref_matvec(int type, const void* w, int rows, int cols, const float* x, float* out);
int l3pref_threads(void);

#ifdef __cplusplus
}
#endif
#endif
