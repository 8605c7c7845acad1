/*
 * engine_harness.c -- runs the reference C engine's own forward pass on a
 * synthetic model (TEST INFRASTRUCTURE ONLY).
 *
 * Compiled twice by tests/engine/Makefile, both into oracle/_ref/:
 *   libl3p_engine_ref.so    the reference llama3pure-c-engine.c as it is;
 *   libl3p_engine_wired.so  the copy whose attention blocks call
 *                           libllama3pure_attn.so (tests/engine/wire_engine.py).
 * The engine source is included with its main() renamed.  Instead of a GGUF
 * file (none is available here) the harness fills the engine's Config and
 * TransformerWeights with seeded Q8_0 weights -- the same bytes in both
 * builds -- allocates the scratch main() allocates (c:5184-5201), and drives
 * transformer_prefill() (c:3439) over the prompt and transformer() (c:3190)
 * greedily for the generated tokens, returning every generated position's
 * logits.  Tokenizer, sampling and the CLI are not involved.
 */
#define main llama3pure_main
#include L3P_ENGINE_SRC
#undef main

#define L3PE_EXPORT __attribute__((visibility("default")))

typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab_size, seq_len;
    int is_gemma3, swa_window;
    float rope_theta, rope_theta_swa, rms_norm_eps;
    unsigned long long seed;
} l3pe_cfg;

static unsigned long long g_rng;

/* splitmix64 -> uniform in [-1, 1) */
static float urand(void) {
    unsigned long long z = (g_rng += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (float)((z >> 40) * (1.0 / 8388608.0)) - 1.0f;
}

/* rows x cols Q8_0 tensor: per block a random int8 vector and a scale so the
 * values span about +-scale */
static int q8_tensor(QuantizedTensor* t, int rows, int cols, float scale) {
    size_t row_size = (size_t)(cols / QK8_0) * sizeof(block_q8_0);
    block_q8_0* b = (block_q8_0*)malloc(row_size * rows);
    if (!b) return 0;
    for (size_t i = 0; i < (size_t)rows * (cols / QK8_0); i++) {
        b[i].d = fp32_to_fp16(scale * (0.75f + 0.25f * urand()) / 127.0f);
        for (int j = 0; j < QK8_0; j++) b[i].qs[j] = (int8_t)(127.0f * urand());
    }
    memset(t, 0, sizeof(*t));
    t->data = b;
    t->type = GGML_TYPE_Q8_0;
    t->n_elements = rows * cols;
    t->rows = rows;
    t->cols = cols;
    t->row_size = get_row_size(cols, GGML_TYPE_Q8_0);
    t->q8_func = get_vec_dot_q8_func(GGML_TYPE_Q8_0);
    t->dot_func = get_vec_dot_func(GGML_TYPE_Q8_0);
    t->deq_func = get_deq_row_func(GGML_TYPE_Q8_0);
    return 1;
}

static float* norm_weights(int n, float spread) {
    float* v = (float*)malloc(sizeof(float) * n);
    for (int i = 0; i < n; i++) v[i] = 1.0f + spread * urand();
    return v;
}

L3PE_EXPORT int l3pe_init(const l3pe_cfg* c) {
#ifdef L3P_WIRED
    l3p_wired_reset();
#endif
    init_fp16_table();
    g_rng = c->seed;
    memset(&config, 0, sizeof(config));
    config.dim = c->dim;
    config.hidden_dim = c->hidden_dim;
    config.n_layers = c->n_layers;
    config.n_heads = c->n_heads;
    config.n_kv_heads = c->n_kv_heads;
    config.head_dim = c->head_dim;
    config.vocab_size = c->vocab_size;
    config.seq_len = c->seq_len;
    config.rope_theta = c->rope_theta;
    config.is_gemma3 = c->is_gemma3;
    config.swa_window = c->swa_window;
    config.swa_pattern = 6; /* as main() sets it (c:5098) */
    config.rope_theta_swa = c->rope_theta_swa;
    config.rms_norm_eps = c->rms_norm_eps;
    int L = c->n_layers, dim = c->dim, hd = c->head_dim;
    int q_dim = c->n_heads * hd, kv_dim = c->n_kv_heads * hd;
    memset(&weights, 0, sizeof(weights));
    QuantizedTensor emb;
    if (!q8_tensor(&emb, c->vocab_size, dim, 1.0f)) return -4;
    weights.token_embedding_data = emb.data;
    weights.token_embedding_type = GGML_TYPE_Q8_0;
    weights.token_embedding_row_size = emb.row_size;
    weights.rms_att_weight = norm_weights(L * dim, 0.1f);
    weights.rms_ffn_weight = norm_weights(L * dim, 0.1f);
    weights.rms_final_weight = norm_weights(dim, 0.1f);
    weights.wq = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    weights.wk = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    weights.wv = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    weights.wo = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    weights.w1 = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    weights.w2 = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    weights.w3 = (QuantizedTensor*)calloc(L, sizeof(QuantizedTensor));
    /* projections scaled so activations stay O(1) through the layers */
    float s_in = 3.0f / sqrtf((float)dim), s_q = 3.0f / sqrtf((float)q_dim), s_h = 3.0f / sqrtf((float)c->hidden_dim);
    for (int l = 0; l < L; l++) {
        if (!q8_tensor(&weights.wq[l], q_dim, dim, 2.0f * s_in) || !q8_tensor(&weights.wk[l], kv_dim, dim, 2.0f * s_in) ||
            !q8_tensor(&weights.wv[l], kv_dim, dim, s_in) || !q8_tensor(&weights.wo[l], dim, q_dim, s_q) ||
            !q8_tensor(&weights.w1[l], c->hidden_dim, dim, s_in) || !q8_tensor(&weights.w2[l], dim, c->hidden_dim, s_h) ||
            !q8_tensor(&weights.w3[l], c->hidden_dim, dim, s_in))
            return -4;
    }
    if (!q8_tensor(&weights.wcls, c->vocab_size, dim, s_in)) return -4;
    if (c->is_gemma3) {
        weights.attn_q_norm = norm_weights(L * hd, 0.2f);
        weights.attn_k_norm = norm_weights(L * hd, 0.2f);
        weights.attn_post_norm = norm_weights(L * dim, 0.1f);
        weights.ffn_post_norm = norm_weights(L * dim, 0.1f);
    }
    malloc_run_state(&state, &config);
    /* the Q8_0 / dequantisation scratch of main() (c:5184-5201) */
    int max_input = dim;
    if (q_dim > max_input) max_input = q_dim;
    if (c->hidden_dim > max_input) max_input = c->hidden_dim;
    free(q8_buf);
    free(deq_buf);
    q8_buf = (block_q8_0*)calloc((max_input + QK8_0 - 1) / QK8_0, sizeof(block_q8_0));
    deq_buf_stride = 4 * max_input;
    deq_buf = (float*)calloc((size_t)omp_get_max_threads() * deq_buf_stride, sizeof(float));
    return 0;
}

/* Prompt of n_prompt tokens: the first n_prompt-1 through transformer_prefill
 * in batches of PREFILL_BATCH_SIZE (as main() does, c:5262-5272), then n_gen
 * greedy steps through transformer(); out_tokens[n_gen], logits[n_gen][vocab]. */
L3PE_EXPORT int l3pe_run(const int* prompt, int n_prompt, int n_gen, int* out_tokens, float* logits) {
    int* toks = (int*)malloc(sizeof(int) * (n_prompt + n_gen));
    memcpy(toks, prompt, sizeof(int) * n_prompt);
    int pos = 0;
    while (pos < n_prompt - 1) {
        int bs = n_prompt - 1 - pos;
        if (bs > PREFILL_BATCH_SIZE) bs = PREFILL_BATCH_SIZE;
        transformer_prefill(toks, pos, bs, &config, &state, &weights);
        pos += bs;
    }
    int tok = toks[n_prompt - 1];
    for (int g = 0; g < n_gen; g++, pos++) {
        transformer(tok, pos, &config, &state, &weights, 1);
        memcpy(logits + (size_t)g * config.vocab_size, state.logits, sizeof(float) * config.vocab_size);
        int best = 0;
        for (int i = 1; i < config.vocab_size; i++)
            if (state.logits[i] > state.logits[best]) best = i;
        out_tokens[g] = best;
        tok = best;
    }
    free(toks);
    return 0;
}
