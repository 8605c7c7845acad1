/*
 * llama3pure_attn.h -- C ABI of libllama3pure_attn.so, the B200 (sm_100a)
 * attention step for llama3pure's C and JavaScript engines.
 *
 * The reference has no attention function: attention is inlined in
 * transformer() (llama3pure-c-engine.c:3299-3359), transformer_prefill()
 * (c:3562-3612) and the four JS forward functions (llama3pure-js-engine.js:
 * 5099-5188, 5375-5457, 5624-5721, 5951-6041).  This library is the seam cut
 * at exactly those lines:
 *   upstream   post-RoPE q, k, v of one token (or a prompt batch) for layer l
 *              (or, through the *_raw entry points, q/k/v straight from the
 *              projections: QK-norm, RoPE and the cache write then run here);
 *   downstream the attention output xb[n_heads*head_dim] fed to `wo`
 *              (c:3362, js:5191).
 *
 * Conventions
 *   - Plain C types only; all sizes in elements unless named *_bytes.
 *   - q is post-RoPE and NOT yet multiplied by the attention scale; the
 *     library multiplies it by cfg.scale first, as the reference's RoPE loop
 *     does (c:3264-3265, c:3288-3289).  An engine that already fused the scale
 *     into its RoPE passes scale = 1.0f.
 *   - Functions without a suffix take HOST pointers and return when the result
 *     is in host memory.  *_dev functions take DEVICE pointers (16-byte
 *     aligned) and a cudaStream_t passed as void* (NULL = the context's
 *     stream) and return after enqueueing.
 *   - Every function returns L3P_OK (0) or a negative L3P_E_* code and never
 *     exits the process (the reference calls exit(1) on allocation failure,
 *     c:373-379, c:499-500); l3p_attn_last_error() describes the failure.
 *   - A context is driven by one host thread (the reference calls attention
 *     from a single thread with OpenMP inside, c:3327-3328; the JS engine is
 *     single threaded, js:7199).
 */
#ifndef LLAMA3PURE_ATTN_H
#define LLAMA3PURE_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define L3P_OK 0
#define L3P_E_INVAL (-1)       /* bad argument or configuration */
#define L3P_E_RANGE (-2)       /* layer / position outside the cache */
#define L3P_E_CUDA (-3)        /* a CUDA runtime call failed */
#define L3P_E_NOMEM (-4)       /* device or host allocation failed */
#define L3P_E_TIMEOUT (-5)     /* a bounded device-side wait gave up */
#define L3P_E_UNSUPPORTED (-6) /* geometry without a kernel in this build */

#define L3P_KV_F32 0  /* fp32 KV cache: the 1e-4 contract against the reference's fp32 loop */
#define L3P_KV_Q8_0 1 /* the reference's own cache format (c:120-123, c:365-372): per 32-value
                         block an fp16 scale (truncating conversion, c:585-599) and 32 int8;
                         K/V rows and q quantised as quantize_to_q8_0_cache (c:1535-1570),
                         scores and V sums as dot_q8_0_q8_0_cache / accum_q8_0_cache
                         (c:1574-1622) */

/* Attention geometry and placement.  Field meanings follow the reference's
 * Config (c:211-229) and RunState (c:280-338). */
typedef struct l3p_attn_config {
    int n_layers;    /* Config.n_layers (c:214) */
    int n_heads;     /* Config.n_heads: query heads (c:215) */
    int n_kv_heads;  /* Config.n_kv_heads (c:216); n_heads % n_kv_heads == 0 */
    int head_dim;    /* Config.head_dim (c:220); 64, 128 or 256 */
    int seq_len;     /* Config.seq_len: KV capacity in positions (c:218) */
    float scale;     /* RunState.attn_scale; 0 => 1.0f/sqrtf(head_dim) (c:434) */
    int is_gemma3;   /* Config.is_gemma3 (c:222) */
    int swa_window;  /* Config.swa_window; 0 = no sliding window (c:226) */
    int swa_pattern; /* Config.swa_pattern (c:228); SWA layers: l%p < p-1 */
    int device;      /* CUDA device ordinal that holds this context's cache */
    int kv_head_begin; /* first KV head owned by this context (head sharding) */
    int kv_head_count; /* KV heads owned; 0 => n_kv_heads - kv_head_begin */
    int seq_begin;     /* first position owned (sequence sharding) */
    int seq_count;     /* positions owned; 0 => seq_len - seq_begin */
    int kv_format;     /* L3P_KV_F32 or L3P_KV_Q8_0 */
} l3p_attn_config;

typedef struct l3p_attn_ctx l3p_attn_ctx;

/* Allocate the device KV cache, [layer][owned kv head][owned position]
 * [head_dim] fp32, the same order as the reference's Q8_0 cache
 * [layer][kv_head][pos][bytes] (c:365-372).  Replaces the KV part of
 * malloc_run_state (c:346-502). */
int l3p_attn_create(const l3p_attn_config* cfg, l3p_attn_ctx** out);
void l3p_attn_destroy(l3p_attn_ctx* ctx);
const char* l3p_attn_last_error(const l3p_attn_ctx* ctx);
/* Synchronise the context's stream and report any device-side error flag
 * (L3P_E_TIMEOUT after a bounded wait gave up), clearing it. */
int l3p_attn_check(l3p_attn_ctx* ctx);
/* Stream used by the host-pointer entry points (NULL = a stream the context
 * created itself). */
int l3p_attn_set_stream(l3p_attn_ctx* ctx, void* stream);

/* Write token `pos`'s K and V rows (k, v: [n_kv_heads*head_dim], all heads;
 * the context stores the heads and position it owns).  Replaces the per-head
 * cache write of c:3299-3308 / js:5099-5119. */
int l3p_attn_kv_append(l3p_attn_ctx* ctx, int layer, int pos, const float* k, const float* v);
int l3p_attn_kv_append_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* k, const float* v,
                           void* stream);

/* Single-token decode attention at `pos` over cached positions
 * [start_t, pos] (start_t from the SWA rule, c:3316-3321).  q, out:
 * [n_heads*head_dim]; only the rows of the owned heads are written.  The
 * context must own the whole sequence (seq_begin == 0, seq_count covering
 * pos).  Replaces c:3310-3359 / js:5122-5188, js:5647-5721. */
int l3p_attn_decode(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* out);
int l3p_attn_decode_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* out,
                        void* stream);

/* The whole per-layer attention block of the engines in one host call:
 * append token `pos`'s K/V rows, then decode q at `pos` (c:3299-3359,
 * js:5099-5188); one host<->device round trip instead of two. */
int l3p_attn_step(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                  const float* v, float* out);
/* Device form of l3p_attn_step: ONE kernel launch that takes the new K/V row
 * straight from k, v ([n_kv_heads*head_dim]), uses it for position pos and
 * stores it into the cache (an L3P_KV_Q8_0 cache: quantised first, the bytes
 * of kv_append, c:3299-3312). */
int l3p_attn_step_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                      const float* v, float* out, void* stream);

/* Decode for `n_layers` consecutive layers in one launch (q, out:
 * [n_layers][n_heads*head_dim]).  For latency-bound shapes whose per-layer
 * work is smaller than one launch; same arithmetic as l3p_attn_decode. */
int l3p_attn_decode_layers_dev(l3p_attn_ctx* ctx, int layer0, int n_layers, int pos,
                               const float* q, float* out, void* stream);

/* Sequence-sharded decode: attention over the positions this context owns
 * within [start_t, pos], emitted as a partial triple per owned q head:
 *   part_o  [n_heads][head_dim]  normalised partial output,
 *   part_ml [n_heads][2]         (m, l): m = running max of score*log2(e),
 *                                l = sum of 2^(score*log2(e) - m);
 * an empty range yields m = -inf, l = 0, o = 0.  Combine the partials of all
 * shards with l3p_attn_lse_merge_dev (after an all-gather between GPUs). */
int l3p_attn_decode_partial_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q,
                                float* part_o, float* part_ml, void* stream);

/* Log-sum-exp merge of n_parts partial triples (layouts as above, stacked on
 * a leading [n_parts] axis) into out [rows][head_dim] for rows
 * [row_begin, row_begin + n_rows).  Has no counterpart in the reference,
 * whose softmax is monolithic (c:3350). */
int l3p_attn_lse_merge_dev(l3p_attn_ctx* ctx, int n_parts, int rows_per_part, int row_begin,
                           int n_rows, const float* parts_o, const float* parts_ml, float* out,
                           void* stream);

/* Causal prompt prefill of n_tok tokens at positions [start_pos,
 * start_pos+n_tok): appends their K/V rows, then each token attends to
 * [start_t(pos), pos] -- the reference's token-by-token loop c:3499-3613 /
 * js:5318-5458, js:5895-6042.  q, out: [n_tok][n_heads*head_dim];
 * k, v: [n_tok][n_kv_heads*head_dim]. */
int l3p_attn_prefill(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                     const float* k, const float* v, float* out);
int l3p_attn_prefill_dev(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok,
                         const float* q, const float* k, const float* v, float* out,
                         void* stream);

/* Bulk cache fill / read-back for positions [pos0, pos0+n_pos) of one layer,
 * head-major k, v: [n_kv_heads][n_pos][head_dim] (all heads; the context
 * copies the slice it owns).  Benchmarks and tests use these; the engines do
 * not (they append token by token). */
int l3p_attn_load_kv(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, const float* k,
                     const float* v);
int l3p_attn_read_kv(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, float* k, float* v);
/* With an L3P_KV_Q8_0 cache, load_kv quantises the rows as kv_append does and
 * read_kv returns the dequantised values d * int8. */

/* An L3P_KV_Q8_0 cache in the reference's own bytes: per KV head and position,
 * head_dim/32 blocks of 34 bytes (fp16 scale little-endian, then 32 int8) --
 * the rows of the reference's key_cache / value_cache (c:365-372).  k_blocks,
 * v_blocks: [n_kv_heads][n_pos][head_dim/32*34] (all heads; the context
 * copies the slice it owns).  An engine that already holds a Q8_0 cache
 * hands it over with load_kv_q8; read_kv_q8 reads the cache back bit for bit. */
int l3p_attn_load_kv_q8(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, const uint8_t* k_blocks,
                        const uint8_t* v_blocks);
int l3p_attn_read_kv_q8(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, uint8_t* k_blocks,
                        uint8_t* v_blocks);

/* Device addresses of one layer's owned cache: [kv_head_count][seq_count]
 * [head_dim] fp32 each (fp32 caches only; L3P_E_UNSUPPORTED for Q8_0). */
int l3p_attn_kv_device_ptr(l3p_attn_ctx* ctx, int layer, float** k, float** v);

/* Overlap mode (off by default).  When enabled, the decode launches of the
 * *_dev decode entry points (decode, step, decode_layers, decode_partial) use
 * programmatic dependent launch: a launch may start while the preceding kernel
 * on its stream is still running and stream the cached rows [start_t, pos)
 * meanwhile; it reads q and the new K/V row only after that kernel has
 * completed.  Enable it only when the kernel that precedes a decode launch
 * does not write this context's KV cache (true when it is the engine's QKV
 * projection or another layer's attention; false right after
 * l3p_attn_kv_append_dev or a prefill of the same layer).  No counterpart in
 * the reference. */
int l3p_attn_set_overlap(l3p_attn_ctx* ctx, int enable);

/* Host-call server (fp32 caches, the whole sequence on the context): with
 * enable != 0, l3p_attn_step and l3p_attn_decode no longer launch a kernel,
 * copy and synchronise per call.  A decode grid stays resident on the
 * context's stream; a call writes its rows into a mailbox in mapped pinned
 * memory, and the grid fetches them, appends, decodes and writes the output
 * back as packets the call polls.  Same arithmetic and results as the
 * launched path with the same split-K.  The resident grid holds every SM, so:
 *   - every other entry point of the context first ends it and waits for it
 *     to leave (the next host call starts it again);
 *   - it leaves by itself after `idle_us` microseconds without a call
 *     (0: 20000), and the next call starts it again;
 *   - work of other contexts or libraries on the same GPU waits until it
 *     leaves: enable it only where this context has the GPU to itself.
 * enable == 0 ends it.  L3P_E_UNSUPPORTED for a Q8_0 cache or a sequence
 * shard.  No counterpart in the reference, whose attention runs in the
 * calling thread. */
int l3p_attn_set_host_server(l3p_attn_ctx* ctx, int enable, long long idle_us);

/* Number of kernels this library has launched since the context was created
 * (the benchmark reports it per step).  No counterpart in the reference. */
long long l3p_attn_launch_count(const l3p_attn_ctx* ctx);

/* The architecture the library's kernels were compiled for, as the CUDA
 * runtime reports it for the decode kernel on `device`: *binary = the SASS
 * version (100 for sm_100a), *ptx = the virtual architecture that SASS was
 * compiled from (100 for compute_100a).  Fails with L3P_E_CUDA when the device
 * cannot run the image.  A runtime check of the build; no counterpart in the
 * reference. */
int l3p_attn_device_arch(int device, int* binary, int* ptx);

/* The split-K decomposition a decode launch at `pos` over `n_slices` layers
 * (or prefill tokens) would use: CTAs per KV-head group (*nsplit) and CTAs
 * per thread-block cluster (*cluster).  Introspection for tests and
 * benchmarks; no counterpart in the reference. */
int l3p_attn_decode_plan(l3p_attn_ctx* ctx, int pos, int n_slices, int* nsplit, int* cluster);

/* ---- The pre-attention step on the device -------------------------------
 * The entry points above take q and k after RoPE.  These take them as the
 * q/k projections produce them and perform the engines' steps between the
 * projections and the cache write on the GPU, bit for bit (IEEE single
 * precision, the reference's operation order, no fused multiply-adds):
 *   Gemma3 QK-RMSNorm, rmsnorm_per_head (c:3150-3165) on every q and k head
 *     with this layer's attn_q_norm / attn_k_norm weights, when the model is
 *     Gemma3 and both weight arrays are given (c:3233-3236, c:3507-3512);
 *   RoPE from per-layer cos/sin tables built exactly as malloc_run_state
 *     builds them (c:381-421; Gemma3 SWA layers use the rope_theta_swa table,
 *     c:456-468): NEOX pairs (i, i+head_dim/2) for Gemma3 (c:3254-3278),
 *     consecutive pairs (2i, 2i+1) otherwise (c:3279-3296);
 *   the K/V cache write (c:3299-3308, c:3562-3567).
 * The attention scale is still applied by the attention itself (so the
 * products are the reference's (x0*cos - x1*sin) * attn_scale). */
typedef struct l3p_attn_rope_config {
    float rope_theta;     /* Config.rope_theta (c:219); <= 0 => 1e6 for Gemma3, 5e5 otherwise (c:5127) */
    float rope_theta_swa; /* Config.rope_theta_swa (c:227); <= 0 => 10000 (c:390) */
    float rms_norm_eps;   /* Config.rms_norm_eps; <= 0 => 1e-5f (c:3198) */
    const float* q_norm;  /* HOST [n_layers][head_dim] attn_q_norm weights (c:274), or NULL */
    const float* k_norm;  /* HOST [n_layers][head_dim] attn_k_norm weights (c:275), or NULL */
} l3p_attn_rope_config;

/* Build the RoPE tables for positions [0, seq_len) on the host, as
 * malloc_run_state does (c:381-421), copy them and the QK-norm weights to the
 * device.  Call before any entry point below; calling it again replaces
 * them.  Device memory: seq_len * head_dim * 4 bytes per table (two tables for
 * Gemma3), plus a buffer for the rotated q/k rows of one token.  The
 * single-token entry points then allocate nothing (they may be captured in a
 * CUDA graph); a prefill of more tokens than any before grows the buffer, so
 * make one call of the largest size before capturing prefills. */
int l3p_attn_set_rope(l3p_attn_ctx* ctx, const l3p_attn_rope_config* rope);

/* QK-norm and RoPE of n_tok tokens at positions [pos0, pos0+n_tok) of
 * `layer` into q_out, k_out (same layouts as q: [n_tok][n_heads*head_dim],
 * k: [n_tok][n_kv_heads*head_dim]; only the owned heads' rows are written).
 * q_out is not multiplied by the attention scale.  No cache write. */
int l3p_attn_rope_dev(l3p_attn_ctx* ctx, int layer, int pos0, int n_tok, const float* q, const float* k,
                      float* q_out, float* k_out, void* stream);

/* l3p_attn_step / l3p_attn_step_dev with q, k straight from the projections
 * (before QK-norm and RoPE); v is the V projection.  Two launches: the
 * pre-attention kernel, then the decode (with overlap mode on, the decode
 * streams the cached rows while the pre-attention kernel runs). */
int l3p_attn_step_raw(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                      const float* v, float* out);
int l3p_attn_step_raw_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                          const float* v, float* out, void* stream);

/* l3p_attn_prefill / l3p_attn_prefill_dev with q, k straight from the
 * projections: the pre-attention kernel writes the prompt's K/V rows into
 * the cache itself, then the prefill attention runs. */
int l3p_attn_prefill_raw(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                         const float* k, const float* v, float* out);
int l3p_attn_prefill_raw_dev(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                             const float* k, const float* v, float* out, void* stream);

/* ---- The wo projection: the attention output's consumer ----------------
 * xb2 = Wo . xb (c:3362, js:5191) with the GGUF-quantised attn_output.weight,
 * on the device.  The reference dequantises each weight row to fp32 and forms
 * fp32 dot products (matmul_quantized -> matmul_deq_4row, c:2091-2176, for
 * the types with a row dequantiser); the library multiplies the same values
 * in a different summation order (within 1e-4 of the reference). */
#define L3P_W_F32 0     /* GGML_TYPE_F32 (c:96): float rows */
#define L3P_W_F16 1     /* GGML_TYPE_F16 (c:97): fp16 rows */
#define L3P_W_Q4_0 2    /* GGML_TYPE_Q4_0 (c:98): 18-byte blocks of 32 values */
#define L3P_W_Q4_1 3    /* GGML_TYPE_Q4_1 (c:99): 20-byte blocks of 32 values */
#define L3P_W_Q5_0 6    /* GGML_TYPE_Q5_0 (c:100): 22-byte blocks of 32 values */
#define L3P_W_Q5_1 7    /* GGML_TYPE_Q5_1 (c:101): 24-byte blocks of 32 values */
#define L3P_W_IQ4_NL 20 /* GGML_TYPE_IQ4_NL (c:110): 18-byte blocks of 32 values */
#define L3P_W_BF16 29   /* GGML_TYPE_BF16 (c:111): bfloat16 rows */
#define L3P_W_Q8_0 8  /* GGML_TYPE_Q8_0 (c:102): 34-byte blocks of 32 values */
#define L3P_W_Q2_K 10 /* GGML_TYPE_Q2_K (c:104): 84-byte blocks of 256 values */
#define L3P_W_Q3_K 11 /* GGML_TYPE_Q3_K (c:105): 110-byte blocks of 256 values */
#define L3P_W_Q4_K 12 /* GGML_TYPE_Q4_K (c:106): 144-byte blocks of 256 values */
#define L3P_W_Q5_K 13 /* GGML_TYPE_Q5_K (c:107): 176-byte blocks of 256 values */
#define L3P_W_Q6_K 14 /* GGML_TYPE_Q6_K (c:108): 210-byte blocks of 256 values */

/* Hand layer `layer`'s attn_output.weight to the context: `dim` rows of
 * n_heads*head_dim values in GGUF `type` blocks, as stored in the file
 * (QuantizedTensor.data, c:2912).  The context copies the columns of the q
 * heads it owns (tensor parallelism by head: with one context per GPU every
 * GPU holds 1/N of the columns); they must fall on whole blocks, and at most
 * 8192 owned columns (16384 for Q6_K). */
int l3p_attn_set_wo(l3p_attn_ctx* ctx, int layer, int type, const void* rows, int dim);

/* xout[dim] = Wo[:, owned columns] . x[owned rows], x: [n_heads*head_dim] (the
 * attention output; only the owned heads' rows are read).  With several
 * contexts (GPUs) each xout is a partial sum; the engine adds them (an
 * all-reduce, or a reduce-scatter when the next step is row-sharded). */
int l3p_attn_wo(l3p_attn_ctx* ctx, int layer, const float* x, float* xout);
int l3p_attn_wo_dev(l3p_attn_ctx* ctx, int layer, const float* x, float* xout, void* stream);

/* The engine's block from the q/k/v projections to wo's output in one host
 * call (c:3233-3362: QK-norm, RoPE, cache write, attention, wo); needs
 * l3p_attn_set_rope and l3p_attn_set_wo.  xout: [dim]. */
int l3p_attn_step_raw_wo(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                         const float* v, float* xout);

/* ---- Sequence groups over NVLink -----------------------------------------
 * The contexts that own the same KV heads and consecutive position ranges of
 * one sequence (one per GPU; seq_begin/seq_count) form a group of n_parts.
 * Instead of all-gathering partial triples through a collective library, each
 * member exports a small exchange region (CUDA IPC), imports the others', and
 * then one l3p_attn_decode_seq_dev per member per layer computes the partial
 * attention over its positions, publishes it, waits (bounded; L3P_E_TIMEOUT
 * through l3p_attn_check if a member never arrives) for the others' and
 * merges the group's triples, reading the peers' over NVLink.  Every member
 * must call it for the same layers and positions in the same order.  No
 * counterpart in the reference. */
/* Allocate the exchange region and write its cudaIpcMemHandle (64 bytes) to
 * *handle; n_parts members (2..16), this context is member `part`. */
int l3p_attn_seq_group_export(l3p_attn_ctx* ctx, int n_parts, int part, void* handle);
/* Map the other members' regions: handles = the n_parts 64-byte handles of
 * the group in member order (this context's own entry is ignored). */
int l3p_attn_seq_group_import(l3p_attn_ctx* ctx, const void* handles);
/* Decode attention at `pos` over the whole group's positions; out: the owned
 * q heads' rows of [n_heads*head_dim], on every member. */
int l3p_attn_decode_seq_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* out,
                            void* stream);

/* ---- Tensor-parallel wo over NVLink ----------------------------------------
 * Head-sharded contexts (one per GPU) each hold the wo columns of their heads,
 * so their projections are partial sums.  Members of a group of n_members
 * export (64-byte CUDA IPC handle of a small exchange region for `dim`-row
 * projections) and import each other's regions once; then
 * l3p_attn_wo_allreduce_dev computes this member's partial and, in the same
 * launch, sums the group's partials over NVLink peer memory: every member
 * sends its partial rows to every member and sums all members' rows in member
 * order (so every member gets the same bits) -- an all-reduce of xb2 in one
 * crossing, without a collective library, (n_members - 1) * dim * 8 bytes sent
 * per member.
 * One launch per call; every member calls it for the same layers in the same
 * order, on identical GPUs.  A member that never arrives makes the others'
 * bounded waits give up (L3P_E_TIMEOUT through l3p_attn_check); the group is
 * then out of step and must be set up anew (new contexts).  No counterpart in
 * the reference. */
int l3p_attn_tp_group_export(l3p_attn_ctx* ctx, int n_members, int member, int dim, void* handle);
int l3p_attn_tp_group_import(l3p_attn_ctx* ctx, const void* handles);
/* xout[dim] = sum over the group of Wo[:, member's columns] . x[member's rows]. */
int l3p_attn_wo_allreduce_dev(l3p_attn_ctx* ctx, int layer, const float* x, float* xout, void* stream);

/* Decode attention that allocates nothing.  No counterpart in the reference.
 *
 * For callers that own every byte of device memory themselves -- typically
 * an engine that plans one arena when the model loads and hands out pointers
 * from it -- and so cannot let a library call cudaMalloc while generating: a
 * runtime allocation can synchronise the device, can fail mid-generation once
 * the arena holds the memory, and escapes the caller's accounting.  The
 * caller creates no context and passes everything:
 *   cfg      geometry as for l3p_attn_create (kv_head_begin/kv_head_count
 *            select the KV heads k_cache/v_cache hold; the whole sequence:
 *            seq_begin 0, seq_count 0 or seq_len; device ignored -- the
 *            current device is used);
 *   layer    used only for the sliding-window rule (c:3316-3321);
 *   k_cache, v_cache  one layer's cache, [kv_head_count][seq_len][head_dim]
 *            fp32 on the current device, rows [start_t, pos] filled;
 *   q, out   [n_heads*head_dim] on the device (owned heads' rows written);
 *   stream   cudaStream_t as void*, NULL = legacy default stream.
 * All device pointers 16-byte aligned.  It calls no cudaMalloc, cudaFree or
 * allocating library routine: the split-K partials and tickets live in a
 * fixed 2 MiB + 4 KiB array in the library's device image, which every GPU
 * that loads the library holds until the process exits.  Geometries whose
 * partials would not fit are rejected with L3P_E_RANGE (at most 1024 (KV
 * head, q-head group) units; a plan is chosen within 2 MiB of partials).
 * The first call on each device looks up the array's device address and sets
 * the kernel's shared-memory attribute; make that first call before any stream
 * capture.  That set-up is kept for the life of the process: after a
 * cudaDeviceReset (or a release and re-creation of the device's primary
 * context) this entry point must not be called on that device again.  `layer`
 * must lie in [0, n_layers) (any layer >= 0 when n_layers is 0), else
 * L3P_E_RANGE.  Every call uses the same array: calls whose kernels may overlap on
 * the GPU (other streams, other host threads) race and must be serialised by
 * the caller.  l3p_attn_noalloc_last_error() describes the last failure of the
 * calling thread. */
int l3p_attn_decode_noalloc(const l3p_attn_config* cfg, int layer, int pos, const float* k_cache,
                            const float* v_cache, const float* q, float* out, void* stream);
const char* l3p_attn_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* LLAMA3PURE_ATTN_H */
