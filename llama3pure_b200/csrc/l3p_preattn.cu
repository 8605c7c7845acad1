// l3p_preattn.cu -- the pre-attention step of the C ABI: RoPE tables and
// QK-norm weights (l3p_attn_set_rope), the rotation kernel's launcher and the
// raw-projection entry points (rope.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "ctx.h"
#include "rope.cuh"

using namespace l3p;

namespace l3p_api {

// The pre-attention kernel (rope.cuh) over n_tok tokens at positions
// [pos0, pos0+n_tok) of `layer`: rotated q rows to q_out, rotated k rows to
// k_out when given, and the K (rotated) and V rows into the cache when
// to_cache.
int launch_rope(l3p_attn_ctx* ctx, int layer, int pos0, int n_tok, const float* q, const float* k, const float* v,
                float* q_out, float* k_out, bool to_cache, cudaStream_t s) {
  RopeArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.q_stride = (long long)ctx->cfg.n_heads * ctx->hd;
  a.kv_stride = (long long)ctx->cfg.n_kv_heads * ctx->hd;
  a.q_out = q_out;
  a.k_out = k_out;
  if (to_cache) {
    const long long off = (long long)layer * ctx->layer_elems;
    if (ctx->q8) {
      a.k8 = ctx->k8 + off;
      a.v8 = ctx->v8 + off;
      a.ksc = ctx->ksc + off / 32;
      a.vsc = ctx->vsc + off / 32;
    } else {
      a.kc = ctx->kc + off;
      a.vc = ctx->vc + off;
    }
  }
  a.head_stride = ctx->head_elems;
  a.row0 = pos0 - ctx->cfg.seq_begin;
  a.cap = ctx->seq_count;
  // per-layer table choice of c:456-468: Gemma3 SWA layers use the rope_theta_swa table
  const int pat = ctx->cfg.swa_pattern;
  const bool swa_layer = pat > 0 && layer % pat < pat - 1;
  a.tab = (ctx->cfg.is_gemma3 && swa_layer) ? ctx->rope_tab_swa : ctx->rope_tab;
  a.q_norm = ctx->qk_norm ? ctx->qk_norm + (long long)layer * ctx->hd : nullptr;
  a.k_norm = ctx->qk_norm ? ctx->qk_norm + ((long long)ctx->cfg.n_layers + layer) * ctx->hd : nullptr;
  a.eps = ctx->rms_eps;
  a.inv_hd = 1.0f / (float)ctx->hd;  // s->inv_head_size, c:437
  a.pos0 = pos0;
  a.n_tok = n_tok;
  a.q_head0 = ctx->cfg.kv_head_begin * ctx->G;
  a.n_qh = ctx->kvh_count * ctx->G;
  a.kv_head0 = ctx->cfg.kv_head_begin;
  a.n_kvh = ctx->kvh_count;
  a.neox = ctx->cfg.is_gemma3 ? 1 : 0;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(n_tok, (a.n_qh + a.n_kvh + kRopeWarps - 1) / kRopeWarps, 1);
  lc.blockDim = dim3(kRopeWarps * 32, 1, 1);
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  if (ctx->overlap) {
    // the kernel reads nothing before its griddepcontrol.wait, so it may always overlap
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  switch (ctx->hd) {
    case 64:
      L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, rope_qkv_kernel<64>, a));
      break;
    case 128:
      L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, rope_qkv_kernel<128>, a));
      break;
    default:
      L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, rope_qkv_kernel<256>, a));
      break;
  }
  ++ctx->launches;
  return L3P_OK;
}

int ensure_rope_buf(l3p_attn_ctx* ctx, size_t floats, cudaStream_t s) {
  if (floats <= ctx->rope_buf_floats) return L3P_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone)
    return fail(ctx, L3P_E_INVAL,
                "the rotated-row buffer must grow to %zu floats, which cannot happen during stream capture: "
                "make one call of this size before capturing", floats);
  if (ctx->rope_buf) {
    L3P_CUDA(ctx, cudaStreamSynchronize(s));
    cudaFree(ctx->rope_buf);
  }
  ctx->rope_buf = nullptr;
  ctx->rope_buf_floats = 0;
  const size_t want = std::max(floats, (size_t)1 << 16);
  if (cudaMalloc(&ctx->rope_buf, want * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    return fail(ctx, L3P_E_NOMEM, "rotated-row buffer allocation of %zu floats failed", want);
  }
  ctx->rope_buf_floats = want;
  return L3P_OK;
}

int check_rope(l3p_attn_ctx* ctx) {
  if (!ctx->rope_tab) return fail(ctx, L3P_E_INVAL, "l3p_attn_set_rope has not been called on this context");
  return L3P_OK;
}

// One token's pre-attention step and decode (step_raw entry points).
int step_raw_core(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k, const float* v, float* out,
                  cudaStream_t s, bool allow_overlap) {
  const size_t qd = (size_t)ctx->cfg.n_heads * ctx->hd, kvd = (size_t)ctx->cfg.n_kv_heads * ctx->hd;
  if (int rc = ensure_rope_buf(ctx, qd + kvd, s)) return rc;
  float* rq = ctx->rope_buf;
  float* rk = rq + qd;
  // the decode takes the rotated K row and V from their producers and stores
  // them (fused append; quantised first for a Q8_0 cache)
  if (int rc = launch_rope(ctx, layer, pos, 1, q, k, nullptr, rq, rk, false, s)) return rc;
  return launch_decode(ctx, layer, 0, pos, 0, 1, rq, out, nullptr, nullptr, s, rk, v, allow_overlap);
}

// A prompt's pre-attention step (K/V rows into the cache) and prefill attention.
int prefill_raw_core(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q, const float* k,
                     const float* v, float* out, cudaStream_t s) {
  const size_t nq = (size_t)ctx->cfg.n_heads * ctx->hd * n_tok;
  if (int rc = ensure_rope_buf(ctx, nq, s)) return rc;
  float* rq = ctx->rope_buf;
  if (int rc = launch_rope(ctx, layer, start_pos, n_tok, q, k, v, rq, nullptr, true, s)) return rc;
  if (ctx->prefill_tc) return launch_prefill_tc(ctx, layer, start_pos, n_tok, rq, out, s);
  return launch_decode(ctx, layer, 0, start_pos, 1, n_tok, rq, out, nullptr, nullptr, s);
}

}  // namespace l3p_api

using namespace l3p_api;

L3P_API int l3p_attn_set_rope(l3p_attn_ctx* ctx, const l3p_attn_rope_config* rope) {
  if (!ctx || !rope) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  const int hd = ctx->hd, half = hd / 2, n_pos = ctx->cfg.seq_len, L = ctx->cfg.n_layers;
  const bool gemma = ctx->cfg.is_gemma3 != 0;
  // defaults of c:5127 (rope_theta), c:390 (rope_theta_swa), c:3198 (eps)
  const float theta = rope->rope_theta > 0.f ? rope->rope_theta : (gemma ? 1000000.0f : 500000.0f);
  const float theta_swa = rope->rope_theta_swa > 0.f ? rope->rope_theta_swa : 10000.0f;
  // the tables of malloc_run_state (c:381-421), the same single-precision
  // library calls in the same order
  auto build = [&](float th, std::vector<float2>& tab) {
    std::vector<float> freq(half);
    for (int i = 0; i < half; i++) freq[i] = 1.0f / powf(th, (float)(i * 2) / (float)hd);
    tab.resize((size_t)n_pos * half);
    for (int pos = 0; pos < n_pos; pos++) {
      float2* row = tab.data() + (size_t)pos * half;
      for (int i = 0; i < half; i++) {
        const float val = pos * freq[i];
        row[i] = make_float2(cosf(val), sinf(val));
      }
    }
  };
  std::vector<float2> tab, tab_swa;
  build(theta, tab);
  if (gemma) build(theta_swa, tab_swa);
  CtxScope dev(ctx);
  L3P_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (ctx->rope_tab_swa != ctx->rope_tab) cudaFree(ctx->rope_tab_swa);
  cudaFree(ctx->rope_tab);
  cudaFree(ctx->qk_norm);
  ctx->rope_tab = ctx->rope_tab_swa = nullptr;
  ctx->qk_norm = nullptr;
  const size_t tab_bytes = tab.size() * sizeof(float2);
  if (cudaMalloc(&ctx->rope_tab, tab_bytes) != cudaSuccess ||
      (gemma && cudaMalloc(&ctx->rope_tab_swa, tab_bytes) != cudaSuccess)) {
    cudaGetLastError();
    cudaFree(ctx->rope_tab);
    ctx->rope_tab = ctx->rope_tab_swa = nullptr;
    return fail(ctx, L3P_E_NOMEM, "RoPE table allocation of %zu bytes failed", tab_bytes);
  }
  if (!gemma) ctx->rope_tab_swa = ctx->rope_tab;
  L3P_CUDA(ctx, cudaMemcpy(ctx->rope_tab, tab.data(), tab_bytes, cudaMemcpyHostToDevice));
  if (gemma) L3P_CUDA(ctx, cudaMemcpy(ctx->rope_tab_swa, tab_swa.data(), tab_bytes, cudaMemcpyHostToDevice));
  // QK-norm only for Gemma3 with both weight arrays (c:3233, c:3507)
  if (gemma && rope->q_norm && rope->k_norm) {
    const size_t n = (size_t)L * hd;
    if (cudaMalloc(&ctx->qk_norm, 2 * n * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      ctx->qk_norm = nullptr;
      return fail(ctx, L3P_E_NOMEM, "QK-norm weight allocation failed");
    }
    L3P_CUDA(ctx, cudaMemcpy(ctx->qk_norm, rope->q_norm, n * sizeof(float), cudaMemcpyHostToDevice));
    L3P_CUDA(ctx, cudaMemcpy(ctx->qk_norm + n, rope->k_norm, n * sizeof(float), cudaMemcpyHostToDevice));
  }
  ctx->rms_eps = rope->rms_norm_eps > 0.f ? rope->rms_norm_eps : 1e-5f;
  // the single-token entry points never allocate (they may run inside a CUDA graph capture)
  return ensure_rope_buf(ctx, (size_t)(ctx->cfg.n_heads + ctx->cfg.n_kv_heads) * hd, ctx->stream);
}

L3P_API int l3p_attn_rope_dev(l3p_attn_ctx* ctx, int layer, int pos0, int n_tok, const float* q, const float* k,
                              float* q_out, float* k_out, void* stream) {
  if (!ctx || !q || !k || !q_out || !k_out || n_tok < 0)
    return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos0 < 0 || pos0 + n_tok > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "tokens [%d, %d) outside [0, %d)", pos0, pos0 + n_tok, ctx->cfg.seq_len);
  if (int rc = check_aligned(ctx, {q, k, q_out, k_out})) return rc;
  if (int rc = check_rope(ctx)) return rc;
  if (n_tok == 0) return L3P_OK;
  CtxScope dev(ctx);
  return launch_rope(ctx, layer, pos0, n_tok, q, k, nullptr, q_out, k_out, false, pick_stream(ctx, stream));
}

L3P_API int l3p_attn_step_raw_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                                  const float* v, float* out, void* stream) {
  if (!ctx || !q || !k || !v || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (int rc = check_aligned(ctx, {q, k, v, out})) return rc;
  if (int rc = check_rope(ctx)) return rc;
  CtxScope dev(ctx);
  return step_raw_core(ctx, layer, pos, q, k, v, out, pick_stream(ctx, stream), true);
}

L3P_API int l3p_attn_prefill_raw_dev(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                                     const float* k, const float* v, float* out, void* stream) {
  if (!ctx || !q || !k || !v || !out || n_tok < 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (n_tok == 0) return L3P_OK;
  if (start_pos < 0 || start_pos + n_tok > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "tokens [%d, %d) outside [0, %d)", start_pos, start_pos + n_tok, ctx->cfg.seq_len);
  if (int rc = check_pos_full(ctx, start_pos + n_tok - 1)) return rc;
  if (int rc = check_aligned(ctx, {q, k, v, out})) return rc;
  if (int rc = check_rope(ctx)) return rc;
  CtxScope dev(ctx);
  return prefill_raw_core(ctx, layer, start_pos, n_tok, q, k, v, out, pick_stream(ctx, stream));
}

// ==========================================================================
// Host-pointer entry points

L3P_API int l3p_attn_step_raw(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                              const float* v, float* out) {
  if (!ctx || !q || !k || !v || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (int rc = check_rope(ctx)) return rc;
  CtxScope dev(ctx);
  const size_t qd = (size_t)ctx->cfg.n_heads * ctx->hd, kvd = (size_t)ctx->cfg.n_kv_heads * ctx->hd;
  const size_t in = qd + 2 * kvd;  // staged inputs: q | k | v
  if (int rc = ensure_staging(ctx, in)) return rc;
  if (int rc = ensure_host_staging(ctx, in + qd)) return rc;
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  const size_t row0 = (size_t)r0 * ctx->hd, nrow = (size_t)(r1 - r0) * ctx->hd;
  memcpy(ctx->hst + row0, q + row0, nrow * 4);
  memcpy(ctx->hst + qd, k, kvd * 4);
  memcpy(ctx->hst + qd + kvd, v, kvd * 4);
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf, ctx->hst, in * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = step_raw_core(ctx, layer, pos, ctx->st_buf, ctx->st_buf + qd, ctx->st_buf + qd + kvd,
                             ctx->hst_dev + in, ctx->stream, false))
    return rc;
  if (int rc = finish_host_call(ctx)) return rc;
  memcpy(out + row0, ctx->hst + in + row0, nrow * 4);
  return L3P_OK;
}

L3P_API int l3p_attn_prefill_raw(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                                 const float* k, const float* v, float* out) {
  if (!ctx || !q || !k || !v || !out || n_tok < 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (n_tok == 0) return L3P_OK;
  if (start_pos < 0 || start_pos + n_tok > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "tokens [%d, %d) outside [0, %d)", start_pos, start_pos + n_tok, ctx->cfg.seq_len);
  if (int rc = check_pos_full(ctx, start_pos + n_tok - 1)) return rc;
  if (int rc = check_rope(ctx)) return rc;
  CtxScope dev(ctx);
  const size_t qd = (size_t)ctx->cfg.n_heads * ctx->hd, kvd = (size_t)ctx->cfg.n_kv_heads * ctx->hd;
  const size_t nq = qd * n_tok, nkv = kvd * n_tok;
  if (int rc = ensure_staging(ctx, 2 * nq + 2 * nkv)) return rc;
  float* dq = ctx->st_buf;
  float* dout = dq + nq;
  float* dk = dout + nq;
  float* dv = dk + nkv;
  L3P_CUDA(ctx, cudaMemcpyAsync(dq, q, nq * 4, cudaMemcpyHostToDevice, ctx->stream));
  L3P_CUDA(ctx, cudaMemcpyAsync(dk, k, nkv * 4, cudaMemcpyHostToDevice, ctx->stream));
  L3P_CUDA(ctx, cudaMemcpyAsync(dv, v, nkv * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = prefill_raw_core(ctx, layer, start_pos, n_tok, dq, dk, dv, dout, ctx->stream)) return rc;
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  L3P_CUDA(ctx, cudaMemcpy2DAsync(out + (size_t)r0 * ctx->hd, qd * 4, dout + (size_t)r0 * ctx->hd, qd * 4,
                                  (size_t)(r1 - r0) * ctx->hd * 4, n_tok, cudaMemcpyDeviceToHost, ctx->stream));
  return finish_host_call(ctx);
}

