// l3p_wo.cu -- the wo projection of the C ABI: weights (l3p_attn_set_wo), the
// GEMV launcher and its entry points (wo.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "ctx.h"
#include "wo.cuh"

using namespace l3p;

namespace {

// The GEMV kernels, (format, 4 or 8 warps): index 2 * wo_format_index + (8 warps)
using WoKernel = void (*)(const WoArgs);
const WoKernel kWoKernels[kWoKernelCount] = {
    wo_gemv_kernel<WoQ8, 4>,                wo_gemv_kernel<WoQ8, 8>,
    wo_gemv_kernel<WoQ4K, 4>,               wo_gemv_kernel<WoQ4K, 8>,
    wo_gemv_kernel<WoQ6K, 4>,               wo_gemv_kernel<WoQ6K, 8>,
    wo_gemv_kernel<WoQ5K, 4>,               wo_gemv_kernel<WoQ5K, 8>,
    wo_gemv_kernel<WoQ2K, 4>,               wo_gemv_kernel<WoQ2K, 8>,
    wo_gemv_kernel<WoQ3K, 4>,               wo_gemv_kernel<WoQ3K, 8>,
    wo_gemv_kernel<WoQ8x<kQxQ4_0>, 4>,      wo_gemv_kernel<WoQ8x<kQxQ4_0>, 8>,
    wo_gemv_kernel<WoQ8x<kQxQ4_1>, 4>,      wo_gemv_kernel<WoQ8x<kQxQ4_1>, 8>,
    wo_gemv_kernel<WoQ8x<kQxQ5_0>, 4>,      wo_gemv_kernel<WoQ8x<kQxQ5_0>, 8>,
    wo_gemv_kernel<WoQ8x<kQxQ5_1>, 4>,      wo_gemv_kernel<WoQ8x<kQxQ5_1>, 8>,
    wo_gemv_kernel<WoQ8x<kQxIQ4NL>, 4>,     wo_gemv_kernel<WoQ8x<kQxIQ4NL>, 8>,
    wo_gemv_kernel<WoFloat<kFlF32>, 4>,     wo_gemv_kernel<WoFloat<kFlF32>, 8>,
    wo_gemv_kernel<WoFloat<kFlF16>, 4>,     wo_gemv_kernel<WoFloat<kFlF16>, 8>,
    wo_gemv_kernel<WoFloat<kFlBF16>, 4>,    wo_gemv_kernel<WoFloat<kFlBF16>, 8>};

int wo_format_index(int type) {
  switch (type) {
    case L3P_W_Q8_0: return 0;
    case L3P_W_Q4_K: return 1;
    case L3P_W_Q6_K: return 2;
    case L3P_W_Q5_K: return 3;
    case L3P_W_Q2_K: return 4;
    case L3P_W_Q3_K: return 5;
    case L3P_W_Q4_0: return 6;
    case L3P_W_Q4_1: return 7;
    case L3P_W_Q5_0: return 8;
    case L3P_W_Q5_1: return 9;
    case L3P_W_IQ4_NL: return 10;
    case L3P_W_F32: return 11;
    case L3P_W_F16: return 12;
    default: return 13;  // L3P_W_BF16
  }
}

}  // namespace

namespace l3p_api {

// The wo GEMV of `layer` (wo.cuh): y[dim] = W[:, owned columns] . x[owned columns].
int launch_wo(l3p_attn_ctx* ctx, int layer, const float* x, float* y, cudaStream_t s, bool tp) {
  const l3p_attn_ctx::WoLayer& L = ctx->wo[layer];
  WoArgs a{};
  if (tp) {
    // y = the group's sum, exchanged through the members' regions (wo.cuh)
    a.tp_members = ctx->tp_members;
    a.tp_member = ctx->tp_member;
    for (int m = 0; m < ctx->tp_members; ++m) a.tp_regions[m] = static_cast<uint8_t*>(ctx->tp_peer[m]);
  }
  a.err = ctx->err_dev;
  a.w = L.w;
  a.wsc = L.wsc;
  a.row_bytes = L.row_bytes;
  a.sc_stride = L.sc_stride;
  a.rows = L.rows;
  a.C = ctx->kvh_count * ctx->G * ctx->hd;
  a.x = x + (long long)ctx->cfg.kv_head_begin * ctx->G * ctx->hd;
  a.y = y;
  const int fi = wo_format_index(L.type);
  const int slice = L.type == L3P_W_Q6_K ? WoQ6K::kSlice : WoQ8::kSlice;
  const int slices = (a.C + slice - 1) / slice;
  a.wc = 1;
  while (a.wc < slices) a.wc <<= 1;
  const int nw = a.wc <= 4 ? 4 : 8;  // warps per CTA
  const int k = fi * 2 + (nw == 8);
  // every SM holds as many CTAs as fit; a CTA takes a contiguous block of rows
  const int target = ctx->num_sms * std::max(ctx->wo_ctas_per_sm[k], 1);
  a.rows_per_cta = std::max(1, (a.rows + target - 1) / target);
  const int grid = (a.rows + a.rows_per_cta - 1) / a.rows_per_cta;
  if (tp && grid > kTpMaxBlocks)
    return fail(ctx, L3P_E_UNSUPPORTED, "tensor-parallel wo grid of %d CTAs exceeds %d", grid, kTpMaxBlocks);
  a.trace = trace_slot(ctx, grid, 1, 1, layer, -1);
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(grid, 1, 1);
  lc.blockDim = dim3(nw * 32, 1, 1);
  lc.dynamicSmemBytes = (size_t)nw * a.rows_per_cta * sizeof(float);
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  if (ctx->overlap) {
    // weights are requested before griddepcontrol.wait; x is read after it
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, kWoKernels[k], a));
  ++ctx->launches;
  return L3P_OK;
}

int check_wo(l3p_attn_ctx* ctx, int layer) {
  if (int rc = check_layer(ctx, layer)) return rc;
  if (ctx->wo.empty() || !ctx->wo[layer].set)
    return fail(ctx, L3P_E_INVAL, "l3p_attn_set_wo has not been called for layer %d", layer);
  return L3P_OK;
}

}  // namespace l3p_api

using namespace l3p_api;

L3P_API int l3p_attn_set_wo(l3p_attn_ctx* ctx, int layer, int type, const void* rows, int dim) {
  if (!ctx || !rows || dim <= 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  int vals, bytes, dev_bytes;  // values and bytes per GGUF block, bytes per device block
  switch (type) {
    case L3P_W_Q8_0: vals = 32, bytes = 34, dev_bytes = 32; break;
    case L3P_W_Q2_K: vals = 256, bytes = 84, dev_bytes = WoQ2K::kBlockBytes; break;
    case L3P_W_Q3_K: vals = 256, bytes = 110, dev_bytes = WoQ3K::kBlockBytes; break;
    case L3P_W_Q4_K: vals = 256, bytes = 144, dev_bytes = 144; break;
    case L3P_W_Q5_K: vals = 256, bytes = 176, dev_bytes = WoQ5K::kBlockBytes; break;
    case L3P_W_Q6_K: vals = 256, bytes = 210, dev_bytes = WoQ6K::kBlockBytes; break;
    case L3P_W_Q4_0:
    case L3P_W_IQ4_NL: vals = 32, bytes = 18, dev_bytes = 16; break;
    case L3P_W_Q4_1: vals = 32, bytes = 20, dev_bytes = 16; break;
    case L3P_W_Q5_0: vals = 32, bytes = 22, dev_bytes = 16; break;
    case L3P_W_Q5_1: vals = 32, bytes = 24, dev_bytes = 16; break;
    case L3P_W_F32: vals = 1, bytes = 4, dev_bytes = 4; break;
    case L3P_W_F16:
    case L3P_W_BF16: vals = 1, bytes = 2, dev_bytes = 2; break;
    default:
      return fail(ctx, L3P_E_UNSUPPORTED,
                  "wo weight type %d (the GGUF types F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, "
                  "Q8_0 = 8, Q2_K .. Q6_K = 10 .. 14, IQ4_NL = 20, BF16 = 29 are supported)",
                  type);
  }
  const int hd = ctx->hd, cols = ctx->cfg.n_heads * hd;
  const int c_lo = ctx->cfg.kv_head_begin * ctx->G * hd, C = ctx->kvh_count * ctx->G * hd;
  const int max_c = 8 * (type == L3P_W_Q6_K ? WoQ6K::kSlice : WoQ8::kSlice);
  // float rows: whole 32-column lane runs (a lane loads 32 values)
  if (cols % vals || c_lo % vals || C % vals || C > max_c || (vals == 1 && (C % 32 || c_lo % 32)))
    return fail(ctx, L3P_E_UNSUPPORTED, "owned wo columns [%d, %d) do not fall on %d-value blocks or exceed %d", c_lo,
                c_lo + C, vals, max_c);
  const uint8_t* src = static_cast<const uint8_t*>(rows);
  const size_t src_row = (size_t)(cols / vals) * bytes, nb = (size_t)C / vals, b0 = (size_t)c_lo / vals;
  // device layout of wo.cuh
  std::vector<uint8_t> w, sc;
  long long row_bytes;
  int sc_stride = 0;
  if (type == L3P_W_Q8_0) {
    row_bytes = C;
    sc_stride = (int)((nb * 2 + 15) / 16 * 16);
    w.resize((size_t)dim * C);
    sc.assign((size_t)dim * sc_stride, 0);
    for (int r = 0; r < dim; ++r)
      for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + (size_t)r * src_row + (b0 + b) * bytes;
        sc[(size_t)r * sc_stride + 2 * b] = blk[0];  // fp16 scale, little-endian
        sc[(size_t)r * sc_stride + 2 * b + 1] = blk[1];
        memcpy(&w[(size_t)r * C + b * 32], blk + 2, 32);
      }
  } else if (vals == 1) {
    // float rows: the owned columns as they are
    row_bytes = (long long)C * bytes;
    w.resize((size_t)dim * row_bytes);
    for (int r = 0; r < dim; ++r)
      memcpy(&w[(size_t)r * row_bytes], src + (size_t)r * src_row + (size_t)c_lo * bytes, (size_t)C * bytes);
  } else if (vals == 32) {
    // Q4_0, Q4_1, Q5_0, Q5_1, IQ4_NL: the 16 quant bytes of every block, and
    // per block 8 bytes [d, m, qh] (m and qh 0 where the type has none)
    row_bytes = (long long)nb * 16;
    sc_stride = (int)(nb * 8);
    w.resize((size_t)dim * row_bytes);
    sc.assign((size_t)dim * sc_stride, 0);
    const int m_off = (type == L3P_W_Q4_1 || type == L3P_W_Q5_1) ? 2 : -1;
    const int qh_off = type == L3P_W_Q5_0 ? 2 : type == L3P_W_Q5_1 ? 4 : -1;
    for (int r = 0; r < dim; ++r)
      for (size_t b = 0; b < nb; ++b) {
        const uint8_t* blk = src + (size_t)r * src_row + (b0 + b) * bytes;
        uint8_t* meta = &sc[(size_t)r * sc_stride + b * 8];
        memcpy(meta, blk, 2);
        if (m_off >= 0) memcpy(meta + 2, blk + m_off, 2);
        if (qh_off >= 0) memcpy(meta + 4, blk + qh_off, 4);
        memcpy(&w[(size_t)r * row_bytes + b * 16], blk + bytes - 16, 16);
      }
  } else {
    // K-quants: each GGUF block at the start of a 16-byte aligned device block
    row_bytes = (long long)nb * dev_bytes;
    w.assign((size_t)dim * row_bytes, 0);
    for (int r = 0; r < dim; ++r)
      for (size_t b = 0; b < nb; ++b)
        memcpy(&w[(size_t)r * row_bytes + b * dev_bytes], src + (size_t)r * src_row + (b0 + b) * bytes, bytes);
  }
  CtxScope dev(ctx);
  L3P_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (ctx->wo.empty()) {
    ctx->wo.resize(ctx->cfg.n_layers);
    if (cudaMalloc(&ctx->wo_x, (size_t)cols * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      ctx->wo.clear();
      return fail(ctx, L3P_E_NOMEM, "wo input buffer allocation failed");
    }
    // resident CTAs per SM of each kernel (grid sizing)
    for (int i = 0; i < kWoKernelCount; ++i)
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctx->wo_ctas_per_sm[i], kWoKernels[i], (i % 2 ? 8 : 4) * 32,
                                                        (size_t)(i % 2 ? 8 : 4) * 64 * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        ctx->wo_ctas_per_sm[i] = 1;
      }
  }
  l3p_attn_ctx::WoLayer& L = ctx->wo[layer];
  cudaFree(L.w);
  cudaFree(L.wsc);
  L = l3p_attn_ctx::WoLayer();
  if (cudaMalloc(&L.w, w.size()) != cudaSuccess || (!sc.empty() && cudaMalloc(&L.wsc, sc.size()) != cudaSuccess)) {
    cudaGetLastError();
    cudaFree(L.w);
    L = l3p_attn_ctx::WoLayer();
    return fail(ctx, L3P_E_NOMEM, "wo weight allocation of %zu bytes failed", w.size());
  }
  L3P_CUDA(ctx, cudaMemcpy(L.w, w.data(), w.size(), cudaMemcpyHostToDevice));
  if (!sc.empty()) L3P_CUDA(ctx, cudaMemcpy(L.wsc, sc.data(), sc.size(), cudaMemcpyHostToDevice));
  L.set = true;
  L.type = type;
  L.rows = dim;
  L.row_bytes = row_bytes;
  L.sc_stride = sc_stride;
  return L3P_OK;
}

L3P_API int l3p_attn_wo_dev(l3p_attn_ctx* ctx, int layer, const float* x, float* xout, void* stream) {
  if (!ctx || !x || !xout) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_wo(ctx, layer)) return rc;
  if (int rc = check_aligned(ctx, {x, xout})) return rc;
  CtxScope dev(ctx);
  return launch_wo(ctx, layer, x, xout, pick_stream(ctx, stream));
}

// ==========================================================================
// Host-pointer entry points

L3P_API int l3p_attn_wo(l3p_attn_ctx* ctx, int layer, const float* x, float* xout) {
  if (!ctx || !x || !xout) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_wo(ctx, layer)) return rc;
  CtxScope dev(ctx);
  const size_t qd = (size_t)ctx->cfg.n_heads * ctx->hd, dim = ctx->wo[layer].rows;
  if (int rc = ensure_host_staging(ctx, qd + dim)) return rc;
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  const size_t row0 = (size_t)r0 * ctx->hd, nrow = (size_t)(r1 - r0) * ctx->hd;
  memcpy(ctx->hst + row0, x + row0, nrow * 4);
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->wo_x + row0, ctx->hst + row0, nrow * 4, cudaMemcpyHostToDevice, ctx->stream));
  // the kernel writes xout into mapped pinned memory
  if (int rc = launch_wo(ctx, layer, ctx->wo_x, ctx->hst_dev + qd, ctx->stream)) return rc;
  if (int rc = finish_host_call(ctx)) return rc;
  memcpy(xout, ctx->hst + qd, dim * 4);
  return L3P_OK;
}

L3P_API int l3p_attn_step_raw_wo(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                                 const float* v, float* xout) {
  if (!ctx || !q || !k || !v || !xout) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (int rc = check_rope(ctx)) return rc;
  if (int rc = check_wo(ctx, layer)) return rc;
  CtxScope dev(ctx);
  const size_t qd = (size_t)ctx->cfg.n_heads * ctx->hd, kvd = (size_t)ctx->cfg.n_kv_heads * ctx->hd;
  const size_t dim = ctx->wo[layer].rows;
  const size_t in = qd + 2 * kvd;  // staged inputs: q | k | v
  if (int rc = ensure_staging(ctx, in)) return rc;
  if (int rc = ensure_host_staging(ctx, in + dim)) return rc;
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  const size_t row0 = (size_t)r0 * ctx->hd, nrow = (size_t)(r1 - r0) * ctx->hd;
  memcpy(ctx->hst + row0, q + row0, nrow * 4);
  memcpy(ctx->hst + qd, k, kvd * 4);
  memcpy(ctx->hst + qd + kvd, v, kvd * 4);
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf, ctx->hst, in * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = step_raw_core(ctx, layer, pos, ctx->st_buf, ctx->st_buf + qd, ctx->st_buf + qd + kvd, ctx->wo_x,
                             ctx->stream, false))
    return rc;
  if (int rc = launch_wo(ctx, layer, ctx->wo_x, ctx->hst_dev + in, ctx->stream)) return rc;
  if (int rc = finish_host_call(ctx)) return rc;
  memcpy(xout, ctx->hst + in, dim * 4);
  return L3P_OK;
}

