// l3p_groups.cu -- the NVLink groups of the C ABI: sequence groups (partial
// attention merged through peer memory, seq_xchg.cuh) and tensor-parallel
// groups (the wo projection summed through peer memory in the tail of its
// GEMV, wo.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "ctx.h"
#include "seq_xchg.cuh"

using namespace l3p;
using namespace l3p_api;

// ==========================================================================
// Sequence groups over NVLink

L3P_API int l3p_attn_seq_group_export(l3p_attn_ctx* ctx, int n_parts, int part, void* handle) {
  if (!ctx || !handle) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (n_parts < 2 || n_parts > kXchgMaxParts || part < 0 || part >= n_parts)
    return fail(ctx, L3P_E_INVAL, "sequence group of %d parts (2..%d), part %d", n_parts, kXchgMaxParts, part);
  if (ctx->kvh_count * ctx->G > kXchgMaxRows)
    return fail(ctx, L3P_E_UNSUPPORTED, "sequence group members own %d q heads (at most %d)", ctx->kvh_count * ctx->G,
                kXchgMaxRows);
  CtxScope dev(ctx);
  if (ctx->xg_region && ctx->xg_parts != n_parts)
    return fail(ctx, L3P_E_INVAL, "the sequence group is already set up with %d parts", ctx->xg_parts);
  if (!ctx->xg_region) {
    // per layer: [n_heads][hd] partial outputs then [n_heads][2] (m, l), padded to 16 bytes;
    // then the inbox of [2][n_parts] slots of 64-bit packets
    ctx->xg_slot_floats = ((long long)ctx->cfg.n_heads * (ctx->hd + 2) + 3) / 4 * 4;
    const size_t bytes = kXchgFlagBytes + (size_t)ctx->cfg.n_layers * ctx->xg_slot_floats * sizeof(float) +
                         2ull * n_parts * ctx->xg_slot_floats * 8;
    if (cudaMalloc(&ctx->xg_region, bytes) != cudaSuccess) {
      cudaGetLastError();
      ctx->xg_region = nullptr;
      return fail(ctx, L3P_E_NOMEM, "exchange region of %zu bytes", bytes);
    }
    L3P_CUDA(ctx, cudaMemset(ctx->xg_region, 0, bytes));
  }
  ctx->xg_parts = n_parts;
  ctx->xg_part = part;
  ctx->xg_ready = false;
  L3P_CUDA(ctx, cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), ctx->xg_region));
  return L3P_OK;
}

L3P_API int l3p_attn_seq_group_import(l3p_attn_ctx* ctx, const void* handles) {
  if (!ctx || !handles) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (!ctx->xg_region) return fail(ctx, L3P_E_INVAL, "l3p_attn_seq_group_export has not been called");
  CtxScope dev(ctx);
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < ctx->xg_parts; ++p) {
    if (p == ctx->xg_part) {
      ctx->xg_peer[p] = ctx->xg_region;
      continue;
    }
    if (ctx->xg_peer[p]) continue;
    L3P_CUDA(ctx, cudaIpcOpenMemHandle(&ctx->xg_peer[p], h[p], cudaIpcMemLazyEnablePeerAccess));
  }
  ctx->xg_ready = true;
  return L3P_OK;
}

L3P_API int l3p_attn_decode_seq_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* out,
                                    void* stream) {
  if (!ctx || !q || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos < 0 || pos >= ctx->cfg.seq_len) return fail(ctx, L3P_E_RANGE, "pos %d outside [0, %d)", pos, ctx->cfg.seq_len);
  if (!ctx->xg_ready) return fail(ctx, L3P_E_INVAL, "sequence group not connected (export, then import)");
  if (int rc = check_aligned(ctx, {q, out})) return rc;
  CtxScope dev(ctx);
  cudaStream_t s = pick_stream(ctx, stream);
  const long long slot = (long long)layer * ctx->xg_slot_floats;
  float* mine = reinterpret_cast<float*>(ctx->xg_region + kXchgFlagBytes) + slot;
  // the partial attention over this context's positions, into its own slot
  if (int rc = launch_decode(ctx, layer, 0, pos, 0, 1, q, nullptr, mine, mine + (long long)ctx->cfg.n_heads * ctx->hd,
                             s, nullptr, nullptr, true))
    return rc;
  XchgArgs a{};
  const size_t inbox_off = kXchgFlagBytes + (size_t)ctx->cfg.n_layers * ctx->xg_slot_floats * sizeof(float);
  for (int p = 0; p < ctx->xg_parts; ++p)
    a.inbox[p] = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(ctx->xg_peer[p]) + inbox_off);
  a.mine = mine;
  a.my_step = reinterpret_cast<unsigned*>(ctx->xg_region) + 16;
  a.slot_floats = ctx->xg_slot_floats;
  a.n_parts = ctx->xg_parts;
  a.part = ctx->xg_part;
  a.hd = ctx->hd;
  a.n_heads = ctx->cfg.n_heads;
  a.row_begin = ctx->cfg.kv_head_begin * ctx->G;
  a.n_rows = ctx->kvh_count * ctx->G;
  a.out = out;
  a.err = ctx->err_dev;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3((a.n_rows * a.hd + kXchgThreads - 1) / kXchgThreads, 1, 1);
  lc.blockDim = dim3(kXchgThreads, 1, 1);
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  if (ctx->overlap) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, seq_merge_kernel, a));
  ++ctx->launches;
  return L3P_OK;
}

L3P_API int l3p_attn_tp_group_export(l3p_attn_ctx* ctx, int n_members, int member, int dim, void* handle) {
  if (!ctx || !handle) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (n_members < 2 || n_members > kXchgMaxParts || member < 0 || member >= n_members || dim <= 0 || dim % 4)
    return fail(ctx, L3P_E_INVAL, "tensor-parallel group of %d members (2..%d), member %d, dim %d (multiple of 4)",
                n_members, kXchgMaxParts, member, dim);
  CtxScope dev(ctx);
  if (ctx->tp_region && (ctx->tp_members != n_members || ctx->tp_dim != dim))
    return fail(ctx, L3P_E_INVAL, "the tensor-parallel group is already set up with another shape");
  if (!ctx->tp_region) {
    const size_t bytes = tp_region_bytes(n_members, dim);
    if (cudaMalloc(&ctx->tp_region, bytes) != cudaSuccess) {
      cudaGetLastError();
      ctx->tp_region = nullptr;
      return fail(ctx, L3P_E_NOMEM, "tensor-parallel exchange region of %zu bytes", bytes);
    }
    L3P_CUDA(ctx, cudaMemset(ctx->tp_region, 0, bytes));
  }
  ctx->tp_members = n_members;
  ctx->tp_member = member;
  ctx->tp_dim = dim;
  ctx->tp_ready = false;
  L3P_CUDA(ctx, cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), ctx->tp_region));
  return L3P_OK;
}

L3P_API int l3p_attn_tp_group_import(l3p_attn_ctx* ctx, const void* handles) {
  if (!ctx || !handles) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (!ctx->tp_region) return fail(ctx, L3P_E_INVAL, "l3p_attn_tp_group_export has not been called");
  CtxScope dev(ctx);
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int p = 0; p < ctx->tp_members; ++p) {
    if (p == ctx->tp_member) {
      ctx->tp_peer[p] = ctx->tp_region;
      continue;
    }
    if (ctx->tp_peer[p]) continue;
    L3P_CUDA(ctx, cudaIpcOpenMemHandle(&ctx->tp_peer[p], h[p], cudaIpcMemLazyEnablePeerAccess));
  }
  ctx->tp_ready = true;
  return L3P_OK;
}

L3P_API int l3p_attn_wo_allreduce_dev(l3p_attn_ctx* ctx, int layer, const float* x, float* xout, void* stream) {
  if (!ctx || !x || !xout) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_wo(ctx, layer)) return rc;
  if (!ctx->tp_ready) return fail(ctx, L3P_E_INVAL, "tensor-parallel group not connected (export, then import)");
  if (ctx->wo[layer].rows != ctx->tp_dim)
    return fail(ctx, L3P_E_INVAL, "wo of layer %d has %d rows, the group was set up for %d", layer,
                ctx->wo[layer].rows, ctx->tp_dim);
  if (int rc = check_aligned(ctx, {x, xout})) return rc;
  CtxScope dev(ctx);
  cudaStream_t s = pick_stream(ctx, stream);
  // one launch: the GEMV and, in its tail, the sum over the group
  return launch_wo(ctx, layer, x, xout, s, true);
}

