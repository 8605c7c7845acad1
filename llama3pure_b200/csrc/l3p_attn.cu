// l3p_attn.cu -- the C ABI of libllama3pure_attn.so (include/llama3pure_attn.h):
// context, device KV cache, launch planning, decode / append / prefill and
// their host-pointer wrappers.  The pre-attention step is in l3p_preattn.cu,
// the wo projection in l3p_wo.cu, the NVLink groups in l3p_groups.cu.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "ctx.h"
#include "decode.cuh"
#include "decode_q8.cuh"
#include "prefill_tc.cuh"
#include "server.cuh"

using namespace l3p;
using namespace l3p_api;


namespace l3p_api {

constexpr long long kWsOFloats = 8ll << 20;  // 32 MiB of split partials
constexpr long long kCounters = 1 << 16;
// Global-stage mergers of a one-wave launch (DecodeArgs::merge_k) when a unit
// has at least kMergersFrom parts: measured on the 8B 8K shards, 79 parts
// (one KV head per GPU) merge 0.8 us faster per layer with 4 mergers, while at
// 16 and 32 parts the waiting mergers cost more than they save.
constexpr int kMergers = 4;
constexpr int kMergersFrom = 48;
constexpr int kDecodeThreads = L3P_DECODE_WARPS * 32;  // DecodeCfg<*, *>::kThreads

// --------------------------------------------------------------------------
// Kernel table: one instantiation per (head_dim, q heads per CTA).

using DecodeFn = void (*)(const DecodeArgs);

template <int HD, int GT>
DecodeFn decode_fn() {
  return decode_f32_kernel<HD, GT>;
}

template <int HD, int GT>
int decode_smem() {
  return DecodeCfg<HD, GT>::kSmemBytes;
}

using ServerFn = void (*)(const DecodeArgs, const ServerArgs);

struct KernelInfo {
  DecodeFn fn = nullptr;
  ServerFn srv = nullptr;  // the host-call server over this kernel's body (fp32 caches)
  int threads = kDecodeThreads;
  int smem = 0;
  int rows = 8;
  int ctas_per_sm = 1;
};

KernelInfo kernel_for(int hd, int gt, bool q8 = false) {
  KernelInfo k;
  if (q8) {
#define L3P_CASE8(H, T)                                   \
  if (hd == H && gt == T) {                               \
    k.fn = decode_q8_kernel<H, T>;                        \
    k.threads = DecodeQ8Cfg<H, T>::kThreads;              \
    k.smem = DecodeQ8Cfg<H, T>::kSmemBytes;               \
    k.rows = DecodeQ8Cfg<H, T>::kR;                       \
    k.ctas_per_sm = DecodeQ8Cfg<H, T>::kCtasPerSm;        \
    return k;                                             \
  }
    L3P_CASE8(64, 1) L3P_CASE8(64, 2) L3P_CASE8(64, 4) L3P_CASE8(64, 8)
    L3P_CASE8(128, 1) L3P_CASE8(128, 2) L3P_CASE8(128, 4) L3P_CASE8(128, 8)
    L3P_CASE8(256, 1) L3P_CASE8(256, 2) L3P_CASE8(256, 4) L3P_CASE8(256, 8)
#undef L3P_CASE8
    return k;
  }
#define L3P_CASE(H, T)                                        \
  if (hd == H && gt == T) {                                   \
    k.fn = decode_fn<H, T>();                                 \
    k.srv = decode_server_kernel<H, T>;                       \
    k.smem = decode_smem<H, T>();                             \
    k.rows = DecodeCfg<H, T>::kR;                             \
    k.ctas_per_sm = DecodeCfg<H, T>::kCtasPerSm;              \
    return k;                                                 \
  }
  L3P_CASE(64, 1) L3P_CASE(64, 2) L3P_CASE(64, 4) L3P_CASE(64, 8)
  L3P_CASE(128, 1) L3P_CASE(128, 2) L3P_CASE(128, 4) L3P_CASE(128, 8)
  L3P_CASE(256, 1) L3P_CASE(256, 2) L3P_CASE(256, 4) L3P_CASE(256, 8)
#undef L3P_CASE
  return k;
}

// Split-K plan: how many CTAs share one unit's position range (nsplit) and
// how they are grouped into thread-block clusters (cluster | nsplit).  Tiles
// are dealt round-robin, so every CTA of a unit gets the same share.  The
// estimate minimised is
//   streaming: max(all bytes / ~5.3 TB/s, waves * share bytes / ~42 GB/s)
//   + per-wave latency
//   + cluster launch and merge (~5 us: cluster scheduling costs more than
//     the merge through distributed shared memory saves, at one cluster per
//     unit and at several)
//   + global merge when a unit spans several clusters or has no cluster
//     (fence, ticket and an L2 round trip, ~2.2 us, plus the partials' bytes
//     read by the one merging CTA at ~60 GB/s: measured 2.8 us for 16 parts,
//     4.5 us for 64, 6.6 us for 128 on one 8192-position KV head)
// The bandwidth figures are what one launch sustains on B200 (a 64 MiB
// stream reaches ~5.3 TB/s with 128 to 148 CTAs, i.e. up to ~42 GB/s per SM).
struct Plan {
  int nsplit = 1;
  int cluster = 1;
};

// What a split-K plan may use: the GPU, the kernel geometry and the scratch.
struct PlanLimits {
  int hd = 0, GT = 1, num_sms = 148;
  double row_bytes = 0;  // K + V bytes of one cached position
  int max_clusters[5] = {0, 0, 0, 0, 0};
  long long ws_o_floats = 0, n_counters = 0;
  int force_nsplit = 0, force_cluster = 0;
};

Plan plan_splits(const PlanLimits* ctx, long long P, long long units, int rows_per_tile, int ctas_per_sm) {
  Plan best;
  if (P <= 0) return best;
  if (ctx->force_nsplit > 0) {
    const long long n_tiles = (P + rows_per_tile - 1) / rows_per_tile;
    const int cs = ctx->force_cluster > 0 ? ctx->force_cluster : 1;
    int ci = 0;
    while ((1 << ci) < cs) ++ci;
    const int ns = ctx->force_nsplit;
    const long long gparts = cs > 1 ? ns / cs : ns;
    const bool ok = (1 << ci) == cs && ci < 5 && ns % cs == 0 && ns <= n_tiles && ns <= kMaxSplits &&
                    (cs == 1 || ctx->max_clusters[ci] > 0) && ctx->GT * ctx->hd / 4 >= cs &&
                    (gparts <= 1 || (units * gparts * ctx->GT * ctx->hd <= ctx->ws_o_floats && units <= ctx->n_counters));
    if (ok) {
      best.nsplit = ns;
      best.cluster = cs;
      return best;
    }
  }
  const double row_bytes = ctx->row_bytes > 0 ? ctx->row_bytes : 2.0 * ctx->hd * 4.0;
  const double part_bytes = (double)ctx->GT * ctx->hd * 4.0;
  const long long n_tiles = (P + rows_per_tile - 1) / rows_per_tile;
  const long long slots = (long long)ctx->num_sms * ctas_per_sm;
  const double total_us = (double)units * P * row_bytes / 5300e3;
  double best_cost = 1e300;
  // plain launches only: every cluster plan measured slower than the best
  // plain plan (8B 8K shards of 1-8 KV heads, 1B, Gemma MQA; one B200, step
  // graphs with programmatic dependent launch), by 1-10 us.  L3P_DECODE_PLAN
  // still pins cluster plans (the tests exercise every merge path).
  for (int ci = 0; ci < 1; ++ci) {
    const int cs = 1 << ci;
    if (cs > 1 && (ctx->max_clusters[ci] <= 0 || cs > n_tiles || ctx->GT * ctx->hd / 4 < cs)) continue;
    for (int nc = 1; nc * cs <= kMaxSplits && nc * cs <= n_tiles; ++nc) {
      const int ns = nc * cs;
      const int gparts = cs > 1 ? nc : ns;  // partials of the global stage
      const bool global = gparts > 1;
      if (global && (units * gparts * ctx->GT * ctx->hd > ctx->ws_o_floats || units > ctx->n_counters)) break;
      long long waves;
      if (cs > 1)
        waves = (units * nc + ctx->max_clusters[ci] - 1) / ctx->max_clusters[ci];
      else
        waves = (units * ns + slots - 1) / slots;
      const double share = (double)((n_tiles + ns - 1) / ns) * rows_per_tile * row_bytes;
      double cost = std::max(total_us, waves * share / 42e3) + waves * 1.0;
      if (global) {
        // merged by `mergers` CTAs that each read a slice of every partial:
        // designated mergers in a one-wave launch (as launch_decode sets them)
        const bool one_wave = waves == 1 && cs == 1;
        const int by_size = std::max(1, (ctx->GT * ctx->hd / 4 + kDecodeThreads - 1) / kDecodeThreads);
        const int by_parts = gparts >= 48 ? 4 : gparts >= 24 ? 2 : 1;
        const int mergers = one_wave ? std::min(gparts, std::max(by_size, by_parts)) : 1;
        cost += 2.2 + gparts * part_bytes / 60e3 / mergers;
      }
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best.nsplit = ns;
        best.cluster = cs;
      }
    }
  }
  return best;
}

PlanLimits limits_of(const l3p_attn_ctx* ctx);

// plan_splits costs ~5 us of host time, and the host entry points run it on
// every call.  Its estimate depends on the attended length only through the
// number of tiles, so plans are kept per (tiles, units, kernel) in a small
// cache: a decode step re-plans once every `rows` positions.
Plan cached_plan(l3p_attn_ctx* ctx, long long P, long long units, const KernelInfo& ki) {
  const long long n_tiles = (P + ki.rows - 1) / ki.rows;
  for (auto& e : ctx->plan_cache)
    if (e.n_tiles == n_tiles && e.units == units && e.rows == ki.rows && e.ctas_per_sm == ki.ctas_per_sm)
      return Plan{e.nsplit, e.cluster};
  const PlanLimits lim = limits_of(ctx);
  const Plan p = plan_splits(&lim, n_tiles * ki.rows, units, ki.rows, ki.ctas_per_sm);
  auto& e = ctx->plan_cache[ctx->plan_cache_next++ % 4];
  e.n_tiles = n_tiles;
  e.units = units;
  e.rows = ki.rows;
  e.ctas_per_sm = ki.ctas_per_sm;
  e.nsplit = p.nsplit;
  e.cluster = p.cluster;
  return p;
}

PlanLimits limits_of(const l3p_attn_ctx* ctx) {
  PlanLimits l;
  l.hd = ctx->hd;
  l.GT = ctx->GT;
  // fp32: 4 bytes per value; Q8_0: 1 byte per value + a 2-byte scale per 32
  l.row_bytes = ctx->q8 ? 2.0 * (ctx->hd + ctx->hd / 16) : 2.0 * ctx->hd * 4.0;
  l.num_sms = ctx->num_sms;
  for (int i = 0; i < 5; ++i) l.max_clusters[i] = ctx->max_clusters[i];
  l.ws_o_floats = ctx->ws_o_floats / kScratchSlots;
  l.n_counters = ctx->n_counters / kScratchSlots;
  l.force_nsplit = ctx->force_nsplit;
  l.force_cluster = ctx->force_cluster;
  return l;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device buffers are read and written 16 bytes at a time.
int check_aligned(l3p_attn_ctx* ctx, std::initializer_list<const void*> ptrs) {
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(ctx, L3P_E_INVAL, "device pointer %p is not 16-byte aligned", p);
  return L3P_OK;
}

int ensure_staging(l3p_attn_ctx* ctx, size_t floats) {
  if (floats <= ctx->st_floats) return L3P_OK;
  if (ctx->st_buf) cudaFree(ctx->st_buf);
  ctx->st_buf = nullptr;
  ctx->st_floats = 0;
  size_t want = std::max(floats, (size_t)1 << 16);
  if (cudaMalloc(&ctx->st_buf, want * sizeof(float)) != cudaSuccess)
    return fail(ctx, L3P_E_NOMEM, "staging allocation of %zu floats failed", want);
  ctx->st_floats = want;
  return L3P_OK;
}

int ensure_host_staging(l3p_attn_ctx* ctx, size_t floats) {
  if (floats <= ctx->hst_floats) return L3P_OK;
  if (ctx->hst) cudaFreeHost(ctx->hst);
  ctx->hst = ctx->hst_dev = nullptr;
  ctx->hst_floats = 0;
  const size_t want = std::max(floats, (size_t)1 << 14);
  if (cudaHostAlloc(&ctx->hst, want * sizeof(float), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(&ctx->hst_dev, ctx->hst, 0) != cudaSuccess) {
    cudaGetLastError();
    if (ctx->hst) cudaFreeHost(ctx->hst);
    ctx->hst = ctx->hst_dev = nullptr;
    return fail(ctx, L3P_E_NOMEM, "pinned staging allocation of %zu floats failed", want);
  }
  ctx->hst_floats = want;
  return L3P_OK;
}

int check_layer(l3p_attn_ctx* ctx, int layer) {
  if (layer < 0 || layer >= ctx->cfg.n_layers)
    return fail(ctx, L3P_E_RANGE, "layer %d outside [0, %d)", layer, ctx->cfg.n_layers);
  return L3P_OK;
}

int read_err(l3p_attn_ctx* ctx) {
  const int e = *reinterpret_cast<volatile int*>(ctx->err_host);
  if (e) {
    *reinterpret_cast<volatile int*>(ctx->err_host) = 0;
    if (e & kErrTimeout) return fail(ctx, L3P_E_TIMEOUT, "a bounded device wait gave up");
    return fail(ctx, L3P_E_CUDA, "device error flag %d", e);
  }
  return L3P_OK;
}

// Stamp buffer of the next traced launch (builds with L3P_DECODE_TRACE; null
// otherwise, or when the grid has more CTAs than a slot holds).  Slot
// metadata: trace ordinal, grid x, y, z, layer, position (-1: a wo launch).
unsigned long long* trace_slot(l3p_attn_ctx* ctx, int gx, int gy, int gz, int layer, int pos) {
#ifdef L3P_DECODE_TRACE
  if (ctx->trace_dev && (long long)gx * gy * gz <= kTraceCtas) {
    const int ts = (int)(ctx->trace_count % kTraceSlots);
    long long* m = ctx->trace_meta[ts];
    m[0] = (long long)ctx->trace_count++, m[1] = gx, m[2] = gy, m[3] = gz, m[4] = layer, m[5] = pos;
    return ctx->trace_dev + (size_t)ts * kTraceCtas * 8;
  }
#endif
  (void)ctx, (void)gx, (void)gy, (void)gz, (void)layer, (void)pos;
  return nullptr;
}

void decode_common_args(const l3p_attn_ctx* ctx, DecodeArgs* a) {
  a->kc = ctx->kc;
  a->vc = ctx->vc;
  a->kc_w = ctx->kc;
  a->k8 = ctx->k8;
  a->v8 = ctx->v8;
  a->ksc = ctx->ksc;
  a->vsc = ctx->vsc;
  a->new_zstride = (long long)ctx->cfg.n_kv_heads * ctx->hd;
  a->layer_stride = ctx->layer_elems;
  a->head_stride = ctx->head_elems;
  a->q_zstride = (long long)ctx->cfg.n_heads * ctx->hd;
  a->ml_zstride = 2ll * ctx->cfg.n_heads;
  a->err = ctx->err_dev;
  a->scale = ctx->scale;
  a->seq_begin = ctx->cfg.seq_begin;
  a->cap = ctx->seq_count;
  a->kv_head_begin = ctx->cfg.kv_head_begin;
  a->G = ctx->G;
  a->n_hg = ctx->n_hg;
  a->is_gemma3 = ctx->cfg.is_gemma3;
  a->swa_window = ctx->cfg.swa_window;
  a->swa_pattern = ctx->cfg.swa_pattern;
  a->layer_step = 0;
  a->pos_step = 0;
  a->wait_pos = INT_MAX;
  a->merge_k = 1;
  a->cluster = 1;
}

// Designated mergers of a one-wave launch without clusters: at least enough
// that each thread merges one float4 of a slice, and more for many parts
// (each merger's threads then split the parts into groups: one L2 round trip
// per 16 parts and group).
int designated_mergers(const l3p_attn_ctx* ctx, int nsplit, int threads) {
  const int by_size = std::max(1, (ctx->GT * ctx->hd / 4 + threads - 1) / threads);
  const int by_parts = nsplit >= 48 ? 4 : nsplit >= 24 ? 2 : 1;
  return std::min(nsplit, std::max(by_size, by_parts));
}

int server_geom(l3p_attn_ctx* ctx, int pos, ServerGeom* g) {
  const KernelInfo ki = kernel_for(ctx->hd, ctx->GT, ctx->q8);
  if (!ki.srv) return fail(ctx, L3P_E_UNSUPPORTED, "the host-call server serves fp32 caches only");
  const long long lo = ctx->cfg.seq_begin;
  const long long hi = std::min<long long>((long long)pos + 1, lo + ctx->seq_count);
  const long long P = std::max<long long>(hi - lo, 0);
  const long long units = (long long)ctx->kvh_count * ctx->n_hg;
  const long long slots = (long long)ctx->num_sms * ki.ctas_per_sm;
  if (units > slots) return fail(ctx, L3P_E_UNSUPPORTED, "%lld decode units do not fit on the GPU at once", units);
  // the plan of a decode launch, without clusters, and no more parts than
  // leave the whole grid resident (the server's CTAs wait for one another)
  const Plan p = cached_plan(ctx, P, units, ki);
  int ns = std::max(1, std::min<int>(p.nsplit, (int)(slots / units)));
  g->nsplit = ns;
  g->merge_k = ns > 1 ? designated_mergers(ctx, ns, ki.threads) : 1;
  g->units = (int)units;
  g->threads = ki.threads;
  g->smem = ki.smem;
  g->fn = reinterpret_cast<const void*>(ki.srv);
  return L3P_OK;
}

// Decode core shared by the single-layer, multi-layer, prefill and partial
// entry points.  z-slices are layers (layer_step=1) or tokens (pos_step=1).
int launch_decode(l3p_attn_ctx* ctx, int layer0, int layer_step, int pos0, int pos_step, int nz,
                  const float* q, float* out, float* part_o, float* part_ml, cudaStream_t s,
                  const float* k_new, const float* v_new, bool allow_overlap) {
  const KernelInfo ki = kernel_for(ctx->hd, ctx->GT, ctx->q8);
  if (!ki.fn) return fail(ctx, L3P_E_UNSUPPORTED, "no decode kernel for head_dim %d", ctx->hd);
  // longest attended range over the slices (upper bound; the kernel clips per slice)
  const int pos_max = pos0 + (nz - 1) * pos_step;
  const long long lo = ctx->cfg.seq_begin;
  const long long hi = std::min<long long>(pos_max + 1, (long long)ctx->cfg.seq_begin + ctx->seq_count);
  const long long P = std::max<long long>(hi - lo, 0);
  const long long units = (long long)nz * ctx->kvh_count * ctx->n_hg;
  const Plan plan = cached_plan(ctx, P, units, ki);
  // Rows a fused append of an earlier launch may still be storing.  Under
  // programmatic dependent launch every launch of a chain but the newest is
  // resident at once (each has triggered, and none of its CTAs exits before
  // the launch before it completes), and a decode CTA holds a whole SM's
  // shared memory, so a store more than num_sms * ctas_per_sm decode launches
  // back has landed; the window doubles that.  The kernel copies the rows from
  // wait_pos on only after griddepcontrol.wait.
  const unsigned long long window = 2ull * ctx->num_sms * ki.ctas_per_sm + 2;
  int wait_pos = INT_MAX;
  for (int z = 0; z < (layer_step ? nz : 1); ++z) {
    auto& d = ctx->recent_stores[layer0 + z * layer_step];
    while (!d.empty() && ctx->launch_seq - d.front().first > window) d.pop_front();
    for (const auto& e : d) wait_pos = std::min(wait_pos, e.second);
  }
  const unsigned long long seq = ctx->launch_seq++;
  const int slot = (int)(seq % kScratchSlots);
  if (k_new)  // this launch stores the row of pos0 + z*pos_step of each slice's layer
    for (int z = 0; z < nz; ++z) ctx->recent_stores[layer0 + z * layer_step].emplace_back(seq, pos0 + z * pos_step);

  DecodeArgs a{};
  decode_common_args(ctx, &a);
  a.k_new = k_new;
  a.v_new = v_new;
  a.q = q;
  a.out = out;
  a.part_o = part_o;
  a.part_ml = part_ml;
  a.ws_o = ctx->ws_o + slot * (ctx->ws_o_floats / kScratchSlots);
  a.ws_ml = ctx->ws_ml + slot * (ctx->ws_ml_floats / kScratchSlots);
  a.counters = ctx->counters + slot * (ctx->n_counters / kScratchSlots);
  a.layer0 = layer0;
  a.layer_step = layer_step;
  a.pos0 = pos0;
  a.pos_step = pos_step;
  a.nsplit = plan.nsplit;
  a.cluster = plan.cluster;
  a.partial = part_o != nullptr;
  // several mergers for the global stage when every CTA of the launch is
  // resident at once (a merger waits for its unit's last part)
  a.wait_pos = wait_pos;
  const long long grid_ctas = (long long)plan.nsplit * units;
  const bool one_wave = grid_ctas <= (long long)ctx->num_sms * ki.ctas_per_sm;
  a.trace = trace_slot(ctx, plan.nsplit, ctx->kvh_count * ctx->n_hg, nz, layer0, pos0);
  if (plan.cluster == 1 && plan.nsplit > 1 && nz <= 65535 && one_wave && !ctx->ticket_merge &&
      units * plan.nsplit <= ctx->n_counters / kScratchSlots) {
    // designated mergers (decode_finish): the flags live in the slot's tickets
    // array; at least enough mergers that each thread merges one float4 of a
    // slice, and more for many parts (each merger's threads then split the
    // parts into groups: one L2 round trip per 16 parts and group)
    a.flags = a.counters;
    a.merge_k = designated_mergers(ctx, plan.nsplit, ki.threads);
  } else if (plan.cluster == 1 && plan.nsplit >= kMergersFrom && nz <= 65535 && one_wave) {
    a.merge_k = kMergers;
  }

  for (int z0 = 0; z0 < nz; z0 += 65535) {
    const int zc = std::min(nz - z0, 65535);
    DecodeArgs b = a;
    b.layer0 = a.layer0 + z0 * layer_step;
    b.pos0 = a.pos0 + z0 * pos_step;
    b.q = a.q + (long long)z0 * a.q_zstride;
    if (b.out) b.out = a.out + (long long)z0 * a.q_zstride;
    if (b.part_o) b.part_o = a.part_o + (long long)z0 * a.q_zstride;
    if (b.part_ml) b.part_ml = a.part_ml + (long long)z0 * a.ml_zstride;
    if (b.k_new) b.k_new = a.k_new + (long long)z0 * a.new_zstride;
    if (b.v_new) b.v_new = a.v_new + (long long)z0 * a.new_zstride;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(plan.nsplit, ctx->kvh_count * ctx->n_hg, zc);
    lc.blockDim = dim3(ki.threads, 1, 1);
    lc.dynamicSmemBytes = ki.smem;
    lc.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned n_attr = 0;
    if (plan.cluster > 1) {
      attr[n_attr].id = cudaLaunchAttributeClusterDimension;
      attr[n_attr].val.clusterDim.x = plan.cluster;
      attr[n_attr].val.clusterDim.y = 1;
      attr[n_attr].val.clusterDim.z = 1;
      ++n_attr;
    }
    if (allow_overlap && ctx->overlap) {
      attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
      ++n_attr;
    }
    lc.attrs = attr;
    lc.numAttrs = n_attr;
    L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, ki.fn, b));
    ++ctx->launches;
  }
  return L3P_OK;
}

// Q8_0 rows: one warp per (token, KV head) row.  k8/ksc point at the first row
// of the destination head block; grid.y heads of head_elems values each.
int launch_append_q8(l3p_attn_ctx* ctx, int8_t* k8, int8_t* v8, uint16_t* ksc, uint16_t* vsc, dim3 grid,
                     const float* k, const float* v, long long src_stride, int kv_head_begin, int row0,
                     cudaStream_t s) {
  cudaLaunchConfig_t lc{};
  lc.gridDim = grid;
  lc.blockDim = dim3(32, 1, 1);
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  pdl_attr(ctx, lc, attr);
  const long long hs = ctx->head_elems;
  switch (ctx->hd) {
    case 64:
      L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, kv_append_q8_kernel<64>, k8, v8, ksc, vsc, hs, k, v, src_stride,
                                       kv_head_begin, row0));
      break;
    case 128:
      L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, kv_append_q8_kernel<128>, k8, v8, ksc, vsc, hs, k, v, src_stride,
                                       kv_head_begin, row0));
      break;
    default:
      L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, kv_append_q8_kernel<256>, k8, v8, ksc, vsc, hs, k, v, src_stride,
                                       kv_head_begin, row0));
      break;
  }
  ++ctx->launches;
  return L3P_OK;
}

int launch_append(l3p_attn_ctx* ctx, int layer, int pos0, int n_tok, const float* k, const float* v,
                  cudaStream_t s) {
  // clip the tokens to the owned position range
  const int own_lo = ctx->cfg.seq_begin, own_hi = ctx->cfg.seq_begin + ctx->seq_count;
  const int t_lo = std::max(pos0, own_lo), t_hi = std::min(pos0 + n_tok, own_hi);
  if (t_hi <= t_lo) return L3P_OK;
  const long long src_stride = (long long)ctx->cfg.n_kv_heads * ctx->hd;
  const long long off = (long long)layer * ctx->layer_elems;
  const float* ks = k + (long long)(t_lo - pos0) * src_stride;
  const float* vs = v + (long long)(t_lo - pos0) * src_stride;
  for (int t0 = t_lo; t0 < t_hi; t0 += 65535) {
    const int nt = std::min(t_hi - t0, 65535);
    dim3 grid(nt, ctx->kvh_count);
    if (ctx->q8) {
      // quantise the rows into the Q8_0 cache (quantize_to_q8_0_cache, c:1535-1570)
      if (int rc = launch_append_q8(ctx, ctx->k8 + off, ctx->v8 + off, ctx->ksc + off / 32, ctx->vsc + off / 32, grid,
                                    ks + (long long)(t0 - t_lo) * src_stride, vs + (long long)(t0 - t_lo) * src_stride,
                                    src_stride, ctx->cfg.kv_head_begin, t0 - own_lo, s))
        return rc;
      continue;
    }
    cudaLaunchConfig_t lc{};
    lc.gridDim = grid;
    lc.blockDim = dim3(ctx->hd / 4, 1, 1);
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    pdl_attr(ctx, lc, attr);
    L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, kv_append_kernel, ctx->kc + off, ctx->vc + off, ctx->head_elems, ctx->hd,
                                     ks + (long long)(t0 - t_lo) * src_stride, vs + (long long)(t0 - t_lo) * src_stride,
                                     src_stride, ctx->cfg.kv_head_begin, t0 - own_lo));
    ++ctx->launches;
  }
  return L3P_OK;
}

// Tensor-core prefill: split the cached K/V rows [0, start_pos+n_tok) into
// tf32 hi/lo chunk images, then run the tcgen05 flash-attention kernel.
template <int HD>
int launch_prefill_tc_hd(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q, float* out,
                         cudaStream_t s) {
  const int n_keys = start_pos + n_tok;
  const int n_ktiles = (n_keys + kPfBN - 1) / kPfBN;
  const size_t need = (size_t)ctx->kvh_count * n_ktiles * PfGeom<HD>::kTileFloats;
  if (need > ctx->pf_img_floats) {
    if (ctx->pf_img) {
      L3P_CUDA(ctx, cudaStreamSynchronize(s));
      cudaFree(ctx->pf_img);
    }
    ctx->pf_img = nullptr;
    ctx->pf_img_floats = 0;
    if (cudaMalloc(&ctx->pf_img, need * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      return fail(ctx, L3P_E_NOMEM, "prefill image allocation of %zu floats failed", need);
    }
    ctx->pf_img_floats = need;
  }
  const long long off = (long long)layer * ctx->layer_elems;
  const int cg = HD == 128 ? ctx->prefill_cg : 1;
  (cg == 2 ? prefill_prep_kernel<(HD == 128 ? 2 : 1), HD> : prefill_prep_kernel<1, HD>)<<<dim3(n_ktiles, ctx->kvh_count), 256, 0, s>>>(
      ctx->q8 ? nullptr : ctx->kc + off, ctx->q8 ? nullptr : ctx->vc + off, ctx->head_elems, n_keys, n_ktiles,
      ctx->pf_img, ctx->q8 ? ctx->k8 + off : nullptr, ctx->q8 ? ctx->v8 + off : nullptr,
      ctx->q8 ? ctx->ksc + off / 32 : nullptr, ctx->q8 ? ctx->vsc + off / 32 : nullptr);
  ++ctx->launches;
  L3P_CUDA(ctx, cudaGetLastError());
  PrefillArgs a{};
  a.q = q;
  a.out = out;
  a.img = ctx->pf_img;
  a.n_heads = ctx->cfg.n_heads;
  a.G = ctx->G;
  a.kv_head_begin = ctx->cfg.kv_head_begin;
  a.n_qh = ctx->kvh_count * ctx->G;
  a.q_pos0 = start_pos;
  a.n_tok = n_tok;
  a.n_qtiles = (n_tok + kPfBM - 1) / kPfBM;
  a.n_ktiles = n_ktiles;
  a.scale = ctx->scale;
  a.layer = layer;
  a.is_gemma3 = ctx->cfg.is_gemma3;
  a.swa_window = ctx->cfg.swa_window;
  a.swa_pattern = ctx->cfg.swa_pattern;
  a.q8 = ctx->q8 ? 1 : 0;
  a.err = ctx->err_dev;
  if constexpr (HD == 128) {
    if (cg == 2) {
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(a.n_qtiles * a.n_qh, 1, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.dynamicSmemBytes = PfCfg<2, 128>::kSmemBytes;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    L3P_CUDA(ctx, cudaLaunchKernelEx(&lc, prefill_tc_kernel<2, 128>, a));
    ++ctx->launches;
    return L3P_OK;
    }
  }
  prefill_tc_kernel<1, HD><<<a.n_qtiles * a.n_qh, 256, PfCfg<1, HD>::kSmemBytes, s>>>(a);
  ++ctx->launches;
  L3P_CUDA(ctx, cudaGetLastError());
  return L3P_OK;
}

int launch_prefill_tc(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q, float* out,
                      cudaStream_t s) {
  if (ctx->hd == 64) return launch_prefill_tc_hd<64>(ctx, layer, start_pos, n_tok, q, out, s);
  return launch_prefill_tc_hd<128>(ctx, layer, start_pos, n_tok, q, out, s);
}

int check_pos_full(l3p_attn_ctx* ctx, int pos) {
  if (pos < 0 || pos >= ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "pos %d outside [0, %d)", pos, ctx->cfg.seq_len);
  if (ctx->cfg.seq_begin != 0 || ctx->seq_count <= pos)
    return fail(ctx, L3P_E_INVAL,
                "full decode needs the whole sequence [0, %d] on this context (owned [%d, %d)); "
                "use l3p_attn_decode_partial_dev",
                pos, ctx->cfg.seq_begin, ctx->cfg.seq_begin + ctx->seq_count);
  return L3P_OK;
}

}  // namespace l3p_api

// ==========================================================================
// Lifecycle

L3P_API int l3p_attn_create(const l3p_attn_config* cfg, l3p_attn_ctx** out) {
  if (!out) return L3P_E_INVAL;
  *out = nullptr;
  if (!cfg) return L3P_E_INVAL;
  const l3p_attn_config& c = *cfg;
  if (c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.seq_len <= 0 ||
      c.n_heads % c.n_kv_heads != 0 || (c.kv_format != L3P_KV_F32 && c.kv_format != L3P_KV_Q8_0))
    return L3P_E_INVAL;
  if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256) return L3P_E_UNSUPPORTED;
  const int kvh_count = c.kv_head_count > 0 ? c.kv_head_count : c.n_kv_heads - c.kv_head_begin;
  const int seq_count = c.seq_count > 0 ? c.seq_count : c.seq_len - c.seq_begin;
  if (c.kv_head_begin < 0 || kvh_count <= 0 || c.kv_head_begin + kvh_count > c.n_kv_heads ||
      c.seq_begin < 0 || seq_count <= 0 || c.seq_begin + seq_count > c.seq_len)
    return L3P_E_INVAL;

  l3p_attn_ctx* ctx = new (std::nothrow) l3p_attn_ctx();
  if (!ctx) return L3P_E_NOMEM;
  ctx->cfg = c;
  ctx->cfg.kv_head_count = kvh_count;
  ctx->cfg.seq_count = seq_count;
  ctx->hd = c.head_dim;
  ctx->G = c.n_heads / c.n_kv_heads;
  ctx->GT = (ctx->G % 8 == 0) ? 8 : (ctx->G % 4 == 0) ? 4 : (ctx->G % 2 == 0) ? 2 : 1;
  ctx->n_hg = ctx->G / ctx->GT;
  ctx->recent_stores.resize(c.n_layers);
  ctx->kvh_count = kvh_count;
  ctx->seq_count = seq_count;
  // L3P_DECODE_MERGE=ticket keeps the last-arrival (ticket) merge for one-wave
  // launches too (tests compare both)
  if (const char* m = getenv("L3P_DECODE_MERGE"))
    if (strcmp(m, "ticket") == 0) ctx->ticket_merge = true;
  if (const char* plan = getenv("L3P_DECODE_PLAN")) {
    if (sscanf(plan, "%d:%d", &ctx->force_nsplit, &ctx->force_cluster) < 1) ctx->force_nsplit = 0;
  }
  // attn_scale = 1.0f / sqrtf((float)head_size), c:434
  ctx->scale = c.scale != 0.f ? c.scale : 1.0f / sqrtf((float)c.head_dim);
  ctx->head_elems = (long long)seq_count * c.head_dim;
  ctx->layer_elems = ctx->head_elems * kvh_count;

  DeviceScope dev(c.device);
  auto bail = [&](int code, const char* what) {
    fail(ctx, code, "%s", what);
    l3p_attn_destroy(ctx);
    return code;
  };
  if (cudaSetDevice(c.device) != cudaSuccess) return bail(L3P_E_CUDA, "cudaSetDevice failed");
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, c.device);
  ctx->q8 = c.kv_format == L3P_KV_Q8_0;
  if (ctx->q8) {
    const size_t vals = (size_t)ctx->layer_elems * c.n_layers, scales = vals / 32;
    if (cudaMalloc(&ctx->k8, vals) != cudaSuccess || cudaMalloc(&ctx->v8, vals) != cudaSuccess ||
        cudaMalloc(&ctx->ksc, scales * 2) != cudaSuccess || cudaMalloc(&ctx->vsc, scales * 2) != cudaSuccess) {
      cudaGetLastError();
      return bail(L3P_E_NOMEM, "KV cache allocation failed");
    }
    // zero the cache: positions never written read as 0 (scale 0) rather than garbage
    if (cudaMemset(ctx->k8, 0, vals) != cudaSuccess || cudaMemset(ctx->v8, 0, vals) != cudaSuccess ||
        cudaMemset(ctx->ksc, 0, scales * 2) != cudaSuccess || cudaMemset(ctx->vsc, 0, scales * 2) != cudaSuccess)
      return bail(L3P_E_CUDA, "cache memset failed");
  } else {
    const size_t cache_bytes = (size_t)ctx->layer_elems * c.n_layers * sizeof(float);
    if (cudaMalloc(&ctx->kc, cache_bytes) != cudaSuccess || cudaMalloc(&ctx->vc, cache_bytes) != cudaSuccess) {
      cudaGetLastError();
      return bail(L3P_E_NOMEM, "KV cache allocation failed");
    }
    // zero the cache: positions never written read as 0 rather than garbage
    if (cudaMemset(ctx->kc, 0, cache_bytes) != cudaSuccess || cudaMemset(ctx->vc, 0, cache_bytes) != cudaSuccess)
      return bail(L3P_E_CUDA, "cache memset failed");
  }
  ctx->ws_o_floats = kWsOFloats;
  ctx->ws_ml_floats = kWsOFloats / 64 * 2;  // GT*HD >= 64, two floats per (split, q head)
  ctx->n_counters = kCounters;
  if (cudaMalloc(&ctx->ws_o, ctx->ws_o_floats * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&ctx->ws_ml, ctx->ws_ml_floats * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&ctx->counters, ctx->n_counters * sizeof(unsigned)) != cudaSuccess) {
    cudaGetLastError();
    return bail(L3P_E_NOMEM, "scratch allocation failed");
  }
  if (cudaMemset(ctx->counters, 0, ctx->n_counters * sizeof(unsigned)) != cudaSuccess)
    return bail(L3P_E_CUDA, "counter memset failed");
  if (cudaHostAlloc(&ctx->err_host, sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(&ctx->err_dev, ctx->err_host, 0) != cudaSuccess) {
    cudaGetLastError();
    return bail(L3P_E_CUDA, "error word allocation failed");
  }
  *ctx->err_host = 0;
#ifdef L3P_DECODE_TRACE
  {
    const size_t tb = (size_t)kTraceSlots * kTraceCtas * 8 * sizeof(unsigned long long);
    if (cudaHostAlloc(&ctx->trace_host, tb, cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(&ctx->trace_dev, ctx->trace_host, 0) != cudaSuccess)
      return bail(L3P_E_NOMEM, "trace buffer allocation failed");
    memset(ctx->trace_host, 0, tb);
  }
#endif
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(L3P_E_CUDA, "stream creation failed");
  ctx->own_stream = true;
  const KernelInfo ki = kernel_for(ctx->hd, ctx->GT, ctx->q8);
  if (!ki.fn) return bail(L3P_E_UNSUPPORTED, "no decode kernel for this geometry");
  if (cudaFuncSetAttribute(ki.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ki.smem) != cudaSuccess)
    return bail(L3P_E_CUDA, "cudaFuncSetAttribute failed");
  // head_dim 64 and 128 prefill runs on the tensor cores unless
  // L3P_PREFILL_PATH=ffma (head_dim 256: the decode kernel in token mode)
  ctx->prefill_tc = c.head_dim == 64 || c.head_dim == 128;
  if (const char* path = getenv("L3P_PREFILL_PATH"))
    if (strcmp(path, "ffma") == 0) ctx->prefill_tc = false;
  // single CTAs by default (measured faster: the pair form pays a second
  // commit per barrier and a relay per chunk); L3P_PREFILL_CG=2 selects CTA
  // pairs (cta_group::2), which take two q heads of one KV head and so need an
  // even GQA group
  ctx->prefill_cg = 1;
  if (const char* cg = getenv("L3P_PREFILL_CG"))
    if (strcmp(cg, "2") == 0 && ctx->G % 2 == 0) ctx->prefill_cg = 2;
  if (ctx->prefill_tc &&
      (cudaFuncSetAttribute(prefill_tc_kernel<1, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            PfCfg<1, 128>::kSmemBytes) != cudaSuccess ||
       cudaFuncSetAttribute(prefill_tc_kernel<2, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            PfCfg<2, 128>::kSmemBytes) != cudaSuccess ||
       cudaFuncSetAttribute(prefill_tc_kernel<1, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            PfCfg<1, 64>::kSmemBytes) != cudaSuccess))
    return bail(L3P_E_CUDA, "cudaFuncSetAttribute (prefill) failed");
  // clusters of up to 16 CTAs (16 is a non-portable size); record how many of
  // each size fit on this GPU at once (0 = that size is not available)
  if (cudaFuncSetAttribute(ki.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    cudaGetLastError();
  for (int ci = 1; ci < 5; ++ci) {
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(1 << ci, 1, 1);
    lc.blockDim = dim3(ki.threads, 1, 1);
    lc.dynamicSmemBytes = ki.smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1 << ci;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, ki.fn, &lc) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    ctx->max_clusters[ci] = n;
  }
  *out = ctx;
  return L3P_OK;
}

L3P_API void l3p_attn_destroy(l3p_attn_ctx* ctx) {
  if (!ctx) return;
  CtxScope dev(ctx);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->kc);
  cudaFree(ctx->vc);
  cudaFree(ctx->k8);
  cudaFree(ctx->v8);
  cudaFree(ctx->ksc);
  cudaFree(ctx->vsc);
  cudaFree(ctx->ws_o);
  cudaFree(ctx->ws_ml);
  cudaFree(ctx->counters);
  cudaFree(ctx->st_buf);
  cudaFree(ctx->pf_img);
  if (ctx->rope_tab_swa != ctx->rope_tab) cudaFree(ctx->rope_tab_swa);
  cudaFree(ctx->rope_tab);
  cudaFree(ctx->qk_norm);
  cudaFree(ctx->rope_buf);
  for (auto& w : ctx->wo) {
    cudaFree(w.w);
    cudaFree(w.wsc);
  }
  cudaFree(ctx->wo_x);
  for (int p = 0; p < ctx->xg_parts; ++p)
    if (p != ctx->xg_part && ctx->xg_peer[p]) cudaIpcCloseMemHandle(ctx->xg_peer[p]);
  cudaFree(ctx->xg_region);
  for (int p = 0; p < ctx->tp_members; ++p)
    if (p != ctx->tp_member && ctx->tp_peer[p]) cudaIpcCloseMemHandle(ctx->tp_peer[p]);
  cudaFree(ctx->tp_region);
  if (ctx->hst) cudaFreeHost(ctx->hst);
  if (ctx->srv_outbox) cudaFreeHost(ctx->srv_outbox);
  if (ctx->srv_stage) cudaFreeHost(ctx->srv_stage);
  if (ctx->srv_copy) cudaStreamDestroy(ctx->srv_copy);
  cudaFree(ctx->srv_dev);
  if (ctx->err_host) cudaFreeHost(ctx->err_host);
#ifdef L3P_DECODE_TRACE
  if (ctx->trace_host) {
    cudaDeviceSynchronize();
    if (const char* path = getenv("L3P_TRACE_FILE")) {
      // [n slots][6 meta][kTraceCtas * 8 stamps] as little-endian int64 / uint64
      if (FILE* f = fopen(path, "wb")) {
        const long long n = (long long)std::min<unsigned long long>(ctx->trace_count, kTraceSlots);
        const long long ctas = kTraceCtas;
        fwrite(&n, 8, 1, f);
        fwrite(&ctas, 8, 1, f);
        for (long long i = 0; i < n; ++i) {
          fwrite(ctx->trace_meta[i], 8, 6, f);
          fwrite(ctx->trace_host + (size_t)i * kTraceCtas * 8, 8, (size_t)kTraceCtas * 8, f);
        }
        fclose(f);
      }
    }
    cudaFreeHost(ctx->trace_host);
  }
#endif
  if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

L3P_API const char* l3p_attn_last_error(const l3p_attn_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : "null context";
}

L3P_API int l3p_attn_check(l3p_attn_ctx* ctx) {
  if (!ctx) return L3P_E_INVAL;
  CtxScope dev(ctx);
  L3P_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  L3P_CUDA(ctx, cudaDeviceSynchronize());
  return read_err(ctx);
}

L3P_API int l3p_attn_set_stream(l3p_attn_ctx* ctx, void* stream) {
  if (!ctx) return L3P_E_INVAL;
  CtxScope dev(ctx);
  if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
  ctx->own_stream = false;
  ctx->stream = static_cast<cudaStream_t>(stream);
  if (!stream) {
    L3P_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
    ctx->own_stream = true;
  }
  return L3P_OK;
}

L3P_API long long l3p_attn_launch_count(const l3p_attn_ctx* ctx) { return ctx ? ctx->launches : -1; }

L3P_API int l3p_attn_device_arch(int device, int* binary, int* ptx) {
  if (!binary || !ptx) return L3P_E_INVAL;
  DeviceScope dev(device);
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, decode_f32_kernel<128, 4>) != cudaSuccess) {
    cudaGetLastError();
    return L3P_E_CUDA;
  }
  *binary = fa.binaryVersion;
  *ptx = fa.ptxVersion;
  return L3P_OK;
}

L3P_API int l3p_attn_set_overlap(l3p_attn_ctx* ctx, int enable) {
  if (!ctx) return L3P_E_INVAL;
  ctx->overlap = enable != 0;
  return L3P_OK;
}

L3P_API int l3p_attn_decode_plan(l3p_attn_ctx* ctx, int pos, int n_slices, int* nsplit, int* cluster) {
  if (!ctx || n_slices <= 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  const KernelInfo ki = kernel_for(ctx->hd, ctx->GT, ctx->q8);
  if (!ki.fn) return fail(ctx, L3P_E_UNSUPPORTED, "no decode kernel for head_dim %d", ctx->hd);
  const long long hi = std::min<long long>((long long)pos + 1, (long long)ctx->cfg.seq_begin + ctx->seq_count);
  const long long P = std::max<long long>(hi - ctx->cfg.seq_begin, 0);
  const Plan plan = cached_plan(ctx, P, (long long)n_slices * ctx->kvh_count * ctx->n_hg, ki);
  if (nsplit) *nsplit = plan.nsplit;
  if (cluster) *cluster = plan.cluster;
  return L3P_OK;
}

// ==========================================================================
// Device-pointer entry points

L3P_API int l3p_attn_kv_append_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* k, const float* v,
                                   void* stream) {
  if (!ctx || !k || !v) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos < 0 || pos >= ctx->cfg.seq_len) return fail(ctx, L3P_E_RANGE, "pos %d outside [0, %d)", pos, ctx->cfg.seq_len);
  if (int rc = check_aligned(ctx, {k, v})) return rc;
  CtxScope dev(ctx);
  return launch_append(ctx, layer, pos, 1, k, v, pick_stream(ctx, stream));
}

L3P_API int l3p_attn_decode_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* out, void* stream) {
  if (!ctx || !q || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (int rc = check_aligned(ctx, {q, out})) return rc;
  CtxScope dev(ctx);
  return launch_decode(ctx, layer, 0, pos, 0, 1, q, out, nullptr, nullptr, pick_stream(ctx, stream), nullptr,
                       nullptr, true);
}

L3P_API int l3p_attn_step_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k, const float* v,
                              float* out, void* stream) {
  if (!ctx || !q || !k || !v || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (int rc = check_aligned(ctx, {q, k, v, out})) return rc;
  CtxScope dev(ctx);
  // one launch: the decode stores the new row (quantised first for a Q8_0
  // cache, c:3299-3312) and attends to it from its producer's copy
  return launch_decode(ctx, layer, 0, pos, 0, 1, q, out, nullptr, nullptr, pick_stream(ctx, stream), k, v, true);
}

L3P_API int l3p_attn_decode_layers_dev(l3p_attn_ctx* ctx, int layer0, int n_layers, int pos, const float* q,
                                       float* out, void* stream) {
  if (!ctx || !q || !out || n_layers <= 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer0)) return rc;
  if (int rc = check_layer(ctx, layer0 + n_layers - 1)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (int rc = check_aligned(ctx, {q, out})) return rc;
  CtxScope dev(ctx);
  return launch_decode(ctx, layer0, 1, pos, 0, n_layers, q, out, nullptr, nullptr, pick_stream(ctx, stream),
                       nullptr, nullptr, true);
}

L3P_API int l3p_attn_decode_partial_dev(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* part_o,
                                        float* part_ml, void* stream) {
  if (!ctx || !q || !part_o || !part_ml) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos < 0 || pos >= ctx->cfg.seq_len) return fail(ctx, L3P_E_RANGE, "pos %d outside [0, %d)", pos, ctx->cfg.seq_len);
  if (int rc = check_aligned(ctx, {q, part_o})) return rc;
  CtxScope dev(ctx);
  return launch_decode(ctx, layer, 0, pos, 0, 1, q, nullptr, part_o, part_ml, pick_stream(ctx, stream), nullptr,
                       nullptr, true);
}

L3P_API int l3p_attn_lse_merge_dev(l3p_attn_ctx* ctx, int n_parts, int rows_per_part, int row_begin, int n_rows,
                                   const float* parts_o, const float* parts_ml, float* out, void* stream) {
  if (!ctx || !parts_o || !parts_ml || !out || n_parts <= 0 || n_rows < 0 || row_begin < 0 ||
      row_begin + n_rows > rows_per_part)
    return ctx ? fail(ctx, L3P_E_INVAL, "bad merge arguments") : L3P_E_INVAL;
  if (n_rows == 0) return L3P_OK;
  CtxScope dev(ctx);
  lse_merge_kernel<<<n_rows, 128, 0, pick_stream(ctx, stream)>>>(n_parts, rows_per_part, row_begin, ctx->hd,
                                                                 parts_o, parts_ml, out);
  ++ctx->launches;
  L3P_CUDA(ctx, cudaGetLastError());
  return L3P_OK;
}

L3P_API int l3p_attn_prefill_dev(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                                 const float* k, const float* v, float* out, void* stream) {
  if (!ctx || !q || !k || !v || !out || n_tok < 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (n_tok == 0) return L3P_OK;
  if (start_pos < 0 || start_pos + n_tok > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "tokens [%d, %d) outside [0, %d)", start_pos, start_pos + n_tok, ctx->cfg.seq_len);
  if (int rc = check_pos_full(ctx, start_pos + n_tok - 1)) return rc;
  if (int rc = check_aligned(ctx, {q, k, v, out})) return rc;
  CtxScope dev(ctx);
  cudaStream_t s = pick_stream(ctx, stream);
  if (int rc = launch_append(ctx, layer, start_pos, n_tok, k, v, s)) return rc;
  if (ctx->prefill_tc) return launch_prefill_tc(ctx, layer, start_pos, n_tok, q, out, s);
  return launch_decode(ctx, layer, 0, start_pos, 1, n_tok, q, out, nullptr, nullptr, s);
}

L3P_API int l3p_attn_kv_device_ptr(l3p_attn_ctx* ctx, int layer, float** k, float** v) {
  if (!ctx) return L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (ctx->q8) return fail(ctx, L3P_E_UNSUPPORTED, "the cache is Q8_0: no fp32 rows to point at");
  if (k) *k = ctx->kc + (long long)layer * ctx->layer_elems;
  if (v) *v = ctx->vc + (long long)layer * ctx->layer_elems;
  return L3P_OK;
}

// ==========================================================================
// Host-pointer entry points: stage through device memory, synchronise.

namespace l3p_api {

int finish_host_call(l3p_attn_ctx* ctx) {
  L3P_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  return read_err(ctx);
}

// rows of the q/out arrays this context owns: [row_lo, row_hi) in head_dim units
void owned_rows(const l3p_attn_ctx* ctx, int* row_lo, int* row_hi) {
  *row_lo = ctx->cfg.kv_head_begin * ctx->G;
  *row_hi = (ctx->cfg.kv_head_begin + ctx->kvh_count) * ctx->G;
}

}  // namespace l3p_api

L3P_API int l3p_attn_kv_append(l3p_attn_ctx* ctx, int layer, int pos, const float* k, const float* v) {
  if (!ctx || !k || !v) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos < 0 || pos >= ctx->cfg.seq_len) return fail(ctx, L3P_E_RANGE, "pos %d outside [0, %d)", pos, ctx->cfg.seq_len);
  CtxScope dev(ctx);
  const size_t kvd = (size_t)ctx->cfg.n_kv_heads * ctx->hd;
  if (int rc = ensure_staging(ctx, 2 * kvd)) return rc;
  if (int rc = ensure_host_staging(ctx, 2 * kvd)) return rc;
  memcpy(ctx->hst, k, kvd * 4);
  memcpy(ctx->hst + kvd, v, kvd * 4);
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf, ctx->hst, 2 * kvd * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = launch_append(ctx, layer, pos, 1, ctx->st_buf, ctx->st_buf + kvd, ctx->stream)) return rc;
  return finish_host_call(ctx);
}

L3P_API int l3p_attn_decode(l3p_attn_ctx* ctx, int layer, int pos, const float* q, float* out) {
  if (!ctx || !q || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (ctx->srv_on) return server_call(ctx, layer, pos, q, nullptr, nullptr, out);
  CtxScope dev(ctx);
  const size_t qd = (size_t)ctx->cfg.n_heads * ctx->hd;
  if (int rc = ensure_staging(ctx, qd)) return rc;
  if (int rc = ensure_host_staging(ctx, 2 * qd)) return rc;
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  const size_t row0 = (size_t)r0 * ctx->hd, nrow = (size_t)(r1 - r0) * ctx->hd;
  memcpy(ctx->hst + row0, q + row0, nrow * 4);
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf + row0, ctx->hst + row0, nrow * 4, cudaMemcpyHostToDevice, ctx->stream));
  // the kernel writes the output into mapped pinned memory: no device->host
  // copy follows.  The host then synchronises the stream: a completion word
  // stored by the kernel's last output writer (after a system-scope fence)
  // measured ~1.7 us per call slower on B200 than the stream synchronisation.
  if (int rc = launch_decode(ctx, layer, 0, pos, 0, 1, ctx->st_buf, ctx->hst_dev + qd, nullptr, nullptr, ctx->stream,
                             nullptr, nullptr))
    return rc;
  if (int rc = finish_host_call(ctx)) return rc;
  memcpy(out + row0, ctx->hst + qd + row0, nrow * 4);
  return L3P_OK;
}

L3P_API int l3p_attn_step(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k,
                          const float* v, float* out) {
  if (!ctx || !q || !k || !v || !out) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (int rc = check_pos_full(ctx, pos)) return rc;
  if (ctx->srv_on) return server_call(ctx, layer, pos, q, k, v, out);
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
  // one host->device copy of all inputs; the kernel writes the output into
  // mapped pinned memory, so no device->host copy follows.  (Carrying the 24 KB
  // of rows in the kernel's launch parameters instead measured 3-4 us per call
  // slower on B200: a launch with a large parameter block costs more than the
  // copy it replaces.)
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf, ctx->hst, in * 4, cudaMemcpyHostToDevice, ctx->stream));
  if (int rc = launch_decode(ctx, layer, 0, pos, 0, 1, ctx->st_buf, ctx->hst_dev + in, nullptr, nullptr, ctx->stream,
                             ctx->st_buf + qd, ctx->st_buf + qd + kvd))
    return rc;
  if (int rc = finish_host_call(ctx)) return rc;
  memcpy(out + row0, ctx->hst + in + row0, nrow * 4);
  return L3P_OK;
}

L3P_API int l3p_attn_prefill(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q,
                             const float* k, const float* v, float* out) {
  if (!ctx || !q || !k || !v || !out || n_tok < 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (n_tok == 0) return L3P_OK;
  if (start_pos < 0 || start_pos + n_tok > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "tokens [%d, %d) outside [0, %d)", start_pos, start_pos + n_tok, ctx->cfg.seq_len);
  if (int rc = check_pos_full(ctx, start_pos + n_tok - 1)) return rc;
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
  if (int rc = launch_append(ctx, layer, start_pos, n_tok, dk, dv, ctx->stream)) return rc;
  if (ctx->prefill_tc) {
    if (int rc = launch_prefill_tc(ctx, layer, start_pos, n_tok, dq, dout, ctx->stream)) return rc;
  } else if (int rc = launch_decode(ctx, layer, 0, start_pos, 1, n_tok, dq, dout, nullptr, nullptr, ctx->stream)) {
    return rc;
  }
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  // owned rows of every token: a strided copy
  L3P_CUDA(ctx, cudaMemcpy2DAsync(out + (size_t)r0 * ctx->hd, qd * 4, dout + (size_t)r0 * ctx->hd, qd * 4,
                                  (size_t)(r1 - r0) * ctx->hd * 4, n_tok, cudaMemcpyDeviceToHost, ctx->stream));
  return finish_host_call(ctx);
}

L3P_API int l3p_attn_load_kv(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, const float* k, const float* v) {
  if (!ctx || !k || !v || n_pos < 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos0 < 0 || pos0 + n_pos > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "positions [%d, %d) outside [0, %d)", pos0, pos0 + n_pos, ctx->cfg.seq_len);
  const int lo = std::max(pos0, ctx->cfg.seq_begin), hi = std::min(pos0 + n_pos, ctx->cfg.seq_begin + ctx->seq_count);
  if (hi <= lo) return L3P_OK;
  CtxScope dev(ctx);
  const size_t row = (size_t)ctx->hd;
  if (ctx->q8) {
    // stage each head's rows and quantise them on the device, as kv_append does
    const size_t n = (size_t)(hi - lo) * row;
    if (int rc = ensure_staging(ctx, 2 * n)) return rc;
    for (int h = 0; h < ctx->kvh_count; ++h) {
      const size_t src = ((size_t)(ctx->cfg.kv_head_begin + h) * n_pos + (lo - pos0)) * row;
      L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf, k + src, n * 4, cudaMemcpyHostToDevice, ctx->stream));
      L3P_CUDA(ctx, cudaMemcpyAsync(ctx->st_buf + n, v + src, n * 4, cudaMemcpyHostToDevice, ctx->stream));
      const long long off = (long long)layer * ctx->layer_elems + (long long)h * ctx->head_elems;
      for (int t0 = 0; t0 < hi - lo; t0 += 65535) {
        const int nt = std::min(hi - lo - t0, 65535);
        if (int rc = launch_append_q8(ctx, ctx->k8 + off, ctx->v8 + off, ctx->ksc + off / 32, ctx->vsc + off / 32,
                                      dim3(nt, 1), ctx->st_buf + (size_t)t0 * row, ctx->st_buf + n + (size_t)t0 * row,
                                      (long long)row, 0, lo - ctx->cfg.seq_begin + t0, ctx->stream))
          return rc;
      }
    }
    return finish_host_call(ctx);
  }
  for (int h = 0; h < ctx->kvh_count; ++h) {
    const size_t src = ((size_t)(ctx->cfg.kv_head_begin + h) * n_pos + (lo - pos0)) * row;
    const size_t dst = (size_t)layer * ctx->layer_elems + (size_t)h * ctx->head_elems +
                       (size_t)(lo - ctx->cfg.seq_begin) * row;
    L3P_CUDA(ctx, cudaMemcpyAsync(ctx->kc + dst, k + src, (size_t)(hi - lo) * row * 4, cudaMemcpyHostToDevice, ctx->stream));
    L3P_CUDA(ctx, cudaMemcpyAsync(ctx->vc + dst, v + src, (size_t)(hi - lo) * row * 4, cudaMemcpyHostToDevice, ctx->stream));
  }
  return finish_host_call(ctx);
}

L3P_API int l3p_attn_read_kv(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, float* k, float* v) {
  if (!ctx || !k || !v || n_pos < 0) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos0 < 0 || pos0 + n_pos > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "positions [%d, %d) outside [0, %d)", pos0, pos0 + n_pos, ctx->cfg.seq_len);
  const int lo = std::max(pos0, ctx->cfg.seq_begin), hi = std::min(pos0 + n_pos, ctx->cfg.seq_begin + ctx->seq_count);
  if (hi <= lo) return L3P_OK;
  CtxScope dev(ctx);
  const size_t row = (size_t)ctx->hd;
  if (ctx->q8) {
    // dequantised values d * int8 (exact in fp32)
    const size_t n = (size_t)(hi - lo) * row;
    if (int rc = ensure_staging(ctx, 2 * n)) return rc;
    for (int h = 0; h < ctx->kvh_count; ++h) {
      const size_t dst = ((size_t)(ctx->cfg.kv_head_begin + h) * n_pos + (lo - pos0)) * row;
      const long long off = (long long)layer * ctx->layer_elems + (long long)h * ctx->head_elems +
                            (long long)(lo - ctx->cfg.seq_begin) * row;
      const int nb = (int)std::min<size_t>((n / 32 + 255) / 256, 4096);
      q8_dequant_kernel<<<nb, 256, 0, ctx->stream>>>(ctx->k8 + off, ctx->ksc + off / 32, (long long)n / 32, ctx->st_buf);
      q8_dequant_kernel<<<nb, 256, 0, ctx->stream>>>(ctx->v8 + off, ctx->vsc + off / 32, (long long)n / 32,
                                                     ctx->st_buf + n);
      ctx->launches += 2;
      L3P_CUDA(ctx, cudaGetLastError());
      L3P_CUDA(ctx, cudaMemcpyAsync(k + dst, ctx->st_buf, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
      L3P_CUDA(ctx, cudaMemcpyAsync(v + dst, ctx->st_buf + n, n * 4, cudaMemcpyDeviceToHost, ctx->stream));
    }
    return finish_host_call(ctx);
  }
  for (int h = 0; h < ctx->kvh_count; ++h) {
    const size_t dst = ((size_t)(ctx->cfg.kv_head_begin + h) * n_pos + (lo - pos0)) * row;
    const size_t src = (size_t)layer * ctx->layer_elems + (size_t)h * ctx->head_elems +
                       (size_t)(lo - ctx->cfg.seq_begin) * row;
    L3P_CUDA(ctx, cudaMemcpyAsync(k + dst, ctx->kc + src, (size_t)(hi - lo) * row * 4, cudaMemcpyDeviceToHost, ctx->stream));
    L3P_CUDA(ctx, cudaMemcpyAsync(v + dst, ctx->vc + src, (size_t)(hi - lo) * row * 4, cudaMemcpyDeviceToHost, ctx->stream));
  }
  return finish_host_call(ctx);
}

// The Q8_0 cache in the reference's own block format: per owned KV head and
// owned position in [pos0, pos0+n_pos), head_dim/32 blocks of 34 bytes (fp16
// scale, little-endian, then 32 int8) -- the bytes of the reference's
// key_cache/value_cache rows (c:365-372).  blocks: [n_kv_heads][n_pos][head_dim/32*34].
namespace {
int q8_block_io(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, uint8_t* kb, uint8_t* vb, const uint8_t* kin,
                const uint8_t* vin) {
  if (!ctx || n_pos < 0 || (!kb && !kin)) return ctx ? fail(ctx, L3P_E_INVAL, "bad argument") : L3P_E_INVAL;
  if (!ctx->q8) return fail(ctx, L3P_E_INVAL, "the cache is not Q8_0");
  if (int rc = check_layer(ctx, layer)) return rc;
  if (pos0 < 0 || pos0 + n_pos > ctx->cfg.seq_len)
    return fail(ctx, L3P_E_RANGE, "positions [%d, %d) outside [0, %d)", pos0, pos0 + n_pos, ctx->cfg.seq_len);
  const int lo = std::max(pos0, ctx->cfg.seq_begin), hi = std::min(pos0 + n_pos, ctx->cfg.seq_begin + ctx->seq_count);
  if (hi <= lo) return L3P_OK;
  CtxScope dev(ctx);
  const size_t rowb = (size_t)ctx->hd / 32 * 34;
  const long long nblk = (long long)(hi - lo) * (ctx->hd / 32);
  const size_t bytes = (size_t)nblk * 34;
  if (int rc = ensure_staging(ctx, (2 * bytes + 3) / 4)) return rc;
  uint8_t* st_k = reinterpret_cast<uint8_t*>(ctx->st_buf);
  uint8_t* st_v = st_k + bytes;
  const int nb = (int)std::min<long long>((nblk + 255) / 256, 4096);
  for (int h = 0; h < ctx->kvh_count; ++h) {
    const size_t hoff = ((size_t)(ctx->cfg.kv_head_begin + h) * n_pos + (lo - pos0)) * rowb;
    const long long off = (long long)layer * ctx->layer_elems + (long long)h * ctx->head_elems +
                          (long long)(lo - ctx->cfg.seq_begin) * ctx->hd;
    if (kin) {
      L3P_CUDA(ctx, cudaMemcpyAsync(st_k, kin + hoff, bytes, cudaMemcpyHostToDevice, ctx->stream));
      L3P_CUDA(ctx, cudaMemcpyAsync(st_v, vin + hoff, bytes, cudaMemcpyHostToDevice, ctx->stream));
      q8_unblock_kernel<<<nb, 256, 0, ctx->stream>>>(st_k, nblk, ctx->k8 + off, ctx->ksc + off / 32);
      q8_unblock_kernel<<<nb, 256, 0, ctx->stream>>>(st_v, nblk, ctx->v8 + off, ctx->vsc + off / 32);
    } else {
      q8_blocks_kernel<<<nb, 256, 0, ctx->stream>>>(ctx->k8 + off, ctx->ksc + off / 32, nblk, st_k);
      q8_blocks_kernel<<<nb, 256, 0, ctx->stream>>>(ctx->v8 + off, ctx->vsc + off / 32, nblk, st_v);
    }
    ctx->launches += 2;
    L3P_CUDA(ctx, cudaGetLastError());
    if (!kin) {
      L3P_CUDA(ctx, cudaMemcpyAsync(kb + hoff, st_k, bytes, cudaMemcpyDeviceToHost, ctx->stream));
      L3P_CUDA(ctx, cudaMemcpyAsync(vb + hoff, st_v, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    }
    // the staging buffer is reused by the next head
    L3P_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  }
  return finish_host_call(ctx);
}
}  // namespace

L3P_API int l3p_attn_read_kv_q8(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, uint8_t* k_blocks,
                                uint8_t* v_blocks) {
  if (!k_blocks || !v_blocks) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  return q8_block_io(ctx, layer, pos0, n_pos, k_blocks, v_blocks, nullptr, nullptr);
}

L3P_API int l3p_attn_load_kv_q8(l3p_attn_ctx* ctx, int layer, int pos0, int n_pos, const uint8_t* k_blocks,
                                const uint8_t* v_blocks) {
  if (!k_blocks || !v_blocks) return ctx ? fail(ctx, L3P_E_INVAL, "null pointer") : L3P_E_INVAL;
  return q8_block_io(ctx, layer, pos0, n_pos, nullptr, nullptr, k_blocks, v_blocks);
}

// ==========================================================================
// Decode without any allocation (l3p_attn_decode_noalloc).
//
// For callers that own every byte of device memory themselves -- an engine
// that plans one arena when the model loads and hands out pointers from it --
// and therefore cannot let a library call cudaMalloc on the token path: a
// runtime allocation can synchronise the device, can fail mid-generation
// once the arena has taken the memory, and escapes the caller's accounting.
// The caller passes the KV cache, q and out; the split-K partials and the
// per-unit tickets live in the fixed array below, which every GPU that loads
// this library holds until the process exits.
//
// The per-device set-up below (the array's device address, the kernel's
// shared-memory attribute) is cached for the life of the process: it assumes
// the device's primary context lives as long as the process does.  A caller
// that resets a device (cudaDeviceReset) or releases and re-creates its
// primary context must not call this entry point on that device afterwards.

namespace {

constexpr long long kNoAllocFloats = 512 * 1024;     // 2 MiB: partial outputs + (m, l) pairs
constexpr long long kNoAllocCounters = 1024;          // tickets, one per (KV head, q-head group)
constexpr int kMaxDevices = 64;

__device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats + kNoAllocCounters];

struct NoAllocDevice {
  bool ready = false;
  float* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int num_sms = 0;
};
NoAllocDevice g_noalloc_dev[kMaxDevices];
unsigned g_noalloc_attr_done[kMaxDevices];  // bit i: smem attribute set for kernel table entry i
std::mutex g_noalloc_mu;
thread_local char g_noalloc_err[256];

int noalloc_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_noalloc_err, sizeof g_noalloc_err, fmt, ap);
  va_end(ap);
  return code;
}

int kernel_index(int hd, int gt) {
  const int h = hd == 64 ? 0 : hd == 128 ? 1 : hd == 256 ? 2 : -1;
  const int g = gt == 1 ? 0 : gt == 2 ? 1 : gt == 4 ? 2 : gt == 8 ? 3 : -1;
  return (h < 0 || g < 0) ? -1 : h * 4 + g;
}

}  // namespace

L3P_API const char* l3p_attn_noalloc_last_error(void) { return g_noalloc_err; }

L3P_API int l3p_attn_decode_noalloc(const l3p_attn_config* cfg, int layer, int pos, const float* k_cache,
                                    const float* v_cache, const float* q, float* out, void* stream) {
  g_noalloc_err[0] = '\0';
  if (!cfg || !k_cache || !v_cache || !q || !out) return noalloc_fail(L3P_E_INVAL, "null argument");
  const l3p_attn_config& c = *cfg;
  if (c.n_heads <= 0 || c.n_kv_heads <= 0 || c.seq_len <= 0 || c.n_heads % c.n_kv_heads != 0 ||
      c.kv_format != L3P_KV_F32)
    return noalloc_fail(L3P_E_INVAL, "bad configuration");
  const int kvh_count = c.kv_head_count > 0 ? c.kv_head_count : c.n_kv_heads - c.kv_head_begin;
  if (c.kv_head_begin < 0 || kvh_count <= 0 || c.kv_head_begin + kvh_count > c.n_kv_heads)
    return noalloc_fail(L3P_E_INVAL, "bad KV-head range");
  if (c.seq_begin != 0 || (c.seq_count != 0 && c.seq_count != c.seq_len))
    return noalloc_fail(L3P_E_INVAL, "the no-allocation decode needs the whole sequence (seq_begin 0)");
  if (pos < 0 || pos >= c.seq_len) return noalloc_fail(L3P_E_RANGE, "pos %d outside [0, %d)", pos, c.seq_len);
  // the layer picks the sliding-window rule (l % swa_pattern); as the context
  // entry points, reject one outside [0, n_layers) (n_layers 0: no upper bound)
  if (layer < 0 || (c.n_layers > 0 && layer >= c.n_layers))
    return noalloc_fail(L3P_E_RANGE, "layer %d outside [0, %d)", layer, c.n_layers);
  for (const void* p : {(const void*)k_cache, (const void*)v_cache, (const void*)q, (const void*)out})
    if (!aligned16(p)) return noalloc_fail(L3P_E_INVAL, "device pointer %p is not 16-byte aligned", p);
  const int hd = c.head_dim;
  const int G = c.n_heads / c.n_kv_heads;
  const int GT = (G % 8 == 0) ? 8 : (G % 4 == 0) ? 4 : (G % 2 == 0) ? 2 : 1;
  const KernelInfo ki = kernel_for(hd, GT);
  const int kidx = kernel_index(hd, GT);
  if (!ki.fn || kidx < 0) return noalloc_fail(L3P_E_UNSUPPORTED, "no decode kernel for head_dim %d", hd);

  // once per device, with that device current: the device address of the
  // scratch array and the kernel's shared-memory attribute
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return noalloc_fail(L3P_E_CUDA, "no current CUDA device");
  NoAllocDevice& d = g_noalloc_dev[dev];
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!d.ready) {
      void* ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess) return noalloc_fail(L3P_E_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return noalloc_fail(L3P_E_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
      d.scratch = static_cast<float*>(ptr);
      d.ready = true;
    }
    if (!(g_noalloc_attr_done[dev] & (1u << kidx))) {
      const cudaError_t e = cudaFuncSetAttribute(ki.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ki.smem);
      if (e != cudaSuccess) return noalloc_fail(L3P_E_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      g_noalloc_attr_done[dev] |= 1u << kidx;
    }
  }

  // split-K plan within the fixed scratch (no clusters: the partials of every
  // split go through the scratch array)
  const int swa = (c.is_gemma3 && c.swa_window > 0 && c.swa_pattern > 0 && (layer % c.swa_pattern) < c.swa_pattern - 1)
                      ? std::max(0, pos - c.swa_window + 1)
                      : 0;
  const long long P = (long long)pos + 1 - swa;
  const int n_hg = G / GT;
  const long long units = (long long)kvh_count * n_hg;
  if (units > kNoAllocCounters)
    return noalloc_fail(L3P_E_RANGE, "%lld (KV head, q-head group) units exceed the no-allocation limit of %lld",
                        units, kNoAllocCounters);
  PlanLimits lim;
  lim.hd = hd;
  lim.GT = GT;
  lim.num_sms = d.num_sms;
  lim.ws_o_floats = kNoAllocFloats * hd / (hd + 2);  // room for the (m, l) pairs after the outputs
  lim.n_counters = kNoAllocCounters;
  const Plan plan = plan_splits(&lim, P, units, ki.rows, ki.ctas_per_sm);
  const long long o_floats = plan.nsplit > 1 ? units * plan.nsplit * GT * hd : 0;
  const long long ml_floats = plan.nsplit > 1 ? units * plan.nsplit * GT * 2 : 0;
  if (o_floats + ml_floats > kNoAllocFloats)
    return noalloc_fail(L3P_E_RANGE, "split partials need %lld floats, above the no-allocation limit of %lld",
                        o_floats + ml_floats, kNoAllocFloats);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* ws_o = d.scratch;
  float* ws_ml = d.scratch + o_floats;
  unsigned* counters = reinterpret_cast<unsigned*>(d.scratch + kNoAllocFloats);
  if (plan.nsplit > 1) {
    // tickets must start at zero; an earlier call may have stopped early
    const cudaError_t e = cudaMemsetAsync(counters, 0, units * sizeof(unsigned), s);
    if (e != cudaSuccess) return noalloc_fail(L3P_E_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  }

  DecodeArgs a{};
  a.kc = k_cache;
  a.vc = const_cast<float*>(v_cache);
  a.kc_w = const_cast<float*>(k_cache);
  a.layer_stride = 0;
  a.head_stride = (long long)c.seq_len * hd;
  a.q = q;
  a.q_zstride = (long long)c.n_heads * hd;
  a.out = out;
  a.ml_zstride = 2ll * c.n_heads;
  a.ws_o = ws_o;
  a.ws_ml = ws_ml;
  a.counters = counters;
  a.scale = c.scale != 0.f ? c.scale : 1.0f / sqrtf((float)hd);
  a.layer0 = layer;
  a.pos0 = pos;
  a.seq_begin = 0;
  a.cap = c.seq_len;
  a.kv_head_begin = c.kv_head_begin;
  a.G = G;
  a.n_hg = n_hg;
  a.nsplit = plan.nsplit;
  a.cluster = 1;
  a.is_gemma3 = c.is_gemma3;
  a.swa_window = c.swa_window;
  a.swa_pattern = c.swa_pattern;
  a.wait_pos = INT_MAX;  // plain stream order: every earlier store has landed
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(plan.nsplit, kvh_count * n_hg, 1);
  lc.blockDim = dim3(kDecodeThreads, 1, 1);
  lc.dynamicSmemBytes = ki.smem;
  lc.stream = s;
  const cudaError_t e = cudaLaunchKernelEx(&lc, ki.fn, a);
  if (e != cudaSuccess) return noalloc_fail(L3P_E_CUDA, "launch: %s", cudaGetErrorString(e));
  return L3P_OK;
}
