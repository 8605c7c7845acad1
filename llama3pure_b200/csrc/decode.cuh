// decode.cuh -- split-K flash-decoding over an fp32 KV cache (sm_100a).
//
// Replaces the reference's per-layer decode attention loop
// (llama3pure-c-engine.c:3310-3359): scores q.K^T for every cached position
// of the window, softmax, and the softmax-weighted sum of V rows, for all
// q heads of a GQA group (c:3333-3357).  The same kernel serves the
// token-by-token causal prefill (c:3582-3612) with one grid slice per token,
// and can take the new token's K/V row straight from its producer (fused
// append, c:3299-3308).
//
// Work decomposition
//   grid.x  split of the attended position range (split-K)
//   grid.y  (owned KV head, group of GT q heads of that KV head)
//   grid.z  layer (multi-layer decode) or token (prefill)
// One CTA of 8 warps reads every K and V row of its share of the range once
// and serves all GT q heads of the group with it (the reference re-reads
// every V row once per q head, c:3352-3357).  The range is cut into tiles of
// R rows dealt round-robin over the CTAs of the unit and their warps, so at
// any moment all SMs read neighbouring tiles.  Each warp streams its tiles
// through a private ring of kStages shared-memory stages with 16-byte
// cp.async copies (kStages-1 tiles in flight while it computes on one);
// copies past the range zero-fill instead of reading.
//
// Per tile a warp forms R*GT partial dot products per lane, reduces them with
// a transposing butterfly (31 shuffles for 32 values, leaving lane j the full
// score of value j), and runs the online softmax in base 2: running max m and
// running sum l per q head, accumulator rescaled by 2^(m_old - m_new).
//
// Merging, so that one launch produces the final normalised output:
//   1. the warps of a CTA, in shared memory;
//   2. the CTAs of a thread-block cluster (up to 16, one cluster per unit
//      when it fits in a wave), through distributed shared memory, each rank
//      merging a slice of the output elements;
//   3. only when a unit spans several clusters (or runs without clusters),
//      the last part to finish merges the parts' partials from global scratch
//      (atomic ticket on a per-unit counter).
//
// Differences from the reference's arithmetic, all inside the 1e-4 contract:
//   * summation order (lane-parallel dot products, blocked softmax sums);
//   * exp via ex2.approx on log2(e)-scaled scores instead of libm expf;
//   * the reference skips V rows whose final weight is below 1e-8 in
//     magnitude (c:1602).  A one-pass online softmax does not know the final
//     weight when it reads V, so every row contributes; the difference is at
//     most (number of such rows) * 1e-8 * max|v| per output element.
#pragma once
#include <cooperative_groups.h>

#include "ptx.cuh"

namespace l3p {

namespace cg = cooperative_groups;

constexpr int kMaxSplits = 160;  // CTAs sharing one position range per launch
constexpr int kMaxCluster = 16;  // CTAs of one thread-block cluster (non-portable size)
constexpr int kMergeBatch = 16;  // partials fetched together by the global merge

// 16-byte global->shared copy; src_bytes = 0 writes zeros and reads nothing.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_gpu(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_gpu(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// L2 prefetch of the 128-byte lines of [p, p + bytes): thread t of the CTA
// takes line t.  L2 is the point of coherence of global memory, so a line
// fetched before its producer (the kernel before this one) writes it still
// reads the written values afterwards.
__device__ __forceinline__ void prefetch_l2(const void* p, int bytes) {
  const int line = (int)threadIdx.x;
  if (line * 128 < bytes)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(p) + line * 128));
}
// Programmatic dependent launch: let the next kernel of the stream start
// launching, and wait for the previous kernel's results (no-ops when the
// launch carries no programmatic dependency).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

struct DecodeArgs {
  const float* kc;         // K cache, all layers: [n_layers][kvh_count][cap][HD]
  float* vc;               // V cache, same layout
  int8_t* k8;              // Q8_0 cache (decode_q8_kernel): int8 values, same layout as kc
  int8_t* v8;              //   (written only by the fused append)
  uint16_t* ksc;           // fp16 block scales: [n_layers][kvh_count][cap][HD/32]
  uint16_t* vsc;
  float* kc_w;             // writable alias of kc (fused append)
  long long layer_stride;  // kvh_count * cap * HD
  long long head_stride;   // cap * HD
  const float* q;          // row of absolute q head h in slice z: q + z*q_zstride + h*HD
  long long q_zstride;
  const float* k_new;      // optional: token row of slice z at k_new + z*new_zstride (all KV heads)
  const float* v_new;
  long long new_zstride;
  float* out;              // final output, indexed like q (partial == 0)
  float* part_o;           // normalised partial output, indexed like q (partial == 1)
  float* part_ml;          // (m, l) per q head: part_ml + z*ml_zstride + 2*h
  long long ml_zstride;
  float* ws_o;             // split scratch [units][nsplit][GT][HD]
  float* ws_ml;            // split scratch [units][nsplit][GT][2]
  unsigned* counters;      // [units] tickets, zero between launches
  int* err;                // device error word
  float scale;             // attention scale applied to q
  int layer0, layer_step;  // layer of slice z = layer0 + z*layer_step
  int pos0, pos_step;      // query position of slice z = pos0 + z*pos_step
  int seq_begin, cap;      // cache row r holds position seq_begin + r
  int kv_head_begin;       // absolute index of the first owned KV head
  int G, n_hg;             // q heads per KV head (kv_mul), groups of GT per KV head
  int nsplit;              // CTAs per unit
  int cluster;             // CTAs per thread-block cluster (1 = no cluster); divides nsplit
  int is_gemma3, swa_window, swa_pattern;
  int partial;
  // mergers of the global stage (no cluster): the last merge_k parts to
  // finish each merge 1/merge_k of the output; > 1 only for launches whose
  // CTAs are all resident at once (a merger waits for the unit's last part)
  int merge_k;
  // cache rows of positions >= wait_pos may still be being stored by an
  // earlier launch in flight: copied only after griddepcontrol.wait (INT_MAX: none)
  int wait_pos;
  unsigned long long* trace;  // per-CTA stage stamps (builds with L3P_DECODE_TRACE), or null
  // designated mergers (one-wave launches without clusters; null: the ticket
  // scheme): flags[unit * nsplit + part] = number of mergers still to read
  // part's partial; parts [0, merge_k) merge, each 1/merge_k of the output
  unsigned* flags;
  // host-call server (server.cuh): a nonzero flag_tag makes every part store
  // the tag (the call number) as its flag instead of a count, and mergers wait
  // for the tag, so nothing returns the flags to 0
  unsigned flag_tag;
};

// Decode trace, compiled in only with -DL3P_DECODE_TRACE (a separate build for
// timing studies; the shipped library has none): thread 0 of every CTA stores
// %globaltimer (ns) at the stages of a launch into trace[cta][k]:
//   0 CTA start                      1 griddepcontrol.wait returned
//   2 q ready                        3 position loop done (last copy landed)
//   4 partial published, ticket taken 5 CTA exit
#ifdef L3P_DECODE_TRACE
__device__ __forceinline__ void trace_stamp(unsigned long long* t, int k) {
  if (t && threadIdx.x == 0)
    t[(((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 8 + k] = globaltimer_ns();
}
#else
__device__ __forceinline__ void trace_stamp(unsigned long long*, int) {}
#endif

#ifndef L3P_DECODE_WARPS
#define L3P_DECODE_WARPS 8  // warps per CTA
#endif
#ifndef L3P_DECODE_RING_KB
#define L3P_DECODE_RING_KB 192  // shared-memory ring per CTA
#endif
#ifndef L3P_DECODE_ROWS
#define L3P_DECODE_ROWS 8  // rows per tile for groups of <= 4 q heads and head_dim <= 128
#endif

template <int HD, int GT>
struct DecodeCfg {
  static_assert(HD == 64 || HD == 128 || HD == 256, "head_dim");
  static_assert(GT == 1 || GT == 2 || GT == 4 || GT == 8, "group");
  static constexpr int kWarps = L3P_DECODE_WARPS;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kR = (GT >= 8 || HD >= 256) ? 4 : L3P_DECODE_ROWS;  // rows per tile
  static constexpr int kNV = kR * GT;           // partial sums per lane per tile
  static constexpr int kLogNV = (kNV == 32) ? 5 : (kNV == 16) ? 4 : (kNV == 8) ? 3 : 2;
  static constexpr int kSH = 5 - kLogNV;        // lane j holds value (j >> kSH)
  static constexpr int kEPL = HD / 32;          // elements of a row per lane
  static constexpr int kTileFloats = kR * HD;
  static constexpr int kCopies = kTileFloats / 128;     // 16-byte copies per lane per tile
  static constexpr int kStageFloats = 2 * kTileFloats;  // K tile + V tile
  static constexpr int kStageBytes = kStageFloats * 4;
  static constexpr int kStagesRaw = (L3P_DECODE_RING_KB * 1024 / kWarps) / kStageBytes;
  static constexpr int kStages = kStagesRaw < 1 ? 1 : (kStagesRaw > 8 ? 8 : kStagesRaw);
  static constexpr int kRingBytes = kWarps * kStages * kStageBytes;
  static constexpr int kSmemBytes = kRingBytes;
  static_assert(kNV <= 32, "values per tile");
  static_assert(kWarps * GT * HD * 4 <= kRingBytes, "merge buffer fits in the ring");
  static_assert(kMaxSplits * GT * 3 * 4 <= kRingBytes, "split merge buffer fits in the ring");
  static_assert(kSmemBytes <= 200 * 1024, "ring fits the SM");
  static constexpr int kCtasPerSm = (kSmemBytes + 8 * 1024) * 2 <= 227 * 1024 ? 2 : 1;
  // Narrow score phase: 8 lanes share a K row (4 rows per warp pass), so the
  // cross-lane reduction is 3 levels over 8 values instead of 5 over 32.
  // Used when a tile holds exactly 8 (row pass, q head) values per lane and
  // the lane's slice of q fits in registers (head_dim <= 128).
  static constexpr bool kNarrow = HD <= 128 && (kR / 4) * GT == 8 && GT * (HD / 8) <= 64;
  static constexpr int kSegC = HD / 32;  // 16-byte chunks of a row per lane (narrow phase)
};

// Shared-memory position of 16-byte chunk `ch` of a K/V row.  The narrow
// score phase reads chunks sg*kSegC + c with 8 lanes per row; XOR-ing the chunk
// with bits of its segment spreads those reads (and the 32-lane V reads) over
// all eight 16-byte bank groups.
template <int HD, bool ON>
__device__ __forceinline__ int swz(int ch) {
  if constexpr (ON) {
    return ch ^ ((ch >> 3) & (HD / 32 - 1));
  } else {
    return ch;
  }
}

// Elements of a row owned by a lane: HD=64 -> {2*lane, 2*lane+1};
// HD>=128 -> {c*128 + 4*lane + i}, so every warp-wide 16-byte access is
// contiguous and shared-memory bank-conflict free.
template <int HD>
__device__ __forceinline__ int lane_elem(int lane, int i) {
  if constexpr (HD == 64) {
    return 2 * lane + i;
  } else {
    return (i >> 2) * 128 + 4 * lane + (i & 3);
  }
}

template <int HD>
__device__ __forceinline__ void load_row(const float* row, float (&x)[HD / 32], int lane) {
  if constexpr (HD == 64) {
    const float2 t = *reinterpret_cast<const float2*>(row + 2 * lane);
    x[0] = t.x;
    x[1] = t.y;
  } else {
#pragma unroll
    for (int c = 0; c < HD / 128; ++c) {
      const float4 t = *reinterpret_cast<const float4*>(row + c * 128 + 4 * lane);
      x[4 * c + 0] = t.x;
      x[4 * c + 1] = t.y;
      x[4 * c + 2] = t.z;
      x[4 * c + 3] = t.w;
    }
  }
}

// Transposing butterfly: NV per-lane values -> lane j holds the warp-wide
// sum of value (j >> (5 - log2 NV)) in v[0].
template <int NV>
__device__ __forceinline__ void transpose_reduce(float (&v)[NV], int lane) {
#pragma unroll
  for (int n = NV, off = 16; n > 1; n >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  // values fewer than lanes: finish with a plain butterfly over the low bits
#pragma unroll
  for (int off = (32 / NV) >> 1; off > 0; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
}

__device__ __forceinline__ int swa_start(const DecodeArgs& a, int layer, int pos) {
  // c:3316-3321: Gemma-3 SWA layers (l % pattern < pattern - 1) see
  // [pos - window + 1, pos]; all other layers see [0, pos].
  if (a.is_gemma3 && a.swa_window > 0 && a.swa_pattern > 0 &&
      (layer % a.swa_pattern) < a.swa_pattern - 1) {
    const int s = pos - a.swa_window + 1;
    return s < 0 ? 0 : s;
  }
  return 0;
}

// Shared state of the merge stages (per CTA).
template <int GT, int W>
struct DecodeMergeSmem {
  float m[W][GT];   // per-warp running max
  float l[W][GT];   // per-warp running sum
  float ww[W][GT];  // warp merge weights
  float cm[GT], cl[GT];   // CTA partial (max, sum), read by the cluster
  float rw[kMaxCluster][GT];  // cluster merge weights
  float M[GT], L[GT];
  int last;
  int mk;  // mergers of the global stage
};

// One batch of the global merge: fold parts sp0, sp0 + stride, ... (up to
// kMergeBatch of them, those < n_parts) of one q head's float4 into the
// running (M, L, O).  ml2 points at the head's (m, l) of part 0 ([part][GT]
// float2), o4 at its float4 of part 0 ([part][GT*HD/4] float4).  All loads are
// issued before any is used.
template <int GT, int HD>
__device__ __forceinline__ void merge_part_batch(const float2* ml2, const float4* o4, int sp0, int stride,
                                                 int n_parts, float& M, float& L, float4& O) {
  float2 ml[kMergeBatch];
  float4 v[kMergeBatch];
#pragma unroll
  for (int j = 0; j < kMergeBatch; ++j) {
    const int sp = sp0 + j * stride;
    ml[j] = sp < n_parts ? __ldcg(ml2 + (long long)sp * GT) : make_float2(-INFINITY, 0.f);
    v[j] = sp < n_parts ? __ldcg(o4 + (long long)sp * (GT * HD / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float Mb = M;
#pragma unroll
  for (int j = 0; j < kMergeBatch; ++j) Mb = fmaxf(Mb, ml[j].x);
  if (Mb == -INFINITY) return;
  const float r = fast_exp2(M - Mb);  // rescale what was accumulated so far
  L *= r;
  O.x *= r;
  O.y *= r;
  O.z *= r;
  O.w *= r;
#pragma unroll
  for (int j = 0; j < kMergeBatch; ++j) {
    const float w = fast_exp2(ml[j].x - Mb);  // 0 for empty partials (m = -inf)
    L = fmaf(ml[j].y, w, L);
    O.x = fmaf(v[j].x, w, O.x);
    O.y = fmaf(v[j].y, w, O.y);
    O.z = fmaf(v[j].z, w, O.z);
    O.w = fmaf(v[j].w, w, O.w);
  }
  M = Mb;
}

// Everything after the position loop of a decode kernel: merge the W warps of
// the CTA (their running (m, l) already in ms.m / ms.l, their accumulators in
// acc with lane_elem<HD> layout), then the CTAs of a cluster, then -- when a
// unit spans several clusters -- the parts of the unit through global scratch,
// and write the normalised output (or the partial triple).  The ring is free
// on entry and becomes the merge buffer.  Shared by the fp32 and Q8_0 kernels.
template <int HD, int GT, int W, int T>
__device__ __forceinline__ void decode_finish(const DecodeArgs& a, DecodeMergeSmem<GT, W>& ms, float* ring,
                                              const float (&acc)[GT][HD / 32], int warp, int lane, int split,
                                              int unit, int z, int h0) {
  float (&s_m)[W][GT] = ms.m;
  float (&s_l)[W][GT] = ms.l;
  float (&s_ww)[W][GT] = ms.ww;
  float (&s_cm)[GT] = ms.cm;
  float (&s_cl)[GT] = ms.cl;
  float (&s_rw)[kMaxCluster][GT] = ms.rw;
  float (&s_M)[GT] = ms.M;
  float (&s_L)[GT] = ms.L;
  int& s_last = ms.last;
  (void)s_m;
  (void)s_l;
  // ---- CTA partial: merge the warps (the ring becomes the merge buffer) ----
  float* wacc = ring;                          // [kWarps][GT][HD]
  float* cta_o = ring + W * GT * HD;   // [GT][HD], unnormalised, relative to s_cm
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < HD / 32; ++e) wacc[(warp * GT + g) * HD + lane_elem<HD>(lane, e)] = acc[g][e];
  __syncthreads();
  if (threadIdx.x < GT) {
    const int g = threadIdx.x;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      const float f = (M == -INFINITY) ? 0.f : fast_exp2(s_m[w][g] - M);
      s_ww[w][g] = f;
      L = fmaf(s_l[w][g], f, L);
    }
    s_cm[g] = M;
    s_cl[g] = L;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < GT * HD; idx += T) {
    const int g = idx / HD;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) O = fmaf(wacc[w * GT * HD + idx], s_ww[w][g], O);
    cta_o[idx] = O;
  }
  __syncthreads();

  float* const out_base = (a.partial ? a.part_o : a.out) + (long long)z * a.q_zstride + (long long)h0 * HD;
  float* const ml_base = a.partial ? a.part_ml + (long long)z * a.ml_zstride + 2 * h0 : nullptr;

  if (a.nsplit == 1) {  // this CTA covers the whole range
    trace_stamp(a.trace, 4);
    for (int idx = threadIdx.x; idx < GT * HD; idx += T) {
      const float L = s_cl[idx / HD];
      out_base[idx] = (a.partial && !(L > 0.f)) ? 0.f : cta_o[idx] / L;
    }
    if (ml_base && threadIdx.x < GT) {
      ml_base[2 * threadIdx.x] = s_cm[threadIdx.x];
      ml_base[2 * threadIdx.x + 1] = s_cl[threadIdx.x];
    }
    trace_stamp(a.trace, 5);
    return;
  }

  int n_parts = a.nsplit;  // partials the global stage merges
  int part = split;
  int rank = 0, cs = 1;
  int mergers = 1;  // CTAs of the global stage that each merge a slice, without a cluster
  bool flag_merge = false;  // designated mergers (a.flags): flags, not the ticket, to reset
  if (a.cluster > 1) {
    // ---- cluster stage: the CTAs of a cluster merge through distributed shared memory ----
    cg::cluster_group cluster = cg::this_cluster();
    cs = (int)cluster.num_blocks();
    rank = (int)cluster.block_rank();
    n_parts = a.nsplit / cs;
    part = split / cs;
    cluster.sync();  // every CTA partial of the cluster is in shared memory
    if (threadIdx.x < GT) {
      const int g = threadIdx.x;
      float M = -INFINITY;
      for (int r = 0; r < cs; ++r) M = fmaxf(M, *cluster.map_shared_rank(&s_cm[g], r));
      float L = 0.f;
      for (int r = 0; r < cs; ++r) {
        const float m = *cluster.map_shared_rank(&s_cm[g], r);
        const float f = (M == -INFINITY) ? 0.f : fast_exp2(m - M);
        s_rw[r][g] = f;
        L = fmaf(*cluster.map_shared_rank(&s_cl[g], r), f, L);
      }
      s_M[g] = M;
      s_L[g] = L;
    }
    __syncthreads();
    // this rank owns elements [rank*slice, (rank+1)*slice) of the group's output
    const int slice = GT * HD / cs;
    const bool last_stage = n_parts == 1;
    const long long gslot = ((long long)unit * n_parts + part) * GT * HD;
    for (int t = threadIdx.x; t < slice; t += T) {
      const int idx = rank * slice + t;
      const int g = idx / HD;
      float O = 0.f;
      for (int r = 0; r < cs; ++r) O = fmaf(*cluster.map_shared_rank(&cta_o[idx], r), s_rw[r][g], O);
      if (last_stage) {
        const float L = s_L[g];
        out_base[idx] = (a.partial && !(L > 0.f)) ? 0.f : O / L;
      } else {
        a.ws_o[gslot + idx] = O;
      }
    }
    if (threadIdx.x < GT) {
      if (last_stage) {
        if (ml_base && rank == 0) {
          ml_base[2 * threadIdx.x] = s_M[threadIdx.x];
          ml_base[2 * threadIdx.x + 1] = s_L[threadIdx.x];
        }
      } else if (rank == 0) {
        a.ws_ml[(((long long)unit * n_parts + part) * GT + threadIdx.x) * 2] = s_M[threadIdx.x];
        a.ws_ml[(((long long)unit * n_parts + part) * GT + threadIdx.x) * 2 + 1] = s_L[threadIdx.x];
      }
    }
    if (last_stage) {
      cluster.sync();  // no CTA leaves while another still reads its shared memory
      trace_stamp(a.trace, 4);
      trace_stamp(a.trace, 5);
      return;
    }
    __threadfence();
    cluster.sync();  // the cluster's partial is written and visible
    if (rank == 0 && threadIdx.x == 0) {
      const int last = atomicAdd(&a.counters[unit], 1u) == (unsigned)(n_parts - 1);
      for (int r = 0; r < cs; ++r) *cluster.map_shared_rank(&s_last, r) = last;
    }
    cluster.sync();
  } else if (a.flags) {
    // ---- no cluster, designated mergers: every part publishes its partial
    // and then its flag (release, no atomic round trip); parts [0, merge_k)
    // -- resident, as every CTA of a one-wave launch is -- wait until every
    // flag is set (one flag per thread, all polled at once) and merge their
    // slice of the output in the global stage below.  Each merger then takes
    // 1 off every flag; the flags return to 0. ----
    const long long gslot = ((long long)unit * n_parts + part) * GT * HD;
    for (int idx = threadIdx.x; idx < GT * HD; idx += T) a.ws_o[gslot + idx] = cta_o[idx];
    if (threadIdx.x < GT) {
      a.ws_ml[(((long long)unit * n_parts + part) * GT + threadIdx.x) * 2] = s_cm[threadIdx.x];
      a.ws_ml[(((long long)unit * n_parts + part) * GT + threadIdx.x) * 2 + 1] = s_cl[threadIdx.x];
    }
    __syncthreads();
    unsigned* const fl = a.flags + (long long)unit * n_parts;
    if (threadIdx.x == 0) {
      fence_acq_rel_gpu();  // the partial (all threads' stores, ordered by the barrier) before the flag
      st_relaxed_gpu(fl + part, a.flag_tag ? a.flag_tag : (unsigned)a.merge_k);
    }
    trace_stamp(a.trace, 4);
    if (part >= a.merge_k) {
      trace_stamp(a.trace, 5);
      return;
    }
    bool arrived = true;
    const unsigned long long t0 = globaltimer_ns();
    for (int sp = threadIdx.x; sp < n_parts && arrived; sp += T)
      while (a.flag_tag ? ld_acquire_gpu(fl + sp) != a.flag_tag : ld_acquire_gpu(fl + sp) == 0u) {
        if (globaltimer_ns() - t0 > kGroupWaitNs) {
          *reinterpret_cast<volatile int*>(a.err) = kErrTimeout;
          arrived = false;
          break;
        }
        __nanosleep(20);
      }
    if (!__syncthreads_and(arrived)) {  // the barrier also orders every thread's reads after the acquires
      trace_stamp(a.trace, 5);
      return;
    }
    rank = part;
    cs = mergers = a.merge_k;
    s_last = 1;  // (read only below, by this CTA)
    flag_merge = true;
  } else {
    // ---- no cluster: every CTA is a part of the global stage ----
    const long long gslot = ((long long)unit * n_parts + part) * GT * HD;
    for (int idx = threadIdx.x; idx < GT * HD; idx += T) a.ws_o[gslot + idx] = cta_o[idx];
    if (threadIdx.x < GT) {
      a.ws_ml[(((long long)unit * n_parts + part) * GT + threadIdx.x) * 2] = s_cm[threadIdx.x];
      a.ws_ml[(((long long)unit * n_parts + part) * GT + threadIdx.x) * 2 + 1] = s_cl[threadIdx.x];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0 && a.merge_k <= 1) {
      s_last = atomicAdd(&a.counters[unit], 1u) == (unsigned)(n_parts - 1);
      ms.mk = 1;
    } else if (threadIdx.x == 0) {
      // the last merge_k arrivals become mergers 0 .. merge_k-1; all but the
      // last wait (bounded) until every part has arrived
      const int k = a.merge_k;
      const int t = (int)atomicAdd(&a.counters[unit], 1u);
      int j = t - (n_parts - k);
      if (j >= 0 && t != n_parts - 1) {
        const unsigned long long t0 = globaltimer_ns();
        while ((int)ld_acquire_gpu(&a.counters[unit]) < n_parts) {
          if (globaltimer_ns() - t0 > kGroupWaitNs) {
            *reinterpret_cast<volatile int*>(a.err) = kErrTimeout;
            j = -1;
            break;
          }
          __nanosleep(32);
        }
      }
      s_last = j >= 0 ? j + 1 : 0;  // 0: not a merger
      ms.mk = k;
    }
    __syncthreads();
    rank = s_last - 1;
    cs = mergers = ms.mk;
  }
  if (!flag_merge) {
    trace_stamp(a.trace, 4);
    if (!s_last) {
      trace_stamp(a.trace, 5);
      return;
    }
    __threadfence();
  }

  // ---- global stage: the last part to finish merges all n_parts partials ----
  // (with a cluster, each rank of the last cluster merges its slice; without,
  // each of the last merge_k parts).  A merger's thread takes one float4 of
  // the slice and fetches the (m, l) pairs and float4s of kMergeBatch parts in
  // one batch, so 16 parts cost a single L2 round trip.  With several mergers
  // the slice is small, so its threads also split the parts into pg groups
  // (thread t: float4 t % slice4, parts t / slice4 + pg * i) whose partial
  // merges combine in shared memory: ceil(n_parts / (pg * kMergeBatch)) round
  // trips.  (Splitting the parts of a single merger measured slower.)
  const long long slot0 = (long long)unit * n_parts;
  const int slice4 = GT * HD / 4 / cs;
  int pg = 1;
  if (mergers > 1 || flag_merge)  // pg * slice4 <= T: one float4 and part group per thread
    while (2 * pg * slice4 <= T && pg * kMergeBatch < n_parts) pg *= 2;
  const float2* ml2 = reinterpret_cast<const float2*>(a.ws_ml) + slot0 * GT;  // [n_parts][GT]
  const float4* o4 = reinterpret_cast<const float4*>(a.ws_o + slot0 * GT * HD);
  if (pg == 1) {
    for (int t = threadIdx.x; t < slice4; t += T) {
      const int idx4 = rank * slice4 + t;
      const int g = (idx4 * 4) / HD;
      float M = -INFINITY, L = 0.f;
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int sp0 = 0; sp0 < n_parts; sp0 += kMergeBatch)
        merge_part_batch<GT, HD>(ml2 + g, o4 + idx4, sp0, 1, n_parts, M, L, O);
      const float inv = (a.partial && !(L > 0.f)) ? 0.f : 1.f / L;
      *reinterpret_cast<float4*>(out_base + idx4 * 4) = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
      if (ml_base && (idx4 * 4) % HD == 0) {
        ml_base[2 * g] = M;
        ml_base[2 * g + 1] = L;
      }
    }
  } else {
    float4* s_o = reinterpret_cast<float4*>(ring);           // [pg][slice4] group merges
    float2* s_ml = reinterpret_cast<float2*>(ring + 4 * T);  // [pg][slice4] their (M, L)
    const int t = threadIdx.x;
    const bool on = t < slice4 * pg;
    const int f = t % slice4, grp = t / slice4;
    const int idx4 = rank * slice4 + f;
    const int g = (idx4 * 4) / HD;
    float M = -INFINITY, L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp0 = grp; on && sp0 < n_parts; sp0 += pg * kMergeBatch)
      merge_part_batch<GT, HD>(ml2 + g, o4 + idx4, sp0, pg, n_parts, M, L, O);
    if (on) {
      s_o[grp * slice4 + f] = O;
      s_ml[grp * slice4 + f] = make_float2(M, L);
    }
    __syncthreads();
    if (on && grp == 0) {
      for (int q = 1; q < pg; ++q) {
        const float2 ml = s_ml[q * slice4 + f];
        const float Mb = fmaxf(M, ml.x);
        if (Mb == -INFINITY) continue;
        const float r0 = fast_exp2(M - Mb), r1 = fast_exp2(ml.x - Mb);
        const float4 o = s_o[q * slice4 + f];
        L = L * r0 + ml.y * r1;
        O.x = O.x * r0 + o.x * r1;
        O.y = O.y * r0 + o.y * r1;
        O.z = O.z * r0 + o.z * r1;
        O.w = O.w * r0 + o.w * r1;
        M = Mb;
      }
      const float inv = (a.partial && !(L > 0.f)) ? 0.f : 1.f / L;
      *reinterpret_cast<float4*>(out_base + idx4 * 4) = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
      if (ml_base && (idx4 * 4) % HD == 0) {
        ml_base[2 * g] = M;
        ml_base[2 * g + 1] = L;
      }
    }
  }
  if (flag_merge) {
    if (a.flag_tag) {  // tagged flags are never reset
      trace_stamp(a.trace, 5);
      return;
    }
    __syncthreads();  // every thread's reads of the partials are done
    for (int sp = threadIdx.x; sp < n_parts; sp += T) red_add_gpu(a.flags + (long long)unit * n_parts + sp, 0xffffffffu);
    trace_stamp(a.trace, 5);
    return;
  }
  // ticket ready for the next launch: with several mergers the last one to
  // finish resets it (each adds one more after its merge)
  if (threadIdx.x == 0) {
    if (mergers <= 1) {
      if (rank == 0) a.counters[unit] = 0u;
    } else if (atomicAdd(&a.counters[unit], 1u) == (unsigned)(n_parts + mergers - 1)) {
      a.counters[unit] = 0u;
    }
  }
  trace_stamp(a.trace, 5);
}

// One CTA's share of a decode launch: the body of decode_f32_kernel, also run
// once per call by the host-call server (server.cuh) over the same grid.
template <int HD, int GT>
__device__ __forceinline__ void decode_f32_cta(const DecodeArgs& a, unsigned char* smem_raw) {
  using C = DecodeCfg<HD, GT>;
  float* ring = reinterpret_cast<float*>(smem_raw);
  __shared__ DecodeMergeSmem<GT, C::kWarps> ms;
  float (&s_m)[C::kWarps][GT] = ms.m;
  float (&s_l)[C::kWarps][GT] = ms.l;
  __shared__ __align__(16) float s_p[C::kNarrow ? C::kWarps : 1][C::kR * GT + 8];  // weights + rescales

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int split = blockIdx.x;
  const int kvh_local = blockIdx.y / a.n_hg;
  const int hg = blockIdx.y - kvh_local * a.n_hg;
  const int z = blockIdx.z;
  const int unit = z * gridDim.y + blockIdx.y;
  const int layer = a.layer0 + z * a.layer_step;
  const int pos = a.pos0 + z * a.pos_step;
  const int kvh = a.kv_head_begin + kvh_local;
  trace_stamp(a.trace, 0);

  const int lo = max(swa_start(a, layer, pos), a.seq_begin);
  const int hi = min(pos + 1, a.seq_begin + a.cap);
  const int n_rows = max(0, hi - lo);
  const int n_tiles = (n_rows + C::kR - 1) / C::kR;
  const int h0 = kvh * a.G + hg * GT;

  const long long row_off = (long long)layer * a.layer_stride + (long long)kvh_local * a.head_stride +
                            (long long)(lo - a.seq_begin) * HD;
  const float* kbase = a.kc + row_off;
  const float* vbase = a.vc + row_off;
  // the new token's row, when fused: read from the producer instead of the cache
  const bool fused = a.k_new != nullptr && pos >= lo && pos < hi;
  const float* knew = fused ? a.k_new + (long long)z * a.new_zstride + (long long)kvh * HD : nullptr;
  const float* vnew = fused ? a.v_new + (long long)z * a.new_zstride + (long long)kvh * HD : nullptr;
  const int new_row = pos - lo;  // index of the new token's row in the range
  // tiles holding the new row are copied only after the preceding kernel has finished
  const bool wait_new = fused;

  // tiles of this warp: t = split + nsplit * (warp + kWarps * i)
  const int first = split + a.nsplit * warp;
  const int step = a.nsplit * C::kWarps;
  const int my_tiles = n_tiles > first ? (n_tiles - first + step - 1) / step : 0;
  float* wring = ring + warp * C::kStages * C::kStageFloats;

  auto issue = [&](int i) {
    const int t = first + i * step;
    const int r0 = t * C::kR;
    float* kd = wring + (i % C::kStages) * C::kStageFloats;
    float* vd = kd + C::kTileFloats;
#pragma unroll
    for (int c = 0; c < C::kCopies; ++c) {
      const int off = c * 128 + lane * 4;  // float offset inside the tile
      const int row = r0 + off / HD;
      const bool ok = row < n_rows;
      const float* ks = kbase + (long long)r0 * HD + off;
      const float* vs = vbase + (long long)r0 * HD + off;
      if (fused && row == new_row) {
        ks = knew + (off % HD);
        vs = vnew + (off % HD);
      }
      const int ch = (off % HD) / 4;
      const int dst = off - 4 * ch + 4 * swz<HD, C::kNarrow>(ch);
      cp_async16(kd + dst, ok ? ks : kbase, ok ? 16u : 0u);
      cp_async16(vd + dst, ok ? vs : vbase, ok ? 16u : 0u);
    }
  };

  // Start the stream before anything else.  q and the new row come from the
  // kernel that precedes this one, and rows from a.wait_pos on may still be
  // being stored by an earlier launch of this layer that is in flight, so
  // with programmatic dependent launch they are read only after pdl_wait():
  // a warp's tiles come in increasing row order, so from its first tile that
  // reaches wait_row on, it waits first.
  pdl_launch_dependents();
  // q's lines into L2 now, so that its load after the wait hits L2
  prefetch_l2(a.q + (long long)z * a.q_zstride + (long long)h0 * HD, GT * HD * 4);
  const int wait_row = min(wait_new ? new_row : INT_MAX, a.wait_pos - lo);
  bool waited = false;
#pragma unroll
  for (int i = 0; i < C::kStages - 1; ++i) {
    if (i < my_tiles) {
      const int r0 = (first + i * step) * C::kR;
      if (!waited && r0 + C::kR > wait_row) {
        pdl_wait();
        waited = true;
      }
      issue(i);
    }
    cp_async_commit();
  }
  pdl_wait();
  trace_stamp(a.trace, 1);

  // the fused append: one CTA per KV head writes the new row into the cache
  if (fused && split == 0 && hg == 0) {
    float* kw = a.kc_w + row_off + (long long)new_row * HD;
    float* vw = a.vc + row_off + (long long)new_row * HD;
    for (int e = threadIdx.x; e < HD; e += C::kThreads) {
      kw[e] = knew[e];
      vw[e] = vnew[e];
    }
  }

  // query rows of the group, scaled as the reference's fused RoPE does.
  // Wide layout: lane holds elements lane_elem(lane, e) of every row.
  // Narrow layout: lane (rq, sg) holds elements [sg*HD/8, (sg+1)*HD/8).
  constexpr int kQ = C::kNarrow ? HD / 8 : C::kEPL;
  float qr[GT][kQ];
  const float* qz = a.q + (long long)z * a.q_zstride;
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    const float* qrow = qz + (long long)(h0 + g) * HD;
    if constexpr (C::kNarrow) {
#pragma unroll
      for (int c = 0; c < C::kSegC; ++c) {
        const float4 t = *reinterpret_cast<const float4*>(qrow + (lane & 7) * (HD / 8) + 4 * c);
        qr[g][4 * c + 0] = t.x;
        qr[g][4 * c + 1] = t.y;
        qr[g][4 * c + 2] = t.z;
        qr[g][4 * c + 3] = t.w;
      }
    } else {
      float t[C::kEPL];
      load_row<HD>(qrow, t, lane);
#pragma unroll
      for (int e = 0; e < C::kEPL; ++e) qr[g][e] = t[e];
    }
#pragma unroll
    for (int e = 0; e < kQ; ++e) qr[g][e] *= a.scale;
  }
  trace_stamp(a.trace, 2);

  float my_m = -INFINITY, my_l = 0.f;
  float acc[GT][C::kEPL];
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < C::kEPL; ++e) acc[g][e] = 0.f;

  for (int i = 0; i < my_tiles; ++i) {
    if (i + C::kStages - 1 < my_tiles) issue(i + C::kStages - 1);
    cp_async_commit();
    cp_async_wait<C::kStages - 1>();
    __syncwarp();
    const float* ks = wring + (i % C::kStages) * C::kStageFloats;
    const float* vs = ks + C::kTileFloats;
    const int nvalid = min(C::kR, n_rows - (first + i * step) * C::kR);

    if constexpr (C::kNarrow) {
      // ---- score phase, 8 lanes per K row ----
      const int rq = lane >> 3, sg = lane & 7;
      float part[8];
#pragma unroll
      for (int pp = 0; pp < C::kR / 4; ++pp) {
        const float* krow = ks + (rq + 4 * pp) * HD;
#pragma unroll
        for (int g = 0; g < GT; ++g) part[pp * GT + g] = 0.f;
#pragma unroll
        for (int c = 0; c < C::kSegC; ++c) {
          const float4 kx = lds128(krow + 4 * swz<HD, true>(sg * C::kSegC + c));
#pragma unroll
          for (int g = 0; g < GT; ++g) {
            float d = part[pp * GT + g];
            d = fmaf(qr[g][4 * c + 0], kx.x, d);
            d = fmaf(qr[g][4 * c + 1], kx.y, d);
            d = fmaf(qr[g][4 * c + 2], kx.z, d);
            d = fmaf(qr[g][4 * c + 3], kx.w, d);
            part[pp * GT + g] = d;
          }
        }
      }
      // transposing reduction over the 8 lanes of a row group: lane sg ends
      // with value sg = (row pass, q head)
#pragma unroll
      for (int n = 8, off = 4; n > 1; n >>= 1, off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int k = 0; k < n / 2; ++k) {
          const float send = upper ? part[k] : part[k + n / 2];
          const float keep = upper ? part[k + n / 2] : part[k];
          part[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      const int g_mine = sg & (GT - 1);
      const int row_mine = rq + 4 * (sg / GT);
      const float s = row_mine < nvalid ? part[0] * kLog2e : -INFINITY;
      // rows of one q head differ in rq (lane bits 3, 4) and in the row pass
      float tmax = s;
#pragma unroll
      for (int off = GT; off < 32; off <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float m_new = fmaxf(my_m, tmax);  // finite: row 0 of a tile is valid
      const float p = fast_exp2(s - m_new);
      const float alpha = fast_exp2(my_m - m_new);
      float tsum = p;
#pragma unroll
      for (int off = GT; off < 32; off <<= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, off);
      my_l = my_l * alpha + tsum;
      my_m = m_new;
      // every lane needs every (row, head) weight: publish through shared memory
      float* sp = s_p[warp];
      sp[row_mine * GT + g_mine] = p;
      if (row_mine == 0) sp[C::kR * GT + g_mine] = alpha;
      __syncwarp();
      float ag[GT];
#pragma unroll
      for (int g = 0; g < GT; g += 4) {
        const float4 t = lds128(sp + C::kR * GT + g);
        ag[g] = t.x;
        if (g + 1 < GT) ag[g + 1] = t.y;
        if (g + 2 < GT) ag[g + 2] = t.z;
        if (g + 3 < GT) ag[g + 3] = t.w;
      }
#pragma unroll
      for (int g = 0; g < GT; ++g)
#pragma unroll
        for (int e = 0; e < C::kEPL; ++e) acc[g][e] *= ag[g];
      // ---- value phase, 32 lanes per V row ----
#pragma unroll
      for (int r = 0; r < C::kR; ++r) {
        float vx[C::kEPL];
        if constexpr (HD == 128) {
          const float4 t = lds128(vs + r * HD + 4 * swz<HD, true>(lane));
          vx[0] = t.x;
          vx[1] = t.y;
          vx[2] = t.z;
          vx[3] = t.w;
        } else {
          const float2 t =
              *reinterpret_cast<const float2*>(vs + r * HD + 4 * swz<HD, true>(lane >> 1) + 2 * (lane & 1));
          vx[0] = t.x;
          vx[1] = t.y;
        }
        float pr[GT];
#pragma unroll
        for (int g = 0; g < GT; g += 4) {
          const float4 t = lds128(sp + r * GT + g);
          pr[g] = t.x;
          if (g + 1 < GT) pr[g + 1] = t.y;
          if (g + 2 < GT) pr[g + 2] = t.z;
          if (g + 3 < GT) pr[g + 3] = t.w;
        }
#pragma unroll
        for (int g = 0; g < GT; ++g)
#pragma unroll
          for (int e = 0; e < C::kEPL; ++e) acc[g][e] = fmaf(pr[g], vx[e], acc[g][e]);
      }
    } else {
      float part[C::kNV];
  #pragma unroll
      for (int r = 0; r < C::kR; ++r) {
        float kx[C::kEPL];
        load_row<HD>(ks + r * HD, kx, lane);
  #pragma unroll
        for (int g = 0; g < GT; ++g) {
          float d = 0.f;
  #pragma unroll
          for (int e = 0; e < C::kEPL; ++e) d = fmaf(qr[g][e], kx[e], d);
          part[r * GT + g] = d;
        }
      }
      transpose_reduce<C::kNV>(part, lane);
      const int j = lane >> C::kSH;
      const float s = (j / GT < nvalid) ? part[0] * kLog2e : -INFINITY;
      float tmax = s;
  #pragma unroll
      for (int off = GT << C::kSH; off < 32; off <<= 1)
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      const float m_new = fmaxf(my_m, tmax);  // finite: row 0 of a tile is valid
      const float p = fast_exp2(s - m_new);
      const float alpha = fast_exp2(my_m - m_new);
      float tsum = p;
  #pragma unroll
      for (int off = GT << C::kSH; off < 32; off <<= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, off);
      my_l = my_l * alpha + tsum;
      my_m = m_new;
  #pragma unroll
      for (int g = 0; g < GT; ++g) {
        const float ag = __shfl_sync(0xffffffffu, alpha, g << C::kSH);
  #pragma unroll
        for (int e = 0; e < C::kEPL; ++e) acc[g][e] *= ag;
      }
  #pragma unroll
      for (int r = 0; r < C::kR; ++r) {
        float vx[C::kEPL];  // rows past the range were zero-filled
        load_row<HD>(vs + r * HD, vx, lane);
  #pragma unroll
        for (int g = 0; g < GT; ++g) {
          const float pr = __shfl_sync(0xffffffffu, p, (r * GT + g) << C::kSH);
  #pragma unroll
          for (int e = 0; e < C::kEPL; ++e) acc[g][e] = fmaf(pr, vx[e], acc[g][e]);
        }
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
  }
  cp_async_wait<0>();
  trace_stamp(a.trace, 3);
  __syncthreads();
  // the lane holding head g's running (max, sum): g (narrow) or g << kSH (wide)
  if constexpr (C::kNarrow) {
    if (lane < GT) {
      s_m[warp][lane] = my_m;
      s_l[warp][lane] = my_l;
    }
  } else if ((lane & ((1 << C::kSH) - 1)) == 0 && (lane >> C::kSH) < GT) {
    s_m[warp][lane >> C::kSH] = my_m;
    s_l[warp][lane >> C::kSH] = my_l;
  }
  decode_finish<HD, GT, C::kWarps, C::kThreads>(a, ms, ring, acc, warp, lane, split, unit, z, h0);
}

template <int HD, int GT>
__global__ void __launch_bounds__(DecodeCfg<HD, GT>::kThreads, DecodeCfg<HD, GT>::kCtasPerSm)
    decode_f32_kernel(const DecodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  decode_f32_cta<HD, GT>(a, smem_raw);
}

// Token K/V rows -> head-major cache rows.  k, v: [n_tok][src_stride] with
// KV head h at offset h*HD; grid (n_tok, kvh_count), HD/4 threads.  The next
// kernel launches when this grid completes (it may read these rows at once).
static __global__ void kv_append_kernel(float* __restrict__ kc, float* __restrict__ vc, long long head_stride,
                                 int hd, const float* __restrict__ k, const float* __restrict__ v,
                                 long long src_stride, int kv_head_begin, int row0) {
  const int tok = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  pdl_wait();  // the rows come from the kernel before this one
  const long long src = (long long)tok * src_stride + (long long)(kv_head_begin + h) * hd + 4 * t;
  const long long dst = (long long)h * head_stride + (long long)(row0 + tok) * hd + 4 * t;
  *reinterpret_cast<float4*>(kc + dst) = *reinterpret_cast<const float4*>(k + src);
  *reinterpret_cast<float4*>(vc + dst) = *reinterpret_cast<const float4*>(v + src);
}

// Log-sum-exp merge of n_parts partial triples.  parts_o: [n_parts][rows][hd],
// parts_ml: [n_parts][rows][2]; one CTA per output row.
static __global__ void lse_merge_kernel(int n_parts, int rows, int row_begin, int hd, const float* __restrict__ parts_o,
                                 const float* __restrict__ parts_ml, float* __restrict__ out) {
  const int row = row_begin + blockIdx.x;
  float M = -INFINITY;
  for (int p = 0; p < n_parts; ++p) M = fmaxf(M, parts_ml[((long long)p * rows + row) * 2]);
  float L = 0.f;
  for (int p = 0; p < n_parts; ++p) {
    const float m = parts_ml[((long long)p * rows + row) * 2];
    if (m != -INFINITY) L = fmaf(parts_ml[((long long)p * rows + row) * 2 + 1], fast_exp2(m - M), L);
  }
  for (int e = threadIdx.x; e < hd; e += blockDim.x) {
    float O = 0.f;
    for (int p = 0; p < n_parts; ++p) {
      const float m = parts_ml[((long long)p * rows + row) * 2];
      if (m == -INFINITY) continue;
      const float w = parts_ml[((long long)p * rows + row) * 2 + 1] * fast_exp2(m - M);
      O = fmaf(parts_o[((long long)p * rows + row) * hd + e], w, O);
    }
    out[(long long)row * hd + e] = L > 0.f ? O / L : 0.f;
  }
}

}  // namespace l3p
