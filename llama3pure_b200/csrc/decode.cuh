// decode.cuh -- split-K flash-decoding over an fp32 KV cache (sm_100a).
//
// Replaces the reference's per-layer decode attention loop
// (llama3pure-c-engine.c:3310-3359): scores q.K^T for every cached position
// of the window, softmax, and the softmax-weighted sum of V rows, for all
// q heads of a GQA group (c:3333-3357).  The same kernel serves the
// token-by-token causal prefill (c:3582-3612) with one grid slice per token.
//
// Work decomposition
//   grid.x  split of the attended position range (split-K)
//   grid.y  (owned KV head, group of GT q heads of that KV head)
//   grid.z  layer (multi-layer decode) or token (prefill)
// One CTA of 8 warps streams a contiguous chunk of K and V rows of one KV head
// exactly once and serves all GT q heads of the group with it (the reference
// re-reads every V row once per q head, c:3352-3357).  Each warp owns a ring
// of kStages shared-memory stages; lane 0 fills a stage with two 1-D bulk
// async copies (R rows of K, R rows of V, cp.async.bulk + mbarrier), so every
// warp keeps kStages-1 tiles in flight while it computes on one.
//
// Per tile a warp forms R*GT partial dot products per lane, reduces them with
// a transposing butterfly (31 shuffles for 32 values, leaving lane j the full
// score of value j), and runs the online softmax in base 2: running max m and
// running sum l per q head, accumulator rescaled by 2^(m_old - m_new).  Warps
// of a CTA are merged in shared memory; splits of a position range are merged
// by the last CTA to finish (atomic ticket on a per-unit counter in scratch
// memory), so one launch produces the final normalised output.
//
// Differences from the reference's arithmetic, all inside the 1e-4 contract:
//   * summation order (lane-parallel dot products, blocked softmax sums);
//   * exp via ex2.approx on log2(e)-scaled scores instead of libm expf;
//   * the reference skips V rows whose final weight is below 1e-8 in
//     magnitude (c:1602).  A one-pass online softmax does not know the final
//     weight when it reads V, so every row contributes; the difference is at
//     most (number of such rows) * 1e-8 * max|v| per output element.
#pragma once
#include "ptx.cuh"

namespace l3p {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxSplits = 160;  // splits of one position range per launch

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct DecodeArgs {
  const float* kc;         // K cache, all layers: [n_layers][kvh_count][cap][HD]
  const float* vc;         // V cache, same layout
  long long layer_stride;  // kvh_count * cap * HD
  long long head_stride;   // cap * HD
  const float* q;          // row of absolute q head h in slice z: q + z*q_zstride + h*HD
  long long q_zstride;
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
  int nsplit, chunk;       // splits per unit and positions per split
  int is_gemma3, swa_window, swa_pattern;
  int partial;
};

template <int HD, int GT>
struct DecodeCfg {
  static_assert(HD == 64 || HD == 128 || HD == 256, "head_dim");
  static_assert(GT == 1 || GT == 2 || GT == 4 || GT == 8, "group");
  static constexpr int kWarps = 8;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kR = (GT >= 8 || HD >= 256) ? 4 : 8;  // rows per tile
  static constexpr int kNV = kR * GT;           // partial sums per lane per tile
  static constexpr int kLogNV = (kNV == 32) ? 5 : (kNV == 16) ? 4 : (kNV == 8) ? 3 : 2;
  static constexpr int kSH = 5 - kLogNV;        // lane j holds value (j >> kSH)
  static constexpr int kEPL = HD / 32;          // elements of a row per lane
  static constexpr int kTileFloats = kR * HD;
  static constexpr int kStageFloats = 2 * kTileFloats;  // K tile + V tile
  static constexpr int kStageBytes = kStageFloats * 4;
  static constexpr int kStagesRaw = (24 * 1024) / kStageBytes;
  static constexpr int kStages = kStagesRaw < 2 ? 2 : (kStagesRaw > 6 ? 6 : kStagesRaw);
  static constexpr int kRingBytes = kWarps * kStages * kStageBytes;
  static constexpr int kSmemBytes = kRingBytes + kWarps * kStages * 8;
  static_assert(kWarps * GT * HD * 4 <= kRingBytes, "merge buffer fits in the ring");
  static_assert(kSmemBytes <= 200 * 1024, "ring fits one CTA per SM");
};

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

template <int HD, int GT>
__global__ void __launch_bounds__(DecodeCfg<HD, GT>::kThreads, 1)
    decode_f32_kernel(const DecodeArgs a) {
  using C = DecodeCfg<HD, GT>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + C::kRingBytes);
  __shared__ float s_m[C::kWarps][GT];
  __shared__ float s_l[C::kWarps][GT];
  __shared__ float s_w[kMaxSplits][GT];  // per-split merge weights
  __shared__ float s_L[GT];
  __shared__ int s_last;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int split = blockIdx.x;
  const int kvh_local = blockIdx.y / a.n_hg;
  const int hg = blockIdx.y - kvh_local * a.n_hg;
  const int z = blockIdx.z;
  const int units_per_z = gridDim.y;
  const int unit = z * units_per_z + blockIdx.y;
  const int layer = a.layer0 + z * a.layer_step;
  const int pos = a.pos0 + z * a.pos_step;

  const int lo = max(swa_start(a, layer, pos), a.seq_begin);
  const int hi = min(pos + 1, a.seq_begin + a.cap);
  const int c0 = lo + split * a.chunk;
  const int n_rows = max(0, min(hi, c0 + a.chunk) - c0);
  const int n_tiles = (n_rows + C::kR - 1) / C::kR;
  const int h0 = (a.kv_head_begin + kvh_local) * a.G + hg * GT;

  const long long row_off = (long long)layer * a.layer_stride + (long long)kvh_local * a.head_stride +
                            (long long)(c0 - a.seq_begin) * HD;
  const float* kbase = a.kc + row_off;
  const float* vbase = a.vc + row_off;

  if (threadIdx.x < C::kWarps * C::kStages) mbar_init(&bars[threadIdx.x], 1);
  fence_mbar_init();
  __syncthreads();

  // query rows of the group, scaled as the reference's fused RoPE does
  float qr[GT][C::kEPL];
  const float* qz = a.q + (long long)z * a.q_zstride;
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    load_row<HD>(qz + (long long)(h0 + g) * HD, qr[g], lane);
#pragma unroll
    for (int e = 0; e < C::kEPL; ++e) qr[g][e] *= a.scale;
  }

  float* wring = ring + warp * C::kStages * C::kStageFloats;
  uint64_t* wbar = bars + warp * C::kStages;
  const int my_tiles = n_tiles > warp ? (n_tiles - warp + C::kWarps - 1) / C::kWarps : 0;
  uint64_t policy = 0;
  if (lane == 0) {
    policy = l2_evict_first_policy();
    const int pre = my_tiles < C::kStages ? my_tiles : C::kStages;
    for (int i = 0; i < pre; ++i) {
      const int tile = warp + i * C::kWarps;
      const int rows = min(C::kR, n_rows - tile * C::kR);
      const uint32_t bytes = (uint32_t)rows * HD * 4u;
      float* st = wring + i * C::kStageFloats;
      mbar_arrive_expect_tx(&wbar[i], 2u * bytes);
      bulk_g2s(st, kbase + (long long)tile * C::kR * HD, bytes, &wbar[i], policy);
      bulk_g2s(st + C::kTileFloats, vbase + (long long)tile * C::kR * HD, bytes, &wbar[i], policy);
    }
  }

  float my_m = -INFINITY, my_l = 0.f;
  float acc[GT][C::kEPL];
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < C::kEPL; ++e) acc[g][e] = 0.f;

  int consumed = 0;
  bool timed_out = false;
  for (int i = 0; i < my_tiles; ++i) {
    const int st = i % C::kStages;
    const bool ready = mbar_wait_bounded(&wbar[st], (uint32_t)((i / C::kStages) & 1), a.err);
    if (!__all_sync(0xffffffffu, ready)) {
      timed_out = true;
      break;
    }
    const float* ks = wring + st * C::kStageFloats;
    const float* vs = ks + C::kTileFloats;
    const int tile = warp + i * C::kWarps;
    const int nvalid = min(C::kR, n_rows - tile * C::kR);

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
      float vx[C::kEPL];
      load_row<HD>(vs + r * HD, vx, lane);
      if (r >= nvalid) {
        // rows past the chunk's end were not copied; their stage memory is stale
#pragma unroll
        for (int e = 0; e < C::kEPL; ++e) vx[e] = 0.f;
      }
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        const float pr = __shfl_sync(0xffffffffu, p, (r * GT + g) << C::kSH);
#pragma unroll
        for (int e = 0; e < C::kEPL; ++e) acc[g][e] = fmaf(pr, vx[e], acc[g][e]);
      }
    }
    __syncwarp();
    consumed = i + 1;
    if (lane == 0 && i + C::kStages < my_tiles) {
      const int ni = i + C::kStages;
      const int ntile = warp + ni * C::kWarps;
      const int rows = min(C::kR, n_rows - ntile * C::kR);
      const uint32_t bytes = (uint32_t)rows * HD * 4u;
      float* stp = wring + st * C::kStageFloats;
      mbar_arrive_expect_tx(&wbar[st], 2u * bytes);
      bulk_g2s(stp, kbase + (long long)ntile * C::kR * HD, bytes, &wbar[st], policy);
      bulk_g2s(stp + C::kTileFloats, vbase + (long long)ntile * C::kR * HD, bytes, &wbar[st], policy);
    }
  }
  if (timed_out && lane == 0) {
    // drain the copies still in flight (bounded) before the ring is reused
    const int issued = min(my_tiles, consumed + C::kStages);
    for (int i = consumed; i < issued; ++i)
      mbar_wait_bounded(&wbar[i % C::kStages], (uint32_t)((i / C::kStages) & 1), a.err);
  }
  __syncthreads();

  // ---- merge the warps of this CTA (the ring becomes the merge buffer) ----
  float* wacc = ring;  // [kWarps][GT][HD]
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < C::kEPL; ++e) wacc[(warp * GT + g) * HD + lane_elem<HD>(lane, e)] = acc[g][e];
  if ((lane & ((1 << C::kSH) - 1)) == 0 && (lane >> C::kSH) < GT) {
    s_m[warp][lane >> C::kSH] = my_m;
    s_l[warp][lane >> C::kSH] = my_l;
  }
  __syncthreads();

  const bool single = a.nsplit == 1;
  for (int idx = threadIdx.x; idx < GT * HD; idx += C::kThreads) {
    const int g = idx / HD, e = idx - g * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::kWarps; ++w) M = fmaxf(M, s_m[w][g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < C::kWarps; ++w) {
        const float f = fast_exp2(s_m[w][g] - M);
        L = fmaf(s_l[w][g], f, L);
        O = fmaf(wacc[(w * GT + g) * HD + e], f, O);
      }
    }
    const int h = h0 + g;
    if (single) {
      if (!a.partial) {
        a.out[(long long)z * a.q_zstride + (long long)h * HD + e] = O / L;
      } else {
        a.part_o[(long long)z * a.q_zstride + (long long)h * HD + e] = L > 0.f ? O / L : 0.f;
        if (e == 0) {
          a.part_ml[(long long)z * a.ml_zstride + 2 * h] = M;
          a.part_ml[(long long)z * a.ml_zstride + 2 * h + 1] = L;
        }
      }
    } else {
      const long long slot = (long long)unit * a.nsplit + split;
      a.ws_o[(slot * GT + g) * HD + e] = O;
      if (e == 0) {
        a.ws_ml[(slot * GT + g) * 2] = M;
        a.ws_ml[(slot * GT + g) * 2 + 1] = L;
      }
    }
  }
  if (single) return;

  // ---- the last CTA of this unit merges all splits ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&a.counters[unit], 1u) == (unsigned)(a.nsplit - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  const long long slot0 = (long long)unit * a.nsplit;
  if (threadIdx.x < GT) {
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < a.nsplit; ++sp) M = fmaxf(M, __ldcg(&a.ws_ml[((slot0 + sp) * GT + g) * 2]));
    float L = 0.f;
    for (int sp = 0; sp < a.nsplit; ++sp) {
      const float m = __ldcg(&a.ws_ml[((slot0 + sp) * GT + g) * 2]);
      const float l = __ldcg(&a.ws_ml[((slot0 + sp) * GT + g) * 2 + 1]);
      const float f = (M == -INFINITY) ? 0.f : fast_exp2(m - M);
      s_w[sp][g] = f;
      L = fmaf(l, f, L);
    }
    s_L[g] = L;
    if (a.partial) {
      const int h = h0 + g;
      a.part_ml[(long long)z * a.ml_zstride + 2 * h] = M;
      a.part_ml[(long long)z * a.ml_zstride + 2 * h + 1] = L;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < GT * HD; idx += C::kThreads) {
    const int g = idx / HD, e = idx - g * HD;
    float O = 0.f;
    for (int sp = 0; sp < a.nsplit; ++sp) O = fmaf(__ldcg(&a.ws_o[((slot0 + sp) * GT + g) * HD + e]), s_w[sp][g], O);
    const float L = s_L[g];
    const long long o = (long long)z * a.q_zstride + (long long)(h0 + g) * HD + e;
    if (!a.partial)
      a.out[o] = O / L;
    else
      a.part_o[o] = L > 0.f ? O / L : 0.f;
  }
  if (threadIdx.x == 0) a.counters[unit] = 0u;  // ticket ready for the next launch
}

// Token K/V rows -> head-major cache rows.  k, v: [n_tok][src_stride] with
// KV head h at offset h*HD; grid (n_tok, kvh_count), HD/4 threads.
__global__ void kv_append_kernel(float* __restrict__ kc, float* __restrict__ vc, long long head_stride,
                                 int hd, const float* __restrict__ k, const float* __restrict__ v,
                                 long long src_stride, int kv_head_begin, int row0) {
  const int tok = blockIdx.x, h = blockIdx.y, t = threadIdx.x;
  const long long src = (long long)tok * src_stride + (long long)(kv_head_begin + h) * hd + 4 * t;
  const long long dst = (long long)h * head_stride + (long long)(row0 + tok) * hd + 4 * t;
  *reinterpret_cast<float4*>(kc + dst) = *reinterpret_cast<const float4*>(k + src);
  *reinterpret_cast<float4*>(vc + dst) = *reinterpret_cast<const float4*>(v + src);
}

// Log-sum-exp merge of n_parts partial triples.  parts_o: [n_parts][rows][hd],
// parts_ml: [n_parts][rows][2]; one CTA per output row.
__global__ void lse_merge_kernel(int n_parts, int rows, int row_begin, int hd, const float* __restrict__ parts_o,
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
