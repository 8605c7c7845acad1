// decode_q8.cuh -- the reference's Q8_0 KV cache on B200 (sm_100a): block
// quantisation of K/V rows and q, and split-K flash decoding over int8 rows.
//
// Q8_0 (the format the reference ships, c:120-123): every 32 consecutive
// values of a row form a block with one scale d = amax/127, stored as fp16
// converted by TRUNCATION (fp32_to_fp16, c:585-599), and 32 int8 values
// q = round-half-away(x * 127/amax) clamped to [-128, 127]
// (quantize_to_q8_0_cache, c:1535-1570).  The quantiser below performs the
// same IEEE operations in the same order, so its bytes equal the reference's.
//
// Device layout (per layer, owned KV head, owned position): the int8 values
// of a row in one array ([cap][head_dim] bytes, 16-byte aligned rows) and the
// row's fp16 block scales in another ([cap][head_dim/32]); the reference
// interleaves them as 34-byte blocks (c:365-372), which no 16-byte copy can
// address.  q8_blocks_kernel / q8_unblock_kernel convert between the two.
//
// Decode arithmetic, as the reference's q8 path (c:3310-3357):
//   q is scaled, then quantised to Q8_0 like a cache row (c:3310-3312);
//   score(t) = sum over blocks b of (d_q[b] * d_k[t][b]) * int32(q8 . k8)
//              (dot_q8_0_q8_0_cache, c:1574-1597; int8 products summed with
//              dp4a, exact);
//   out += int8(v) * (d_v[t][b] * w_t) (accum_q8_0_cache, c:1600-1622).
// The softmax is the online base-2 form of decode.cuh (same differences from
// the reference: summation order of the block terms, ex2.approx, no skip of
// weights below 1e-8), and the merge stages are decode.cuh's decode_finish.
#pragma once
#include <cuda_fp16.h>

#include "decode.cuh"

namespace l3p {

// fp32 -> fp16 bits by truncation of the mantissa: values below half's
// subnormal range become signed zero, values at or above 2^16 (and nan)
// signed inf (fp32_to_fp16, c:585-599).
__device__ __forceinline__ uint16_t fp32_to_fp16_trunc(float f) {
  const uint32_t b = __float_as_uint(f);
  const uint16_t sign = (uint16_t)((b >> 16) & 0x8000u);
  const int e = (int)((b >> 23) & 0xff) - 112;  // rebias 127 -> 15
  const uint32_t sig = (b & 0x7fffffu) | 0x800000u;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e > 0) return (uint16_t)(sign | (uint16_t)(e << 10) | (uint16_t)((b >> 13) & 0x3ffu));
  if (e < -10) return sign;
  return (uint16_t)(sign | (uint16_t)(sig >> (14 - e)));
}

// fp16 bits -> fp32: exact for every finite half (the reference's fp16_table,
// c:545-582, holds the same values).
__device__ __forceinline__ float fp16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Quantise the N consecutive values x[] a lane holds, where the lanes of one
// 32-value block are the aligned group of 32/N lanes containing this one.
// Writes the int8 values into packed words and returns the block's fp16 scale
// bits.  Every lane of the warp must call it.
template <int N>
__device__ __forceinline__ uint16_t q8_quantize_lanes(const float (&x)[N], uint32_t (&w)[(N + 3) / 4]) {
  static_assert(N == 2 || N == 4 || N == 8 || N == 16 || N == 32, "values per lane");
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
  for (int off = 1; off < 32 / N; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float d = amax / 127.0f;
  const float inv = d > 0.0f ? 127.0f / amax : 0.0f;
#pragma unroll
  for (int i = 0; i < (N + 3) / 4; ++i) w[i] = 0u;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    int q = (int)roundf(x[i] * inv);
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    w[i / 4] |= ((uint32_t)q & 0xffu) << (8 * (i % 4));
  }
  return fp32_to_fp16_trunc(d);
}

// One row of HD values quantised by a warp: lane holds values
// [lane*HD/32, (lane+1)*HD/32) of src; returns the scale of the lane's block.
template <int HD>
__device__ __forceinline__ uint16_t q8_quantize_row(const float* src, int lane, uint32_t (&w)[(HD / 32 + 3) / 4]) {
  constexpr int N = HD / 32;
  float x[N];
#pragma unroll
  for (int i = 0; i < N; ++i) x[i] = src[lane * N + i];
  return q8_quantize_lanes<N>(x, w);
}

// Store a row quantised by q8_quantize_row: its int8 values at dst8 (the row's
// first byte) and its block scales at dsc (the row's first scale); global or
// shared memory.
template <int HD>
__device__ __forceinline__ void q8_store_row(int8_t* dst8, uint16_t* dsc, int lane, const uint32_t (&w)[(HD / 32 + 3) / 4],
                                             uint16_t d) {
  constexpr int N = HD / 32;
  if constexpr (N == 2) {
    *reinterpret_cast<uint16_t*>(dst8 + lane * N) = (uint16_t)w[0];
  } else {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) reinterpret_cast<uint32_t*>(dst8 + lane * N)[i] = w[i];
  }
  if ((lane * N) % 32 == 0) dsc[lane * N / 32] = d;
}

// Token K/V rows -> Q8_0 cache rows: one warp per (token, owned KV head) row,
// HD/32 values per lane.  k, v: [n_tok][src_stride] with KV head h at h*HD.
template <int HD>
__global__ void kv_append_q8_kernel(int8_t* __restrict__ k8, int8_t* __restrict__ v8, uint16_t* __restrict__ ksc,
                                    uint16_t* __restrict__ vsc, long long head_stride, const float* __restrict__ k,
                                    const float* __restrict__ v, long long src_stride, int kv_head_begin, int row0) {
  const int tok = blockIdx.x, h = blockIdx.y, lane = threadIdx.x;
  pdl_wait();  // the rows come from the kernel before this one
  const long long src = (long long)tok * src_stride + (long long)(kv_head_begin + h) * HD;
  const long long row = (long long)h * head_stride / HD + row0 + tok;  // row index in the cache
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    uint32_t w[(HD / 32 + 3) / 4];
    const uint16_t d = q8_quantize_row<HD>((which ? v : k) + src, lane, w);
    q8_store_row<HD>((which ? v8 : k8) + row * HD, (which ? vsc : ksc) + row * (HD / 32), lane, w, d);
  }
}

// Cache rows -> the reference's 34-byte blocks (fp16 scale little-endian, then
// 32 int8), [rows][HD/32 * 34] bytes; one thread per block.
static __global__ void q8_blocks_kernel(const int8_t* __restrict__ d8, const uint16_t* __restrict__ dsc, long long n_blocks,
                                 uint8_t* __restrict__ out) {
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks; b += (long long)gridDim.x * blockDim.x) {
    uint8_t* o = out + b * 34;
    const uint16_t d = dsc[b];
    o[0] = (uint8_t)(d & 0xff);
    o[1] = (uint8_t)(d >> 8);
    for (int j = 0; j < 32; ++j) o[2 + j] = (uint8_t)d8[b * 32 + j];
  }
}

// The reference's 34-byte blocks -> cache rows (inverse of q8_blocks_kernel).
static __global__ void q8_unblock_kernel(const uint8_t* __restrict__ in, long long n_blocks, int8_t* __restrict__ d8,
                                  uint16_t* __restrict__ dsc) {
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks; b += (long long)gridDim.x * blockDim.x) {
    const uint8_t* s = in + b * 34;
    dsc[b] = (uint16_t)(s[0] | (s[1] << 8));
    for (int j = 0; j < 32; ++j) d8[b * 32 + j] = (int8_t)s[2 + j];
  }
}

// Cache rows -> fp32 values d * int8 (exact), [blocks * 32]; one thread per block.
static __global__ void q8_dequant_kernel(const int8_t* __restrict__ d8, const uint16_t* __restrict__ dsc, long long n_blocks,
                                  float* __restrict__ out) {
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < n_blocks; b += (long long)gridDim.x * blockDim.x) {
    const float d = fp16_to_f32(dsc[b]);
    for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)d8[b * 32 + j] * d;
  }
}

#ifndef L3P_Q8_WARPS
#define L3P_Q8_WARPS 8  // warps per CTA
#endif
#ifndef L3P_Q8_ROWS
#define L3P_Q8_ROWS 16  // rows per tile for head_dim <= 128 (see kR)
#endif
#ifndef L3P_Q8_RING_KB
#define L3P_Q8_RING_KB 192  // shared-memory ring per CTA
#endif
#ifndef L3P_Q8_CTAS_PER_SM
#define L3P_Q8_CTAS_PER_SM 1  // resident CTAs per SM the launch bounds ask for
#endif

template <int HD, int GT>
struct DecodeQ8Cfg {
  static_assert(HD == 64 || HD == 128 || HD == 256, "head_dim");
  static_assert(GT == 1 || GT == 2 || GT == 4 || GT == 8, "group");
  static constexpr int kWarps = L3P_Q8_WARPS;
  static constexpr int kThreads = kWarps * 32;
  // rows per tile (4 per pass, 8 lanes per row): halved at head_dim 256,
  // doubled at head_dim 128 for groups of <= 4 q heads (the 8B shapes: 32-row
  // tiles measured 0.5 us faster per 8K layer than 16-row ones)
  static constexpr int kR = HD >= 256 ? L3P_Q8_ROWS / 2 : (HD == 128 && GT <= 4 ? 2 * L3P_Q8_ROWS : L3P_Q8_ROWS);
  static constexpr int kScB = HD / 16;           // scale bytes per row
  static constexpr int kTileKB = kR * HD;        // int8 bytes of a K (or V) tile
  static constexpr int kTileSB = kR * kScB;      // scale bytes of a K (or V) tile
  static constexpr int kStageBytes = 2 * (kTileKB + kTileSB);
  static constexpr int kStagesRaw = (L3P_Q8_RING_KB * 1024 / kWarps) / kStageBytes;
  static constexpr int kStages = kStagesRaw < 2 ? 2 : (kStagesRaw > 8 ? 8 : kStagesRaw);
  // the ring doubles as the warps' merge buffer: at least (kWarps + 1) * GT * HD floats
  static constexpr int kRingBytes = kWarps * kStages * kStageBytes > (kWarps + 1) * GT * HD * 4
                                        ? kWarps * kStages * kStageBytes
                                        : (kWarps + 1) * GT * HD * 4;
  static constexpr int kSmemBytes = kRingBytes;
  static constexpr int kEPL = HD / 32;  // values of a V row per lane
  static constexpr int kKB = HD / 8;    // K bytes per lane in the score phase (8 lanes per row)
  static constexpr int kKW = kKB / 4;   // ... as 32-bit words
  static constexpr int kLanesPerBlock = 32 / kKB;  // lanes sharing one 32-value block in the score phase
  static constexpr int kCtasPerSm = L3P_Q8_CTAS_PER_SM;
  static_assert(kTileKB % 512 == 0, "K tile copies cover the warp");
  static_assert(kR % 4 == 0 && kR <= 32, "4-row passes; one lane per row copies the scales");
  static_assert(kStageBytes % 16 == 0, "stage alignment");
  static_assert((kWarps + 1) * GT * HD * 4 <= kRingBytes, "merge buffer fits in the ring");
  static_assert(kMaxSplits * GT * 3 * 4 <= kRingBytes, "split merge buffer fits in the ring");
};

template <int BYTES>
__device__ __forceinline__ void cp_async_small(void* smem_dst, const void* gmem_src, uint32_t src_bytes) {
  static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16, "cp.async size");
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src), "n"(BYTES),
               "r"(src_bytes)
               : "memory");
}

template <int HD, int GT>
__global__ void __launch_bounds__(DecodeQ8Cfg<HD, GT>::kThreads, DecodeQ8Cfg<HD, GT>::kCtasPerSm)
    decode_q8_kernel(const DecodeArgs a) {
  using C = DecodeQ8Cfg<HD, GT>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float* ring = reinterpret_cast<float*>(smem_raw);
  __shared__ DecodeMergeSmem<GT, C::kWarps> ms;
  // per row of the current tile, block of the row and q head: softmax weight
  // times the V block's scale, the factor accumulator += int8 v * factor uses
  constexpr int kNB = HD / 32;
  __shared__ __align__(16) float s_w[C::kWarps][C::kR][kNB][GT];

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

  const long long row0 = (long long)layer * (a.layer_stride / HD) + (long long)kvh_local * (a.head_stride / HD) +
                         (lo - a.seq_begin);  // cache row of position lo
  const int8_t* kbase = a.k8 + row0 * HD;
  const int8_t* vbase = a.v8 + row0 * HD;
  const uint16_t* ksbase = a.ksc + row0 * (HD / 32);
  const uint16_t* vsbase = a.vsc + row0 * (HD / 32);

  const int first = split + a.nsplit * warp;
  const int step = a.nsplit * C::kWarps;
  const int my_tiles = n_tiles > first ? (n_tiles - first + step - 1) / step : 0;
  unsigned char* wring = smem_raw + warp * C::kStages * C::kStageBytes;

  // Fused append (k_new set): the warp whose tile holds the new row quantises
  // the token's K and V rows itself (the bytes kv_append_q8_kernel writes,
  // c:3299-3312) and attends to them from registers; in the units of q-head
  // group 0 it also stores them into the cache.
  const bool fused = a.k_new != nullptr && pos >= lo && pos < hi;
  const int new_row = pos - lo;
  const int new_tile = new_row / C::kR;
  const bool own_new = fused && new_tile >= first && (new_tile - first) % step == 0;  // warp-uniform
  const int new_i = own_new ? (new_tile - first) / step : -1;

  // stage: [K int8 tile][V int8 tile][K scales][V scales]
  auto issue = [&](int i) {
    const int t = first + i * step;
    const int r0 = t * C::kR;
    unsigned char* st = wring + (i % C::kStages) * C::kStageBytes;
#pragma unroll
    for (int c = 0; c < C::kTileKB / 512; ++c) {
      const int off = (c * 32 + lane) * 16;  // byte offset inside the tile
      const bool ok = r0 + off / HD < n_rows;
      cp_async16(st + off, ok ? kbase + (long long)r0 * HD + off : kbase, ok ? 16u : 0u);
      cp_async16(st + C::kTileKB + off, ok ? vbase + (long long)r0 * HD + off : vbase, ok ? 16u : 0u);
    }
    if (lane < C::kR) {
      const bool ok = r0 + lane < n_rows;
      const long long so = (long long)(r0 + lane) * (HD / 32);
      cp_async_small<C::kScB>(st + 2 * C::kTileKB + lane * C::kScB, ok ? ksbase + so : ksbase, ok ? C::kScB : 0u);
      cp_async_small<C::kScB>(st + 2 * C::kTileKB + C::kTileSB + lane * C::kScB, ok ? vsbase + so : vsbase,
                              ok ? C::kScB : 0u);
    }
  };

  // q of the group, scaled (c:3264-3265 / c:3288-3289) and quantised to Q8_0
  // (c:3310-3312) once per CTA by warp 0 into shared memory.  Warp 0 loads q
  // before it issues any copy: behind the CTA's cache copies the small q loads
  // would wait for HBM.  The q rows h0..h0+GT-1 are contiguous.
  constexpr int kQV = GT * HD;                      // q values of the group
  constexpr int kQN = kQV >= 512 ? 16 : kQV / 32;   // values per lane and pass
  __shared__ __align__(16) uint32_t s_q8[kQV / 4];  // int8 q, packed
  __shared__ float s_dq[kQV / 32];                  // block scales
  pdl_launch_dependents();
  prefetch_l2(a.q + (long long)z * a.q_zstride + (long long)h0 * HD, kQV * 4);  // q's lines into L2 before the wait
  if (warp == 0) {
    pdl_wait();
    const float* qg = a.q + (long long)z * a.q_zstride + (long long)h0 * HD;
#pragma unroll
    for (int p = 0; p < kQV / (32 * kQN); ++p) {
      const int base = p * 32 * kQN + lane * kQN;
      float x[kQN];
#pragma unroll
      for (int i = 0; i < kQN; i += 2) {
        const float2 t = *reinterpret_cast<const float2*>(qg + base + i);
        x[i] = t.x * a.scale;
        x[i + 1] = t.y * a.scale;
      }
      uint32_t w[(kQN + 3) / 4];
      const uint16_t d = q8_quantize_lanes<kQN>(x, w);
      if constexpr (kQN == 2) {
        reinterpret_cast<uint16_t*>(s_q8)[base / 2] = (uint16_t)w[0];
      } else {
#pragma unroll
        for (int i = 0; i < kQN / 4; ++i) s_q8[base / 4 + i] = w[i];
      }
      if (base % 32 == 0) s_dq[base / 32] = fp16_to_f32(d);
    }
  }
  // cached rows [lo, pos) come from earlier launches (those from a.wait_pos
  // on are copied after the wait, as in decode_f32_kernel); the row of pos,
  // when fused, replaces its stale copy in the stage after the copy lands
  const int wait_row = a.wait_pos - lo;
  bool waited = warp == 0;
#pragma unroll
  for (int i = 0; i < C::kStages - 1; ++i) {
    if (i < my_tiles) {
      if (!waited && (first + i * step) * C::kR + C::kR > wait_row) {
        pdl_wait();
        waited = true;
      }
      issue(i);
    }
    cp_async_commit();
  }
  pdl_wait();
  trace_stamp(a.trace, 1);
  trace_stamp(a.trace, 2);  // q was quantised by warp 0 before its copies
  constexpr int kNW = (HD / 32 + 3) / 4;  // packed int8 words of a lane's share of a row
  uint32_t nkw[kNW], nvw[kNW];
  uint16_t nkd = 0, nvd = 0;
  if (own_new) {
    const long long src = (long long)z * a.new_zstride + (long long)kvh * HD;
    nkd = q8_quantize_row<HD>(a.k_new + src, lane, nkw);
    nvd = q8_quantize_row<HD>(a.v_new + src, lane, nvw);
    if (hg == 0) {
      const long long crow = row0 + new_row;  // cache row of pos
      q8_store_row<HD>(a.k8 + crow * HD, a.ksc + crow * (HD / 32), lane, nkw, nkd);
      q8_store_row<HD>(a.v8 + crow * HD, a.vsc + crow * (HD / 32), lane, nvw, nvd);
    }
  }
  __syncthreads();  // s_q8 / s_dq written
  // score layout: lane (rq, sg) holds values [sg*HD/8, (sg+1)*HD/8) of every
  // q row and the scale of their block
  const int rq = lane >> 3, sg = lane & 7;
  uint32_t qw[GT][C::kKW];
  float dq[GT];
#pragma unroll
  for (int g = 0; g < GT; ++g) {
#pragma unroll
    for (int w = 0; w < C::kKW; ++w) qw[g][w] = s_q8[(g * HD + sg * C::kKB) / 4 + w];
    dq[g] = s_dq[(g * HD + sg * C::kKB) / 32];
  }

  float my_m[GT], my_l[GT];
  float acc[GT][C::kEPL];
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    my_m[g] = -INFINITY;
    my_l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < C::kEPL; ++e) acc[g][e] = 0.f;
  }
  const int kblk = sg * C::kKB / 32;  // block of this lane's K values

  for (int i = 0; i < my_tiles; ++i) {
    if (i + C::kStages - 1 < my_tiles) issue(i + C::kStages - 1);
    cp_async_commit();
    cp_async_wait<C::kStages - 1>();
    __syncwarp();
    unsigned char* stw = wring + (i % C::kStages) * C::kStageBytes;
    if (i == new_i) {  // the stage holds the cache's old row of pos: put the token's row in its place
      const int r = new_row - (first + i * step) * C::kR;
      q8_store_row<HD>(reinterpret_cast<int8_t*>(stw) + r * HD,
                       reinterpret_cast<uint16_t*>(stw + 2 * C::kTileKB) + r * (HD / 32), lane, nkw, nkd);
      q8_store_row<HD>(reinterpret_cast<int8_t*>(stw) + C::kTileKB + r * HD,
                       reinterpret_cast<uint16_t*>(stw + 2 * C::kTileKB + C::kTileSB) + r * (HD / 32), lane, nvw, nvd);
      __syncwarp();
    }
    const unsigned char* st = stw;
    const int8_t* kt = reinterpret_cast<const int8_t*>(st);
    const int8_t* vt = kt + C::kTileKB;
    const uint16_t* kst = reinterpret_cast<const uint16_t*>(st + 2 * C::kTileKB);
    const uint16_t* vst = reinterpret_cast<const uint16_t*>(st + 2 * C::kTileKB + C::kTileSB);
    const int nvalid = min(C::kR, n_rows - (first + i * step) * C::kR);

    // ---- scores: 8 lanes per K row, 4 rows per pass ----
    float sc[C::kR / 4][GT];
#pragma unroll
    for (int pp = 0; pp < C::kR / 4; ++pp) {
      const int r = rq + 4 * pp;
      uint32_t kw[C::kKW];
      if constexpr (C::kKW == 2) {
        const uint2 t = *reinterpret_cast<const uint2*>(kt + r * HD + sg * C::kKB);
        kw[0] = t.x;
        kw[1] = t.y;
      } else {
#pragma unroll
        for (int w = 0; w < C::kKW; w += 4) {
          const uint4 t = *reinterpret_cast<const uint4*>(kt + r * HD + sg * C::kKB + 4 * w);
          kw[w] = t.x;
          kw[w + 1] = t.y;
          kw[w + 2] = t.z;
          kw[w + 3] = t.w;
        }
      }
      const float dk = fp16_to_f32(kst[r * (HD / 32) + kblk]);
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        int isum = 0;
#pragma unroll
        for (int w = 0; w < C::kKW; ++w) isum = __dp4a((int)kw[w], (int)qw[g][w], isum);
        // lanes of one block: exact int32 sum
#pragma unroll
        for (int off = 1; off < C::kLanesPerBlock; off <<= 1) isum += __shfl_xor_sync(0xffffffffu, isum, off);
        float t = (dq[g] * dk) * (float)isum;
        // blocks of the row
#pragma unroll
        for (int off = C::kLanesPerBlock; off < 8; off <<= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
        sc[pp][g] = r < nvalid ? t * kLog2e : -INFINITY;
      }
    }
    // ---- online softmax per q head (row 0 of a tile is valid, so maxima are finite) ----
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      float tmax = sc[0][g];
#pragma unroll
      for (int pp = 1; pp < C::kR / 4; ++pp) tmax = fmaxf(tmax, sc[pp][g]);
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 8));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
      const float m_new = fmaxf(my_m[g], tmax);
      const float alpha = fast_exp2(my_m[g] - m_new);
      float tsum = 0.f;
#pragma unroll
      for (int pp = 0; pp < C::kR / 4; ++pp) {
        sc[pp][g] = fast_exp2(sc[pp][g] - m_new);
        tsum += sc[pp][g];
      }
      tsum += __shfl_xor_sync(0xffffffffu, tsum, 8);
      tsum += __shfl_xor_sync(0xffffffffu, tsum, 16);
      my_l[g] = my_l[g] * alpha + tsum;
      my_m[g] = m_new;
#pragma unroll
      for (int e = 0; e < C::kEPL; ++e) acc[g][e] *= alpha;
    }
    // lane sg of a row's 8 (each holds the row's weights of every head)
    // takes block sg of the row: its scale times each head's weight
    float (*sw)[kNB][GT] = s_w[warp];
    if (sg < kNB) {
#pragma unroll
      for (int pp = 0; pp < C::kR / 4; ++pp) {
        const int r = rq + 4 * pp;
        const float dvb = fp16_to_f32(vst[r * kNB + sg]);
#pragma unroll
        for (int g = 0; g < GT; ++g) sw[r][sg][g] = dvb * sc[pp][g];
      }
    }
    __syncwarp();
    // ---- values: 32 lanes per V row, lane_elem layout ----
#pragma unroll
    for (int r = 0; r < C::kR; ++r) {
      // int8 -> fp32 exactly, two values per instruction: byte b + 128 as the
      // low mantissa byte of 2^23, minus 2^23 + 128
      float2 vx[C::kEPL / 2];
      const float2 kBias = make_float2(-8388736.0f, -8388736.0f);
      if constexpr (HD == 64) {
        const uint32_t t = *reinterpret_cast<const uint16_t*>(vt + r * HD + 2 * lane) ^ 0x8080u;
        vx[0] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(t, 0x4B000000u, 0x7540)),
                                       __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7541))),
                           kBias);
      } else {
#pragma unroll
        for (int c = 0; c < HD / 128; ++c) {
          const uint32_t t = *reinterpret_cast<const uint32_t*>(vt + r * HD + c * 128 + 4 * lane) ^ 0x80808080u;
          vx[2 * c] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(t, 0x4B000000u, 0x7540)),
                                             __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7541))),
                                 kBias);
          vx[2 * c + 1] = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(t, 0x4B000000u, 0x7542)),
                                                 __uint_as_float(__byte_perm(t, 0x4B000000u, 0x7543))),
                                     kBias);
        }
      }
      // acc += v * (block scale * weight), as c:1605; the packed FMA rounds
      // each half like fmaf.  Value e of the lane lies in block
      // HD == 64 ? lane / 16 : (e / 4) * 4 + lane / 8.
#pragma unroll
      for (int c = 0; c < (C::kEPL + 3) / 4; ++c) {
        const int b = HD == 64 ? lane / 16 : c * 4 + lane / 8;
        float f[GT];
#pragma unroll
        for (int g = 0; g < GT; g += 4) {
          if constexpr (GT >= 4) {
            const float4 t = lds128(&sw[r][b][g]);
            f[g] = t.x;
            f[g + 1] = t.y;
            f[g + 2] = t.z;
            f[g + 3] = t.w;
          }
        }
        if constexpr (GT < 4) {
#pragma unroll
          for (int g = 0; g < GT; ++g) f[g] = sw[r][b][g];
        }
#pragma unroll
        for (int g = 0; g < GT; ++g) {
#pragma unroll
          for (int e = 4 * c; e < 4 * c + 4 && e < C::kEPL; e += 2) {
            const float2 r2 = __ffma2_rn(vx[e / 2], make_float2(f[g], f[g]), make_float2(acc[g][e], acc[g][e + 1]));
            acc[g][e] = r2.x;
            acc[g][e + 1] = r2.y;
          }
        }
      }
    }
    __syncwarp();  // every lane is done with this stage and s_w before they are refilled
  }
  cp_async_wait<0>();
  trace_stamp(a.trace, 3);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      ms.m[warp][g] = my_m[g];
      ms.l[warp][g] = my_l[g];
    }
  }
  decode_finish<HD, GT, C::kWarps, C::kThreads>(a, ms, ring, acc, warp, lane, split, unit, z, h0);
}

}  // namespace l3p
