// rope.cuh -- the engines' pre-attention step on the device (sm_100a): Gemma3
// QK-RMSNorm, rotary position embedding of q and K, and the K/V cache write,
// in one launch, so the projection outputs never leave the GPU.
//
// Replaces, per token at position pos of layer l:
//   rmsnorm_per_head on q and k (c:3150-3165, applied when the model is
//     Gemma3 and has attn_q_norm / attn_k_norm weights, c:3233-3236,
//     c:3507-3512):  ss = sum_j x_j*x_j (in order j = 0..hd-1),
//     r = 1/sqrtf(ss * (1/hd) + eps), o_j = w_j * (r * x_j);
//   RoPE with the per-layer cos/sin tables (c:381-421, c:456-468):
//     Gemma3 NEOX pairs (i, i + hd/2) (c:3254-3278, c:3518-3541),
//     Llama consecutive pairs (2i, 2i+1) (c:3279-3296, c:3542-3560),
//     x0' = x0*cos - x1*sin, x1' = x0*sin + x1*cos;
//   the cache write of K and V (c:3299-3308, c:3562-3567), fp32 or Q8_0.
// q leaves here rotated but not yet multiplied by attn_scale: the attention
// kernels multiply it elementwise, which is the reference's own last step of
// its fused RoPE expression ((x0*cos - x1*sin) * attn_scale, c:3264, c:3288).
//
// Every operation is the IEEE single-precision operation the reference
// performs, in the same order, with no contraction into fused multiply-adds:
// the sum of squares runs sequentially in one thread, the square root and the
// division are correctly rounded.  The results are therefore bit-identical to
// the reference built without fast-math (its -Ofast build vectorises the sum
// and may contract products, which changes the last bits).
//
// Work decomposition: one warp per (token, head row); the owned q heads come
// first, then the owned KV heads (K rotated, V copied).  Lane l holds the HD/32
// consecutive values [l*HD/32, (l+1)*HD/32) of its row -- whole consecutive
// pairs for the Llama form, and for the NEOX form the partner of value i < hd/2
// sits in lane l + 16 at the same slot.  This is also the lane layout of the
// Q8_0 quantiser (q8_quantize_lanes), so a K or V row is quantised straight
// from registers.
#pragma once
#include "decode_q8.cuh"

namespace l3p {

constexpr int kRopeWarps = 8;  // rows per CTA

struct RopeArgs {
  const float* q;     // [n_tok][q_stride], q head h at h*HD
  const float* k;     // [n_tok][kv_stride]
  const float* v;     // [n_tok][kv_stride] (read only when writing the cache)
  long long q_stride, kv_stride;
  float* q_out;       // rotated q rows, same layout as q (owned heads only)
  float* k_out;       // optional rotated k rows, same layout as k (owned heads only)
  // optional cache destination of K (rotated) and V, already offset to the
  // layer and the first owned KV head: fp32 rows (kc, vc) or Q8_0 (k8/ksc, v8/vsc)
  float* kc;
  float* vc;
  int8_t* k8;
  int8_t* v8;
  uint16_t* ksc;
  uint16_t* vsc;
  long long head_stride;  // cache values per owned KV head (cap * HD)
  int row0;               // cache row of token 0 (pos0 - seq_begin); rows outside [0, cap) are not written
  int cap;
  const float2* tab;      // (cos, sin) of this layer's table: [seq_len][HD/2]
  const float* q_norm;    // this layer's attn_q_norm / attn_k_norm weights [HD], or null (no QK-norm)
  const float* k_norm;
  float eps;              // rms_norm_eps (c:3198)
  float inv_hd;           // 1.0f / (float)HD (c:437)
  int pos0, n_tok;
  int q_head0, n_qh;      // owned q heads
  int kv_head0, n_kvh;    // owned KV heads
  int neox;               // Gemma3 pairing
};

// One row: optional per-head RMS norm, then the rotation.  x[] holds this
// lane's N values; red is this warp's HD-float scratch.
template <int HD>
__device__ __forceinline__ void rope_row(float (&x)[HD / 32], const float* __restrict__ w, const float2* __restrict__ cs,
                                         bool neox, float eps, float inv_hd, float* red, int lane) {
  constexpr int N = HD / 32;
  if (w != nullptr) {
    // ss accumulated in the reference's order: squares in parallel, the sum in one thread
#pragma unroll
    for (int i = 0; i < N; ++i) red[lane * N + i] = __fmul_rn(x[i], x[i]);
    __syncwarp();
    float r = 0.f;
    if (lane == 0) {
      float ss = 0.f;
#pragma unroll 8
      for (int j = 0; j < HD; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(red + j);
        ss = __fadd_rn(ss, t.x);
        ss = __fadd_rn(ss, t.y);
        ss = __fadd_rn(ss, t.z);
        ss = __fadd_rn(ss, t.w);
      }
      r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, inv_hd), eps)));
    }
    r = __shfl_sync(0xffffffffu, r, 0);
    __syncwarp();  // red is reused by the next row of this warp
#pragma unroll
    for (int i = 0; i < N; ++i) x[i] = __fmul_rn(w[lane * N + i], __fmul_rn(r, x[i]));
  }
  if (neox) {
    // pair (i, i + HD/2): value slot s of lane l < 16 pairs with slot s of lane l + 16
    const bool lo = lane < 16;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, x[i], 16);
      const float2 t = cs[(lane & 15) * N + i];
      const float v0 = lo ? x[i] : other, v1 = lo ? other : x[i];
      x[i] = lo ? __fsub_rn(__fmul_rn(v0, t.x), __fmul_rn(v1, t.y)) : __fadd_rn(__fmul_rn(v0, t.y), __fmul_rn(v1, t.x));
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 t = cs[(lane * N + i) / 2];
      const float v0 = x[i], v1 = x[i + 1];
      x[i] = __fsub_rn(__fmul_rn(v0, t.x), __fmul_rn(v1, t.y));
      x[i + 1] = __fadd_rn(__fmul_rn(v0, t.y), __fmul_rn(v1, t.x));
    }
  }
}

template <int N>
__device__ __forceinline__ void load_lane(const float* __restrict__ src, float (&x)[N]) {
  if constexpr (N == 2) {
    const float2 t = *reinterpret_cast<const float2*>(src);
    x[0] = t.x;
    x[1] = t.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(src + i);
      x[i] = t.x;
      x[i + 1] = t.y;
      x[i + 2] = t.z;
      x[i + 3] = t.w;
    }
  }
}

template <int N>
__device__ __forceinline__ void store_lane(float* __restrict__ dst, const float (&x)[N]) {
  if constexpr (N == 2) {
    *reinterpret_cast<float2*>(dst) = make_float2(x[0], x[1]);
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
  }
}

// One Q8_0 cache row from a warp's registers (quantize_to_q8_0_cache, c:1535-1570).
template <int N>
__device__ __forceinline__ void store_q8_lane(int8_t* __restrict__ d8, uint16_t* __restrict__ dsc, const float (&x)[N],
                                              int lane) {
  uint32_t w[(N + 3) / 4];
  const uint16_t d = q8_quantize_lanes<N>(x, w);
  int8_t* dst = d8 + lane * N;
  if constexpr (N == 2) {
    *reinterpret_cast<uint16_t*>(dst) = (uint16_t)w[0];
  } else {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) reinterpret_cast<uint32_t*>(dst)[i] = w[i];
  }
  if ((lane * N) % 32 == 0) dsc[lane * N / 32] = d;
}

// grid (n_tok, ceil((n_qh + n_kvh) / kRopeWarps)), kRopeWarps * 32 threads.
template <int HD>
__global__ void __launch_bounds__(kRopeWarps * 32) rope_qkv_kernel(RopeArgs a) {
  constexpr int N = HD / 32;
  __shared__ __align__(16) float red[kRopeWarps][HD];
  // the inputs come from the kernel before this one
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok = blockIdx.x;
  const int r = blockIdx.y * kRopeWarps + warp;
  if (r >= a.n_qh + a.n_kvh) return;
  const int pos = a.pos0 + tok;
  const float2* cs = a.tab + (long long)pos * (HD / 2);
  float x[N];
  if (r < a.n_qh) {
    const long long off = (long long)tok * a.q_stride + (long long)(a.q_head0 + r) * HD + lane * N;
    load_lane<N>(a.q + off, x);
    rope_row<HD>(x, a.q_norm, cs, a.neox != 0, a.eps, a.inv_hd, red[warp], lane);
    store_lane<N>(a.q_out + off, x);
    return;
  }
  const int kvl = r - a.n_qh;  // owned KV head index
  const long long off = (long long)tok * a.kv_stride + (long long)(a.kv_head0 + kvl) * HD + lane * N;
  load_lane<N>(a.k + off, x);
  rope_row<HD>(x, a.k_norm, cs, a.neox != 0, a.eps, a.inv_hd, red[warp], lane);
  if (a.k_out) store_lane<N>(a.k_out + off, x);
  const int row = a.row0 + tok;
  if (row < 0 || row >= a.cap || (a.kc == nullptr && a.k8 == nullptr)) return;
  const long long crow = (long long)kvl * a.head_stride + (long long)row * HD;  // value offset of the cache row
  float xv[N];
  load_lane<N>(a.v + off, xv);
  if (a.k8 != nullptr) {
    store_q8_lane<N>(a.k8 + crow, a.ksc + crow / 32, x, lane);
    store_q8_lane<N>(a.v8 + crow, a.vsc + crow / 32, xv, lane);
  } else {
    store_lane<N>(a.kc + crow + lane * N, x);
    store_lane<N>(a.vc + crow + lane * N, xv);
  }
}

}  // namespace l3p
