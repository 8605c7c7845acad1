// wo.cuh -- the attention output's consumer on the device (sm_100a): the
// `wo` projection xout = Wo . xb with GGUF-quantised weights (c:3362,
// js:5191), tensor-parallel by head.
//
// The reference's matmul_quantized (c:2091-2132) takes one of three paths
// per weight type, and so does this file:
//   - row dequantiser, fp32 dots (matmul_deq_4row, c:2136-2176):
//       Q8_0  (34-byte blocks of 32)   value = d * q8                 (c:691-702)
//       Q2_K, Q3_K, Q5_K: the formats at WoQ2K, WoQ3K, WoQ5K (c:748-871)
//       Q4_K  (144-byte blocks of 256) value = d*sc_j * q4 - dmin*m_j (c:704-746)
//       Q6_K  (210-byte blocks of 256) value = d * sc_k * (q6 - 32)   (c:873-902)
//   - x quantised to Q8_0, exact integer block dots: Q4_0, Q4_1, Q5_0, Q5_1,
//     IQ4_NL (WoQ8x);
//   - fp32 dots with the converted weights: F32, F16, BF16 (WoFloat).
// The products are the same; the summation order is not (per lane, then
// across lanes and warps; scale factors applied per sub-block), which moves
// results by a few ulps of the row sum, inside the 1e-4 contract.
//
// A context owns the q heads of its KV heads, so it holds the columns
// [q_head0*hd, (q_head0+n_qh)*hd) of every row: its xout is the partial sum
// over its heads, and one context per GPU gives the by-head tensor-parallel
// split (the partials add up across GPUs).
//
// Device layout per layer (row-major, every row 16-byte aligned):
//   Q8_0  int8 values [dim][C] and fp16 scales [dim][sc_stride/2]
//         (sc_stride = C/16 bytes rounded up to 16)
//   Q4_K  the GGUF blocks as they are, [dim][C/256][144]
//   Q6_K  blocks padded to 224 bytes: ql 128 | qh 64 | scales 16 | d 2 | 14 spare
//
// Kernel.  A row is cut into column slices of 1024 values (Q8_0, Q4_K) or
// 2048 (Q6_K); lane l of a warp always covers the same columns of its slice,
// so it loads its x values once into registers and reuses them for every
// row, and every warp-wide weight load is 512 contiguous bytes.  The NW warps
// of a CTA form wc column groups (one slice each) x NW/wc row groups; a CTA
// takes a contiguous block of rows, each warp keeps kUnroll rows of weight
// loads in flight in registers, and the column groups' per-row partials are
// added in shared memory.  CTAs are small (4 warps when the owned columns fit
// 4 slices) and use little shared memory, so under programmatic dependent
// launch they become resident beside the attention kernel's CTAs, request
// their first rows while it finishes and wait (griddepcontrol.wait) only
// before reading x.
//
// Integers become floats by placing them in the mantissa of 2^23 (one byte
// permute) and subtracting 2^23 plus the offset (one add): exact, and on the
// full-rate pipes (an int-to-float conversion per value would run at a
// quarter of the rate and bound the kernel).
#pragma once
#include "decode_q8.cuh"
#include "limits.cuh"

namespace l3p {

struct WoArgs {
  const uint8_t* w;     // this layer's weight rows (format above), owned columns only
  const uint8_t* wsc;   // Q8_0 scales, sc_stride bytes per row
  long long row_bytes;  // bytes of one weight row in `w`
  int sc_stride;        // bytes of one row of Q8_0 scales (0 for the K-quants)
  int rows, C;          // output rows (dim), owned columns
  int rows_per_cta;
  int wc;               // column groups per CTA (power of two <= warps)
  const float* x;       // owned columns of the attention output (x[0] = column q_head0*hd)
  float* y;             // [rows]
  // tensor-parallel group (tp_members > 0): y receives the SUM of every
  // member's partial, reduce-scattered and all-gathered through the members'
  // exchange regions (layout in limits.cuh; protocol at wo_tp_exchange)
  int tp_members, tp_member;
  uint8_t* tp_regions[kXchgMaxParts];  // every member's exchange region (own included)
  int* err;                            // device error word (kErrTimeout)
  // stage stamps of the tensor-parallel tail (builds with L3P_DECODE_TRACE):
  // 0 start, 1 after griddepcontrol.wait, 2 GEMV done, 3 partial sent to every
  // member, 4 every member's rows arrived and summed, 5 exit
  unsigned long long* trace;
};

// Byte i (0..3) of w as the float 2^23 + byte: exact for every byte.
__device__ __forceinline__ float byte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)i));
}
constexpr float kTwo23 = 8388608.f;
// Bytes i and i+1 of w, minus `bias`, as two exact floats: two byte permutes
// and one packed subtraction.
__device__ __forceinline__ float2 byte_pair(uint32_t w, int i, float bias) {
  return __fadd2_rn(make_float2(byte_f(w, i), byte_f(w, i + 1)), make_float2(-bias, -bias));
}

// Sums of x over the two 16-value runs of a lane (the formats with mins).
struct WoSums {
  float s[2];
};

// Per-format lane work: the lane's columns, its state of x (prepared once per
// launch), its loads of one row's slice and the dot product.

struct WoQ8 {
  static constexpr int kSlice = 1024;  // columns per warp slice
  static constexpr int kLaneCols = 32;
  using X = WoSums;  // per-lane state of x, prepared once per launch
  static constexpr int kUnroll = 8;
  struct Raw {
    uint4 a, b;
    uint16_t d0, d1;
  };
  // lane l: columns [16l, 16l+16) and [512+16l, 512+16l+16) of its slice
  __device__ static int col(int lane, int i) { return (i < 16 ? 16 * lane : 512 + 16 * lane - 16) + i; }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31;
    const uint8_t* s = p.w + (long long)row * p.row_bytes + c0 + 16 * lane;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(p.wsc + (long long)row * p.sc_stride) + c0 / 32 + lane / 2;
    r.a = __ldg(reinterpret_cast<const uint4*>(s));
    r.d0 = __ldg(sc);
    // the owned columns may end inside the slice's second half
    if (c0 + 512 + 16 * lane < p.C) {
      r.b = __ldg(reinterpret_cast<const uint4*>(s + 512));
      r.d1 = __ldg(sc + 16);
    } else {
      r.b = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // zeros after the bias flip
      r.d1 = 0;
    }
  }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const WoSums&) {
    // int8 q: (q ^ 0x80) is q + 128 as an unsigned byte
    const uint32_t wa[4] = {r.a.x ^ 0x80808080u, r.a.y ^ 0x80808080u, r.a.z ^ 0x80808080u, r.a.w ^ 0x80808080u};
    const uint32_t wb[4] = {r.b.x ^ 0x80808080u, r.b.y ^ 0x80808080u, r.b.z ^ 0x80808080u, r.b.w ^ 0x80808080u};
    // packed pairs (i, i+1): two products per FFMA2, each rounded like fmaf
    float2 s[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)}, t[2] = {s[0], s[1]};
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      s[(i / 2) % 2] = __ffma2_rn(byte_pair(wa[i / 4], i % 4, kTwo23 + 128.f), make_float2(x[i], x[i + 1]), s[(i / 2) % 2]);
      t[(i / 2) % 2] =
          __ffma2_rn(byte_pair(wb[i / 4], i % 4, kTwo23 + 128.f), make_float2(x[16 + i], x[17 + i]), t[(i / 2) % 2]);
    }
    return fp16_to_f32(r.d0) * ((s[0].x + s[1].x) + (s[0].y + s[1].y)) +
           fp16_to_f32(r.d1) * ((t[0].x + t[1].x) + (t[0].y + t[1].y));
  }
  __device__ static void prep(const float (&)[kLaneCols], WoSums& xs) { xs.s[0] = xs.s[1] = 0.f; }
};

struct WoQ4K {
  static constexpr int kSlice = 1024;  // 4 blocks of 256
  static constexpr int kLaneCols = 32;
  using X = WoSums;  // per-lane state of x, prepared once per launch
  static constexpr int kUnroll = 8;
  struct Raw {
    uint4 h;  // d, dmin, 12 scale bytes
    uint4 q;  // 16 quant bytes: 16 low nibbles (sub-block 2p) and 16 high (sub-block 2p+1)
  };
  // lane = 8*block + c; quant bytes [16c, 16c+16) of the block hold values
  // o+i of sub-blocks 2p (low nibble) and 2p+1 (high), p = c/2, o = 16*(c%2)
  __device__ static int col(int lane, int i) {
    const int b = lane >> 3, c = lane & 7, p = c >> 1, o = 16 * (c & 1);
    return 256 * b + 64 * p + o + (i < 16 ? i : 32 + (i - 16));
  }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31;
    const uint8_t* blk = p.w + (long long)row * p.row_bytes + (long long)(c0 / 256 + (lane >> 3)) * 144;
    r.h = __ldg(reinterpret_cast<const uint4*>(blk));
    r.q = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * (lane & 7)));
  }
  // byte k (0..11) of the packed scales, held in the words s0 s1 s2 (selects, no local memory)
  __device__ static int sbyte(uint32_t s0, uint32_t s1, uint32_t s2, int k) {
    const uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
    return (int)((w >> (8 * (k & 3))) & 0xffu);
  }
  // 6-bit scale and min of sub-block j from the 12 packed bytes (c:705-713)
  __device__ static void scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& m) {
    if (j < 4) {
      sc = sbyte(s0, s1, s2, j) & 63;
      m = sbyte(s0, s1, s2, j + 4) & 63;
    } else {
      sc = (sbyte(s0, s1, s2, j + 4) & 15) | ((sbyte(s0, s1, s2, j - 4) >> 6) << 4);
      m = (sbyte(s0, s1, s2, j + 4) >> 4) | ((sbyte(s0, s1, s2, j) >> 6) << 4);
    }
  }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const WoSums& xs) {
    const int lane = threadIdx.x & 31, p = (lane & 7) >> 1;
    const float d = fp16_to_f32((uint16_t)(r.h.x & 0xffffu)), dmin = fp16_to_f32((uint16_t)(r.h.x >> 16));
    int sc0, m0, sc1, m1;
    scale_min(r.h.y, r.h.z, r.h.w, 2 * p, sc0, m0);
    scale_min(r.h.y, r.h.z, r.h.w, 2 * p + 1, sc1, m1);
    const uint32_t q[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
    float2 lo = make_float2(0.f, 0.f), hi = lo;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const uint32_t l4 = q[i / 4] & 0x0f0f0f0fu, h4 = (q[i / 4] >> 4) & 0x0f0f0f0fu;
      lo = __ffma2_rn(byte_pair(l4, i % 4, kTwo23), make_float2(x[i], x[i + 1]), lo);
      hi = __ffma2_rn(byte_pair(h4, i % 4, kTwo23), make_float2(x[16 + i], x[17 + i]), hi);
    }
    return d * ((float)sc0 * (lo.x + lo.y) + (float)sc1 * (hi.x + hi.y)) -
           dmin * ((float)m0 * xs.s[0] + (float)m1 * xs.s[1]);
  }
  __device__ static void prep(const float (&x)[kLaneCols], WoSums& xs) {
    xs.s[0] = xs.s[1] = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      xs.s[0] += x[i];
      xs.s[1] += x[16 + i];
    }
  }
};

// Q5_K: Q4_K's lanes and sub-block pairs plus the fifth bit of every value
// from qh (c:834-871): sub-block 2p takes bit 2p of qh[l], 2p+1 bit 2p+1.
// Device block: the GGUF block as is (176 bytes: d, dmin, 12 scale bytes,
// qh[32], qs[128]).
struct WoQ5K {
  static constexpr int kSlice = 1024;  // 4 blocks of 256
  static constexpr int kLaneCols = 32;
  using X = WoSums;  // per-lane state of x, prepared once per launch
  static constexpr int kUnroll = 6;
  static constexpr int kBlockBytes = 176;
  struct Raw {
    uint4 h;   // d, dmin, 12 scale bytes
    uint4 q;   // 16 bytes of qs: low nibbles (sub-block 2p), high (2p+1)
    uint4 qh;  // qh[16*(c%2) ..+16): the fifth bits of those values
  };
  __device__ static int col(int lane, int i) { return WoQ4K::col(lane, i); }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31;
    const uint8_t* blk = p.w + (long long)row * p.row_bytes + (long long)(c0 / 256 + (lane >> 3)) * kBlockBytes;
    r.h = __ldg(reinterpret_cast<const uint4*>(blk));
    r.qh = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 16 * (lane & 1)));
    r.q = __ldg(reinterpret_cast<const uint4*>(blk + 48 + 16 * (lane & 7)));
  }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const WoSums& xs) {
    const int lane = threadIdx.x & 31, p = (lane & 7) >> 1;
    const float d = fp16_to_f32((uint16_t)(r.h.x & 0xffffu)), dmin = fp16_to_f32((uint16_t)(r.h.x >> 16));
    int sc0, m0, sc1, m1;
    WoQ4K::scale_min(r.h.y, r.h.z, r.h.w, 2 * p, sc0, m0);
    WoQ4K::scale_min(r.h.y, r.h.z, r.h.w, 2 * p + 1, sc1, m1);
    const uint32_t q[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
    const uint32_t hb[4] = {r.qh.x, r.qh.y, r.qh.z, r.qh.w};
    float2 lo = make_float2(0.f, 0.f), hi = lo;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const uint32_t l5 = (q[i / 4] & 0x0f0f0f0fu) | (((hb[i / 4] >> (2 * p)) & 0x01010101u) << 4);
      const uint32_t h5 = ((q[i / 4] >> 4) & 0x0f0f0f0fu) | (((hb[i / 4] >> (2 * p + 1)) & 0x01010101u) << 4);
      lo = __ffma2_rn(byte_pair(l5, i % 4, kTwo23), make_float2(x[i], x[i + 1]), lo);
      hi = __ffma2_rn(byte_pair(h5, i % 4, kTwo23), make_float2(x[16 + i], x[17 + i]), hi);
    }
    return d * ((float)sc0 * (lo.x + lo.y) + (float)sc1 * (hi.x + hi.y)) -
           dmin * ((float)m0 * xs.s[0] + (float)m1 * xs.s[1]);
  }
  __device__ static void prep(const float (&x)[kLaneCols], WoSums& xs) { WoQ4K::prep(x, xs); }
};

// Q2_K and Q3_K: per half h of a 256-value block, bit pair j of 32 quant
// bytes gives 32 values (two sub-blocks of 16).  lane = 8*block + 4h + j
// takes those 32 values, columns 128h + 32j + i (c:748-832).
__device__ __forceinline__ int wo_k2_col(int lane, int i) {
  return 256 * (lane >> 3) + 128 * ((lane >> 2) & 1) + 32 * (lane & 3) + i;
}

// Q2_K: value = (d * (s & 15)) * q - dmin * (s >> 4), q 2-bit, s the
// sub-block's scale byte (scales[8h + 2j], [8h + 2j + 1]).  Device block
// (96 bytes): the GGUF block's 84 (scales[16], qs[64], d, dmin), padded.
struct WoQ2K {
  static constexpr int kSlice = 1024;  // 4 blocks of 256
  static constexpr int kLaneCols = 32;
  using X = WoSums;  // per-lane state of x, prepared once per launch
  static constexpr int kUnroll = 8;
  static constexpr int kBlockBytes = 96;
  struct Raw {
    uint4 q0, q1;  // qs[32h ..+32)
    uint32_t dd;   // d, dmin
    uint16_t sc;   // the two sub-blocks' scale bytes
  };
  __device__ static int col(int lane, int i) { return wo_k2_col(lane, i); }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31, h = (lane >> 2) & 1, j = lane & 3;
    const uint8_t* blk = p.w + (long long)row * p.row_bytes + (long long)(c0 / 256 + (lane >> 3)) * kBlockBytes;
    r.q0 = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * h));
    r.q1 = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * h));
    r.sc = __ldg(reinterpret_cast<const uint16_t*>(blk + 8 * h + 2 * j));
    r.dd = __ldg(reinterpret_cast<const uint32_t*>(blk + 80));
  }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const WoSums& xs) {
    const int shift = 2 * (threadIdx.x & 3);
    const float d = fp16_to_f32((uint16_t)(r.dd & 0xffffu)), dmin = fp16_to_f32((uint16_t)(r.dd >> 16));
    const int s0 = r.sc & 0xff, s1 = r.sc >> 8;
    const uint32_t a[4] = {r.q0.x, r.q0.y, r.q0.z, r.q0.w};
    const uint32_t b[4] = {r.q1.x, r.q1.y, r.q1.z, r.q1.w};
    float2 lo = make_float2(0.f, 0.f), hi = lo;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      lo = __ffma2_rn(byte_pair((a[i / 4] >> shift) & 0x03030303u, i % 4, kTwo23), make_float2(x[i], x[i + 1]), lo);
      hi = __ffma2_rn(byte_pair((b[i / 4] >> shift) & 0x03030303u, i % 4, kTwo23), make_float2(x[16 + i], x[17 + i]),
                      hi);
    }
    return d * ((float)(s0 & 15) * (lo.x + lo.y) + (float)(s1 & 15) * (hi.x + hi.y)) -
           dmin * ((float)(s0 >> 4) * xs.s[0] + (float)(s1 >> 4) * xs.s[1]);
  }
  __device__ static void prep(const float (&x)[kLaneCols], WoSums& xs) { WoQ4K::prep(x, xs); }
};

// Q3_K: value = (d * (s - 32)) * (q - 4 * !hbit), q 2-bit, hbit bit 4h + j of
// hmask[i], s the sub-block's 6-bit scale: the low nibble of byte k (k < 8)
// or the high nibble of byte k - 8, above it bit pair k/4 of byte 8 + k%4.
// Device block (112 bytes): the GGUF block's 110 (hmask[32], qs[64],
// scales[12], d), padded.
struct WoQ3K {
  static constexpr int kSlice = 1024;  // 4 blocks of 256
  static constexpr int kLaneCols = 32;
  using X = WoSums;  // per-lane state of x, prepared once per launch
  static constexpr int kUnroll = 4;
  static constexpr int kBlockBytes = 112;
  struct Raw {
    uint4 q0, q1;  // qs[32h ..+32)
    uint4 m0, m1;  // hmask[0 ..32)
    uint4 s;       // scales[12], d
  };
  __device__ static int col(int lane, int i) { return wo_k2_col(lane, i); }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31, h = (lane >> 2) & 1;
    const uint8_t* blk = p.w + (long long)row * p.row_bytes + (long long)(c0 / 256 + (lane >> 3)) * kBlockBytes;
    r.m0 = __ldg(reinterpret_cast<const uint4*>(blk));
    r.m1 = __ldg(reinterpret_cast<const uint4*>(blk + 16));
    r.q0 = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * h));
    r.q1 = __ldg(reinterpret_cast<const uint4*>(blk + 48 + 32 * h));
    r.s = __ldg(reinterpret_cast<const uint4*>(blk + 96));
  }
  __device__ static int scale(const uint4& s, int k) {
    const int low = k < 8 ? WoQ4K::sbyte(s.x, s.y, s.z, k) & 15 : WoQ4K::sbyte(s.x, s.y, s.z, k - 8) >> 4;
    const int high = (WoQ4K::sbyte(s.x, s.y, s.z, 8 + (k & 3)) >> (2 * (k >> 2))) & 3;
    return (low | (high << 4)) - 32;
  }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const WoSums&) {
    const int lane = threadIdx.x & 31, h = (lane >> 2) & 1, j = lane & 3;
    const int shift = 2 * j, bit = 4 * h + j;
    const float d = fp16_to_f32((uint16_t)(r.s.w & 0xffffu));
    const int sc0 = scale(r.s, 8 * h + 2 * j), sc1 = scale(r.s, 8 * h + 2 * j + 1);
    const uint32_t a[4] = {r.q0.x, r.q0.y, r.q0.z, r.q0.w};
    const uint32_t b[4] = {r.q1.x, r.q1.y, r.q1.z, r.q1.w};
    const uint32_t ma[4] = {r.m0.x, r.m0.y, r.m0.z, r.m0.w};
    const uint32_t mb[4] = {r.m1.x, r.m1.y, r.m1.z, r.m1.w};
    float2 lo = make_float2(0.f, 0.f), hi = lo;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      // q + 4*hbit in 0..7; the value is that minus 4
      const uint32_t ua = ((a[i / 4] >> shift) & 0x03030303u) | (((ma[i / 4] >> bit) & 0x01010101u) << 2);
      const uint32_t ub = ((b[i / 4] >> shift) & 0x03030303u) | (((mb[i / 4] >> bit) & 0x01010101u) << 2);
      lo = __ffma2_rn(byte_pair(ua, i % 4, kTwo23 + 4.f), make_float2(x[i], x[i + 1]), lo);
      hi = __ffma2_rn(byte_pair(ub, i % 4, kTwo23 + 4.f), make_float2(x[16 + i], x[17 + i]), hi);
    }
    return d * ((float)sc0 * (lo.x + lo.y) + (float)sc1 * (hi.x + hi.y));
  }
  __device__ static void prep(const float (&)[kLaneCols], WoSums& xs) { xs.s[0] = xs.s[1] = 0.f; }
};

struct WoQ6K {
  static constexpr int kSlice = 2048;  // 8 blocks of 256
  static constexpr int kLaneCols = 64;
  using X = WoSums;  // per-lane state of x, prepared once per launch
  static constexpr int kUnroll = 4;
  static constexpr int kBlockBytes = 224;
  struct Raw {
    uint4 l0, l1, h;  // ql[64h+16j..], ql[64h+32+16j..], qh[32h+16j..]
    uint2 sc;         // scales [8h, 8h+8)
    uint16_t d;
  };
  // lane = 4*block + 2*half + j: values l = 16j+i (i < 16) of the half at
  // columns 128*half + l + {0, 32, 64, 96}
  __device__ static int col(int lane, int i) {
    const int b = lane >> 2, h = (lane >> 1) & 1, j = lane & 1;
    return 256 * b + 128 * h + 16 * j + 32 * (i / 16) + (i % 16);
  }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31, h = (lane >> 1) & 1, j = lane & 1;
    const uint8_t* blk = p.w + (long long)row * p.row_bytes + (long long)(c0 / 256 + (lane >> 2)) * kBlockBytes;
    r.l0 = __ldg(reinterpret_cast<const uint4*>(blk + 64 * h + 16 * j));
    r.l1 = __ldg(reinterpret_cast<const uint4*>(blk + 64 * h + 32 + 16 * j));
    r.h = __ldg(reinterpret_cast<const uint4*>(blk + 128 + 32 * h + 16 * j));
    r.sc = __ldg(reinterpret_cast<const uint2*>(blk + 192 + 8 * h));
    r.d = __ldg(reinterpret_cast<const uint16_t*>(blk + 208));
  }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const WoSums&) {
    const int j = threadIdx.x & 1;
    const uint32_t a[4] = {r.l0.x, r.l0.y, r.l0.z, r.l0.w};
    const uint32_t b[4] = {r.l1.x, r.l1.y, r.l1.z, r.l1.w};
    const uint32_t c[4] = {r.h.x, r.h.y, r.h.z, r.h.w};
    float2 s0 = make_float2(0.f, 0.f), s1 = s0, s2 = s0, s3 = s0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // four 6-bit values per byte lane: low/high nibbles of ql with bit pairs of qh (c:885-888)
      const uint32_t q0 = (a[k] & 0x0f0f0f0fu) | ((c[k] & 0x03030303u) << 4);
      const uint32_t q1 = (b[k] & 0x0f0f0f0fu) | (((c[k] >> 2) & 0x03030303u) << 4);
      const uint32_t q2 = ((a[k] >> 4) & 0x0f0f0f0fu) | (((c[k] >> 4) & 0x03030303u) << 4);
      const uint32_t q3 = ((b[k] >> 4) & 0x0f0f0f0fu) | (((c[k] >> 6) & 0x03030303u) << 4);
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        const int i = 4 * k + e;
        s0 = __ffma2_rn(byte_pair(q0, e, kTwo23 + 32.f), make_float2(x[i], x[i + 1]), s0);
        s1 = __ffma2_rn(byte_pair(q1, e, kTwo23 + 32.f), make_float2(x[16 + i], x[17 + i]), s1);
        s2 = __ffma2_rn(byte_pair(q2, e, kTwo23 + 32.f), make_float2(x[32 + i], x[33 + i]), s2);
        s3 = __ffma2_rn(byte_pair(q3, e, kTwo23 + 32.f), make_float2(x[48 + i], x[49 + i]), s3);
      }
    }
    const uint32_t sw[2] = {r.sc.x, r.sc.y};
    auto sc = [&](int k) { return (float)(int8_t)(sw[k / 4] >> (8 * (k % 4))); };
    return fp16_to_f32(r.d) * (sc(j) * (s0.x + s0.y) + sc(j + 2) * (s1.x + s1.y) + sc(j + 4) * (s2.x + s2.y) +
                               sc(j + 6) * (s3.x + s3.y));
  }
  __device__ static void prep(const float (&)[kLaneCols], WoSums& xs) { xs.s[0] = xs.s[1] = 0.f; }
};

// The types the reference multiplies with x quantised to Q8_0
// (matmul_quantized's q8 path, c:2102-2116): x is quantised per 32-value
// block exactly as quantize_row_q8_0 does (c:1508-1529, the cache quantiser's
// steps, so the same int8 values and fp16 scale), and every weight block
// gives an exact int32 sum of products, scaled as the reference does:
//   Q4_0   dw*dx*isum, q = nibble - 8                (c:1625-1643)
//   Q4_1   dw*dx*isum + mw*dx*xsum, q = nibble       (c:1646-1665)
//   Q5_0   dw*dx*isum, q = (nibble | qh bit << 4) - 16 (c:1668-1690)
//   Q5_1   dw*dx*isum + mw*dx*xsum, q = nibble | qh bit << 4 (c:1693-1717)
//   IQ4_NL dw*dx*isum, q = the format's table at the nibble (c:1994-2013)
// Lane l takes one block, columns [32l, 32l+32) of its slice.  Device layout:
// the quant bytes [dim][C/32][16], then per block 8 bytes [d, m, qh] in `wsc`
// ([dim][sc_stride]).
enum : int { kQxQ4_0, kQxQ4_1, kQxQ5_0, kQxQ5_1, kQxIQ4NL };

struct WoQ8xState {
  uint32_t q[8];  // the lane's 32 int8 values of x, packed
  float dx;       // their fp16 scale, as a float
  int xsum;       // their sum
};

// four 4-bit values t (bits 0..3) -> bit 0 of bytes 0..3
__device__ __forceinline__ uint32_t spread4(uint32_t t) { return (t * 0x00204081u) & 0x01010101u; }

// IQ4_NL's 16 values (the format's table, c:204-206)
constexpr int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
__host__ __device__ constexpr uint32_t iq4nl_word(int i) {
  return (uint32_t)(uint8_t)kIq4nl[i] | (uint32_t)(uint8_t)kIq4nl[i + 1] << 8 |
         (uint32_t)(uint8_t)kIq4nl[i + 2] << 16 | (uint32_t)(uint8_t)kIq4nl[i + 3] << 24;
}

// IQ4_NL: the table value of each byte of w (each 0..15), as signed bytes
__device__ __forceinline__ uint32_t iq4nl_lookup(uint32_t w) {
  // two permute tables of 8 entries
  constexpr uint32_t t0 = iq4nl_word(0), t1 = iq4nl_word(4), t2 = iq4nl_word(8), t3 = iq4nl_word(12);
  const uint32_t sel = (w & 7u) | ((w >> 4) & 0x70u) | ((w >> 8) & 0x700u) | ((w >> 12) & 0x7000u);
  const uint32_t lo = __byte_perm(t0, t1, sel), hi = __byte_perm(t2, t3, sel);
  const uint32_t m = ((w >> 3) & 0x01010101u) * 0xffu;  // bytes with bit 3 set take the high table
  return (lo & ~m) | (hi & m);
}

template <int T>
struct WoQ8x {
  static constexpr int kSlice = 1024;
  static constexpr int kLaneCols = 32;
  using X = WoQ8xState;
  static constexpr int kUnroll = 8;
  struct Raw {
    uint4 q;     // 16 quant bytes: byte j holds values j (low nibble) and j + 16 (high)
    uint2 meta;  // fp16 d | fp16 m << 16, qh
  };
  __device__ static int col(int lane, int i) { return 32 * lane + i; }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31;
    const long long b = c0 / 32 + lane;
    r.q = __ldg(reinterpret_cast<const uint4*>(p.w + (long long)row * p.row_bytes + b * 16));
    r.meta = __ldg(reinterpret_cast<const uint2*>(p.wsc + (long long)row * p.sc_stride + b * 8));
  }
  __device__ static void prep(const float (&x)[kLaneCols], X& xs) {
    xs.dx = fp16_to_f32(q8_quantize_lanes<32>(x, xs.q));
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) sum = __dp4a((int)xs.q[k], 0x01010101, sum);
    xs.xsum = sum;
  }
  __device__ static float dot(const Raw& r, const float (&)[kLaneCols], const X& xs) {
    const uint32_t q[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
    const uint32_t qh = r.meta.y;
    int isum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t lo = q[k] & 0x0f0f0f0fu, hi = (q[k] >> 4) & 0x0f0f0f0fu;  // values 4k.. and 16+4k..
      if constexpr (T == kQxQ5_0 || T == kQxQ5_1) {
        lo |= spread4((qh >> (4 * k)) & 15u) << 4;
        hi |= spread4((qh >> (16 + 4 * k)) & 15u) << 4;
      }
      if constexpr (T == kQxIQ4NL) {
        lo = iq4nl_lookup(lo);
        hi = iq4nl_lookup(hi);
      }
      isum = __dp4a((int)lo, (int)xs.q[k], isum);
      isum = __dp4a((int)hi, (int)xs.q[4 + k], isum);
    }
    if constexpr (T == kQxQ4_0) isum -= 8 * xs.xsum;
    if constexpr (T == kQxQ5_0) isum -= 16 * xs.xsum;
    const float dw = fp16_to_f32((uint16_t)(r.meta.x & 0xffffu));
    if constexpr (T == kQxQ4_1 || T == kQxQ5_1) {
      const float mw = fp16_to_f32((uint16_t)(r.meta.x >> 16));
      return dw * xs.dx * (float)isum + mw * xs.dx * (float)xs.xsum;
    } else {
      return dw * xs.dx * (float)isum;
    }
  }
};

// F32 / F16 / BF16 rows: fp32 products with x (vec_dot_f32 / vec_dot_f16 /
// vec_dot_bf16, c:1467-1494).  Lane l takes columns [32l, 32l+32) of its
// slice; device layout: the owned columns of each row as they are.
enum : int { kFlF32, kFlF16, kFlBF16 };

template <int T>
struct WoFloat {
  static constexpr int kSlice = 1024;
  static constexpr int kLaneCols = 32;
  using X = WoSums;
  static constexpr int kWords = T == kFlF32 ? 8 : 4;  // 16-byte loads per lane and row
  static constexpr int kUnroll = T == kFlF32 ? 2 : 4;
  struct Raw {
    uint4 v[kWords];
  };
  __device__ static int col(int lane, int i) { return 32 * lane + i; }
  __device__ static void load(const WoArgs& p, int row, int c0, Raw& r) {
    const int lane = threadIdx.x & 31;
    const uint4* s = reinterpret_cast<const uint4*>(p.w + (long long)row * p.row_bytes +
                                                   (long long)(c0 + 32 * lane) * (T == kFlF32 ? 4 : 2));
#pragma unroll
    for (int k = 0; k < kWords; ++k) r.v[k] = __ldg(s + k);
  }
  __device__ static void prep(const float (&)[kLaneCols], X& xs) { xs.s[0] = xs.s[1] = 0.f; }
  __device__ static float dot(const Raw& r, const float (&x)[kLaneCols], const X&) {
    float2 a = make_float2(0.f, 0.f), b = a;
#pragma unroll
    for (int k = 0; k < kWords; ++k) {
      const uint32_t w[4] = {r.v[k].x, r.v[k].y, r.v[k].z, r.v[k].w};
      if constexpr (T == kFlF32) {
        a = __ffma2_rn(make_float2(__uint_as_float(w[0]), __uint_as_float(w[1])), make_float2(x[4 * k], x[4 * k + 1]), a);
        b = __ffma2_rn(make_float2(__uint_as_float(w[2]), __uint_as_float(w[3])),
                       make_float2(x[4 * k + 2], x[4 * k + 3]), b);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 f;
          if constexpr (T == kFlF16) {
            f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          } else {
            f = make_float2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xffff0000u));
          }
          if (e % 2 == 0)
            a = __ffma2_rn(f, make_float2(x[8 * k + 2 * e], x[8 * k + 2 * e + 1]), a);
          else
            b = __ffma2_rn(f, make_float2(x[8 * k + 2 * e], x[8 * k + 2 * e + 1]), b);
        }
      }
    }
    return (a.x + a.y) + (b.x + b.y);
  }
};

// Tensor-parallel sum of the partial projections over NVLink, in the tail of
// the GEMV: an all-to-all of the partial rows, one NVLink crossing, spread
// over the CTAs.  The grid is the same on every member (same rows, kernel and
// GPU), so CTA j covers the same row block j everywhere.  Call e (1, 2, ...
// counted by the device step word, read after griddepcontrol.wait, when the
// previous call's grid has completed):
//   1. CTA j sends its partial rows to slot [e&1][member] of every member's
//      recv array (peer stores, its own included);
//   2. CTA j waits (bounded) for every member's rows of its block, sums them
//      in member order -- the same order, hence the same bits, on every
//      member -- and writes the sums to y;
//   3. the last CTA to leave (exit ticket) writes e into the step word.
// Every value travels as one 64-bit packet (float | e << 32), stored and
// loaded with relaxed system-scope 64-bit accesses, which cannot tear: a
// receiver that sees e in a packet has its value, so no fence, counter or flag
// orders anything (a system-scope fence after the peer stores measured ~4.6 us
// on B200).  Per call a member sends its dim partial rows to each of the
// n_members - 1 others, dim * 8 bytes each.  A reduce-scatter (partials to
// the block's owner) followed by an all-gather (sums from the owner) sends
// less but crosses NVLink twice: 8.8 against 7.6 us per call at two members.
// Two slots suffice: finishing call e needs every member's rows of call e,
// so no member sends call e + 2 (slot e&1) before every member has read
// call e.  A wait that gives up sets kErrTimeout; the group is then out of
// step and must be set up anew.

__device__ __forceinline__ void wo_tp_exchange(const WoArgs& p, const float* red, int r_begin, int r_end) {
  __shared__ unsigned s_e;
  const int n = r_end - r_begin;
  const int N = p.tp_members, me = p.tp_member;
  uint8_t* const mine = p.tp_regions[me];
  unsigned* const hdr = reinterpret_cast<unsigned*>(mine);
  if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile unsigned*>(hdr + kTpStepWord) + 1u;
  __syncthreads();
  const unsigned e = s_e;
  const long long par = e & 1u;
  // 1. this block's partial rows to every member
  for (int r = threadIdx.x; r < n; r += blockDim.x) {
    float s = 0.f;
    for (int c = 0; c < p.wc; ++c) s += red[c * p.rows_per_cta + r];
    for (int m = 0; m < N; ++m)
      ll_store(reinterpret_cast<unsigned long long*>(p.tp_regions[m] + kTpRecvOff) + (par * N + me) * p.rows +
                   r_begin + r,
               s, e);
  }
  trace_stamp(p.trace, 3);
  // 2. every member's rows of this block, summed in member order
  const unsigned long long* rv = reinterpret_cast<const unsigned long long*>(mine + kTpRecvOff) + par * N * p.rows;
  bool ok = true;
  for (int r = threadIdx.x; r < n && ok; r += blockDim.x) {
    float v[kXchgMaxParts];
    ok = ll_wait<kXchgMaxParts>(rv + r_begin + r, p.rows, N, e, v, p.err);
    if (!ok) break;
    float s = v[0];
#pragma unroll
    for (int m = 1; m < kXchgMaxParts; ++m)  // member order (unrolled: v stays in registers)
      if (m < N) s += v[m];
    p.y[r_begin + r] = s;
  }
  trace_stamp(p.trace, 4);
  // 3. the last CTA to leave advances the step (the next call reads it after
  // this grid has completed)
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(hdr + kTpTicketWord, 1u) == gridDim.x - 1) {
    hdr[kTpTicketWord] = 0u;
    *reinterpret_cast<volatile unsigned*>(hdr + kTpStepWord) = e;
  }
  trace_stamp(p.trace, 5);
}

// grid: ceil(rows / rows_per_cta) CTAs of NW warps; dynamic shared memory:
// NW * rows_per_cta floats.
template <class F, int NW>
__global__ void __launch_bounds__(NW * 32) wo_gemv_kernel(const WoArgs p) {
  extern __shared__ float red[];  // [wc][rows_per_cta]
  constexpr int U = F::kUnroll;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wcol = warp % p.wc, wrow = warp / p.wc, wr = NW / p.wc;
  const int r_begin = blockIdx.x * p.rows_per_cta;
  const int r_end = min(p.rows, r_begin + p.rows_per_cta);
  const int c0 = wcol * F::kSlice;                 // this warp's slice
  const bool active = c0 + F::col(lane, 0) < p.C;  // lanes past the owned columns idle
  const int n_my = r_end - r_begin > wrow ? (r_end - r_begin - wrow + wr - 1) / wr : 0;
  trace_stamp(p.trace, 0);

  // weights first: they do not depend on the kernel before this one
  pdl_launch_dependents();
  typename F::Raw raw[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (active && u < n_my) F::load(p, r_begin + wrow + wr * u, c0, raw[u]);
  pdl_wait();
  trace_stamp(p.trace, 1);
  float x[F::kLaneCols];
  typename F::X xs;
  // the lane's columns come in runs of 16 consecutive values (x = 0 past C)
#pragma unroll
  for (int i = 0; i < F::kLaneCols; i += 4) {
    const int c = c0 + F::col(lane, i);
    const float4 t = c < p.C ? __ldg(reinterpret_cast<const float4*>(p.x + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    x[i] = t.x;
    x[i + 1] = t.y;
    x[i + 2] = t.z;
    x[i + 3] = t.w;
  }
  F::prep(x, xs);

  for (int t0 = 0; t0 < n_my; t0 += U) {
    float acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = (active && t0 + u < n_my) ? F::dot(raw[u], x, xs) : 0.f;
    // the next rows' loads before the reductions
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (active && t0 + U + u < n_my) F::load(p, r_begin + wrow + wr * (t0 + U + u), c0, raw[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float v = acc[u];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0 && t0 + u < n_my) red[wcol * p.rows_per_cta + wrow + wr * (t0 + u)] = v;
    }
  }
  __syncthreads();
  trace_stamp(p.trace, 2);
  if (p.tp_members == 0) {
    for (int r = threadIdx.x; r < r_end - r_begin; r += blockDim.x) {
      float s = 0.f;
      for (int c = 0; c < p.wc; ++c) s += red[c * p.rows_per_cta + r];
      p.y[r_begin + r] = s;
    }
    return;
  }
  wo_tp_exchange(p, red, r_begin, r_end);
}

}  // namespace l3p
