// prefill_tc.cuh -- causal prompt attention on the tcgen05 tensor cores in
// 3xTF32 (sm_100a), head_dim 128.
//
// Semantics are those of the reference's token-by-token prefill
// (llama3pure-c-engine.c:3499-3613): query token at position p attends to the
// cached positions [start_t(p), p] (start_t from the SWA rule, c:3574-3580)
// with softmax(q.K^T * scale) . V.  The cache rows of the batch are appended
// before this kernel runs.
//
// 3xTF32: every fp32 operand x is split into hi = x with the low 13 mantissa
// bits cleared (exact in tf32) and lo = x - hi (exact in fp32); products are
// hi*hi + hi*lo + lo*hi, accumulated in fp32 in tensor memory.  The dropped
// lo*lo term and the tf32 rounding of lo are ~2^-21 relative.
//
// One CTA = one q head x 128 query rows; keys in tiles of 32.
//   warp 0       producer: 1-D bulk copies of pre-split K/V tile images
//                (prefill_prep_kernel) into a 3-stage shared-memory ring
//   warp 1       MMA issuer (one thread): S = Q.K^T (48 MMAs, M=128 N=32 K=8)
//                and O += P.V (12 MMAs, M=128 N=128 K=8) per key tile
//   warps 4..7   one query row per thread: Q into tensor memory, online
//                softmax on S, P into tensor memory, lazy rescale of O (only
//                when the running max grows by more than 2^8), epilogue
// Tensor memory (512 columns): Q hi [0,128) Q lo [128,256) S0 [256,288)
// S1 [288,320) P hi [320,352) P lo [352,384) O [384,512).
// Shared memory per stage: K hi | K lo | V hi | V lo, 16 KB each.
//   K image: K-major, 128-byte swizzle, 32 keys x 128 dims, four 32-dim atoms.
//   V image: MN-major, 128-byte swizzle with 32-byte units (the only MN-major
//            layout the tensor cores accept for 32-bit elements), four
//            32-dim atoms of eight 4-key groups.
#pragma once
#include "ptx.cuh"
#include "tc.cuh"

namespace l3p {

constexpr int kPfBM = 128;       // query rows per CTA
constexpr int kPfBN = 32;        // keys per tile
constexpr int kPfHD = 128;       // head_dim of this kernel
constexpr int kPfStages = 3;
constexpr int kPfImgFloats = 2 * kPfBN * kPfHD;  // hi + lo image of one K (or V) tile
constexpr int kPfStageBytes = 2 * kPfImgFloats * 4;
constexpr int kPfSmemBytes = kPfStages * kPfStageBytes + 1024;  // + alignment slack
constexpr float kPfRescale = 8.f;  // lazy rescale threshold (log2 units)

struct PrefillArgs {
  const float* q;       // [n_tok][n_heads][128], query token t at position q_pos0 + t
  float* out;           // same layout
  const float* kimg;    // [kvh_count][n_ktiles][2][32*128] K tile images (hi, lo)
  const float* vimg;    // same for V
  int n_heads, G, kv_head_begin, n_qh;  // owned q heads = n_qh, absolute first = kv_head_begin*G
  int q_pos0, n_tok, n_qtiles, n_ktiles;
  float scale;
  int layer, is_gemma3, swa_window, swa_pattern;
  int* err;
};

__device__ __forceinline__ int pf_start_t(const PrefillArgs& a, int pos) {
  if (a.is_gemma3 && a.swa_window > 0 && a.swa_pattern > 0 && (a.layer % a.swa_pattern) < a.swa_pattern - 1) {
    const int s = pos - a.swa_window + 1;
    return s < 0 ? 0 : s;
  }
  return 0;
}

__device__ __forceinline__ uint64_t sdesc_mn_sw128_32b(uint32_t addr) {
  // MN-major, 32-byte-unit 128-byte swizzle: next 32-dim atom at +4096 (LBO),
  // next 4-key group at +512 (SBO), layout type 1
  uint64_t d = tc::sdesc_sw128(addr, 4096, 512);
  d &= ~((uint64_t)7 << 61);
  d |= (uint64_t)1 << 61;
  return d;
}

__global__ void __launch_bounds__(256, 1) prefill_tc_kernel(const PrefillArgs a) {
  extern __shared__ unsigned char pf_smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ __align__(8) uint64_t bar_kv_full[kPfStages], bar_kv_empty[kPfStages];
  __shared__ __align__(8) uint64_t bar_s_full[2], bar_s_free[2];
  __shared__ __align__(8) uint64_t bar_p_full, bar_pv_done, bar_q_ready;
  unsigned char* sbase = (unsigned char*)(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // heaviest query tiles first
  const int qt = a.n_qtiles - 1 - (int)blockIdx.x / a.n_qh;
  const int hq = (int)blockIdx.x % a.n_qh;
  const int h = a.kv_head_begin * a.G + hq;  // absolute q head
  const int kvh_local = hq / a.G;
  const int qbase = a.q_pos0 + qt * kPfBM;
  const int q_end = a.q_pos0 + a.n_tok;     // exclusive
  const int k_hi = min(qbase + kPfBM, q_end) - 1;
  const int j0 = pf_start_t(a, qbase) / kPfBN;
  const int j1 = k_hi / kPfBN;
  const int nt = j1 - j0 + 1;

  if (warp == 0) {
    tc::tmem_alloc(&s_tmem, 512);
    tc::tmem_relinquish();
  }
  if (tid == 32) {
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_s_full[b], 1);
      mbar_init(&bar_s_free[b], 4);
    }
    mbar_init(&bar_p_full, 4);
    mbar_init(&bar_pv_done, 1);
    mbar_init(&bar_q_ready, 4);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = s_tmem;
  const uint32_t T_QHI = tm + 0, T_QLO = tm + 128, T_S = tm + 256, T_PHI = tm + 320, T_PLO = tm + 352,
                 T_O = tm + 384;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const float* kimg = a.kimg + ((long long)kvh_local * a.n_ktiles) * kPfImgFloats;
      const float* vimg = a.vimg + ((long long)kvh_local * a.n_ktiles) * kPfImgFloats;
      for (int jj = 0; jj < nt; ++jj) {
        const int s = jj % kPfStages, u = jj / kPfStages;
        if (u >= 1 && !mbar_wait_bounded(&bar_kv_empty[s], (uint32_t)((u - 1) & 1), a.err)) break;
        unsigned char* st = sbase + s * kPfStageBytes;
        const long long tile = j0 + jj;
        mbar_arrive_expect_tx(&bar_kv_full[s], (uint32_t)kPfStageBytes);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_addr(st)),
            "l"(kimg + tile * kPfImgFloats), "r"((uint32_t)(kPfImgFloats * 4)), "r"(smem_addr(&bar_kv_full[s]))
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_addr(st + kPfImgFloats * 4)),
            "l"(vimg + tile * kPfImgFloats), "r"((uint32_t)(kPfImgFloats * 4)), "r"(smem_addr(&bar_kv_full[s]))
            : "memory");
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_tf32(kPfBM, kPfBN, false);
      const uint32_t id_o = tc::idesc_tf32(kPfBM, kPfHD, true);
      bool ok = mbar_wait_bounded(&bar_q_ready, 0, a.err);
      tc::fence_after_sync();
      auto issue_s = [&](int jj) -> bool {
        const int s = jj % kPfStages, u = jj / kPfStages, b = jj & 1;
        if (!mbar_wait_bounded(&bar_kv_full[s], (uint32_t)(u & 1), a.err)) return false;
        if (jj >= 2 && !mbar_wait_bounded(&bar_s_free[b], (uint32_t)(((jj - 2) >> 1) & 1), a.err)) return false;
        tc::fence_after_sync();
        const uint32_t kh = smem_addr(sbase + s * kPfStageBytes), kl = kh + kPfImgFloats * 2;
        const uint32_t dst = T_S + b * kPfBN;
#pragma unroll
        for (int kk = 0; kk < kPfHD / 8; ++kk) {
          const uint32_t off = (kk >> 2) * 4096 + (kk & 3) * 32;
          const uint64_t dh = tc::sdesc_sw128(kh + off, 16, 1024);
          const uint64_t dl = tc::sdesc_sw128(kl + off, 16, 1024);
          tc::mma_tf32_ts(dst, T_QHI + kk * 8, dh, id_s, kk > 0);
          tc::mma_tf32_ts(dst, T_QHI + kk * 8, dl, id_s, true);
          tc::mma_tf32_ts(dst, T_QLO + kk * 8, dh, id_s, true);
        }
        tc::commit(&bar_s_full[b]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int jj = 0; ok && jj < nt; ++jj) {
        if (jj + 1 < nt && !issue_s(jj + 1)) break;
        if (!mbar_wait_bounded(&bar_p_full, (uint32_t)(jj & 1), a.err)) break;
        tc::fence_after_sync();
        const int s = jj % kPfStages;
        const uint32_t vh = smem_addr(sbase + s * kPfStageBytes + kPfImgFloats * 4), vl = vh + kPfImgFloats * 2;
#pragma unroll
        for (int ks = 0; ks < kPfBN / 8; ++ks) {
          const uint64_t dh = sdesc_mn_sw128_32b(vh + ks * 1024);
          const uint64_t dl = sdesc_mn_sw128_32b(vl + ks * 1024);
          tc::mma_tf32_ts(T_O, T_PHI + ks * 8, dh, id_o, jj > 0 || ks > 0);
          tc::mma_tf32_ts(T_O, T_PHI + ks * 8, dl, id_o, true);
          tc::mma_tf32_ts(T_O, T_PLO + ks * 8, dh, id_o, true);
        }
        tc::commit(&bar_pv_done);
        tc::commit(&bar_kv_empty[s]);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax warpgroup: thread = query row ----------------
    const int row = (warp - 4) * 32 + lane;
    const int qpos = qbase + row;
    const bool valid = qpos < q_end;
    const int kmin = valid ? pf_start_t(a, qpos) : 0;
    const uint32_t lb = (uint32_t)((warp - 4) * 32) << 16;
    const float* qrow = a.q + ((long long)(qpos - a.q_pos0) * a.n_heads + h) * kPfHD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float hi[32], lo[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 t = valid ? *reinterpret_cast<const float4*>(qrow + c * 32 + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float x[4] = {t.x * a.scale, t.y * a.scale, t.z * a.scale, t.w * a.scale};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hi[4 * i + e] = tc::tf32_hi(x[e]);
          lo[4 * i + e] = x[e] - hi[4 * i + e];
        }
      }
      tc::st32(T_QHI + lb + c * 32, hi);
      tc::st32(T_QLO + lb + c * 32, lo);
    }
    tc::wait_st();
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_q_ready);

    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < nt; ++jj) {
      const int b = jj & 1;
      ok = mbar_wait_bounded(&bar_s_full[b], (uint32_t)((jj >> 1) & 1), a.err);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc::fence_after_sync();
      float sv[32];
      tc::ld32(T_S + lb + b * kPfBN, sv);
      tc::wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_s_free[b]);
      const int key0 = (j0 + jj) * kPfBN;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int key = key0 + c;
        const bool in = valid && key <= qpos && key >= kmin;
        sv[c] = in ? sv[c] * kLog2e : -INFINITY;
        mt = fmaxf(mt, sv[c]);
      }
      if (jj >= 1) {
        ok = mbar_wait_bounded(&bar_pv_done, (uint32_t)((jj - 1) & 1), a.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc::fence_after_sync();
      }
      const float m_new = fmaxf(m, mt);
      const bool grow = m_new > m + kPfRescale;  // true on the first finite score (m = -inf)
      float alpha = 1.f;
      if (grow) {
        alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      if (jj >= 1 && __any_sync(0xffffffffu, grow)) {
        // rescale O (warp-wide tensor-memory access; rows that keep their max use 1)
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tc::ld32(T_O + lb + c * 32, ov);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tc::st32(T_O + lb + c * 32, ov);
        }
      }
      float ph[32], pl[32];
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p = (m == -INFINITY) ? 0.f : fast_exp2(sv[c] - m);
        lsum += p;
        ph[c] = tc::tf32_hi(p);
        pl[c] = p - ph[c];
      }
      l += lsum;
      tc::st32(T_PHI + lb, ph);
      tc::st32(T_PLO + lb, pl);
      tc::wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p_full);
    }
    // ---------------- epilogue ----------------
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar_pv_done, (uint32_t)((nt - 1) & 1), a.err));
    if (ok) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float* orow = a.out + ((long long)(qpos - a.q_pos0) * a.n_heads + h) * kPfHD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tc::ld32(T_O + lb + c * 32, ov);
        tc::wait_ld();
        if (valid) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(orow + c * 32 + 4 * i) =
                make_float4(ov[4 * i] * inv, ov[4 * i + 1] * inv, ov[4 * i + 2] * inv, ov[4 * i + 3] * inv);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tm, 512);
  }
}

// K/V tile images for prefill_tc_kernel: per (owned KV head, 32-key tile),
// hi then lo, from the head-major cache.  Keys at or beyond n_keys read as 0.
// grid (n_ktiles, kvh_count), 256 threads.
__global__ void prefill_prep_kernel(const float* __restrict__ kc, const float* __restrict__ vc, long long head_stride,
                                    int n_keys, int n_ktiles, float* __restrict__ kimg, float* __restrict__ vimg) {
  const int j = blockIdx.x, hl = blockIdx.y;
  const long long img = ((long long)hl * n_ktiles + j) * kPfImgFloats;
  unsigned char* kh = reinterpret_cast<unsigned char*>(kimg + img);
  unsigned char* vh = reinterpret_cast<unsigned char*>(vimg + img);
  const int lo_off = kPfBN * kPfHD * 4;  // bytes of one hi image
  for (int idx = threadIdx.x; idx < kPfBN * kPfHD / 4; idx += blockDim.x) {
    const int key = idx / (kPfHD / 4), c16 = idx % (kPfHD / 4);  // 16-byte chunk of the row
    const int pos = j * kPfBN + key;
    float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
    if (pos < n_keys) {
      kx = *reinterpret_cast<const float4*>(kc + hl * head_stride + (long long)pos * kPfHD + 4 * c16);
      vx = *reinterpret_cast<const float4*>(vc + hl * head_stride + (long long)pos * kPfHD + 4 * c16);
    }
    const float4 khi = make_float4(tc::tf32_hi(kx.x), tc::tf32_hi(kx.y), tc::tf32_hi(kx.z), tc::tf32_hi(kx.w));
    const float4 klo = make_float4(kx.x - khi.x, kx.y - khi.y, kx.z - khi.z, kx.w - khi.w);
    const float4 vhi = make_float4(tc::tf32_hi(vx.x), tc::tf32_hi(vx.y), tc::tf32_hi(vx.z), tc::tf32_hi(vx.w));
    const float4 vlo = make_float4(vx.x - vhi.x, vx.y - vhi.y, vx.z - vhi.z, vx.w - vhi.w);
    // K: K-major, 128-byte swizzle (16-byte chunk ^ key % 8), 32-dim atoms of 4 KB
    const int katom = c16 >> 3, kchunk = c16 & 7;
    const int kb = katom * 4096 + key * 128 + ((kchunk ^ (key & 7)) << 4);
    *reinterpret_cast<float4*>(kh + kb) = khi;
    *reinterpret_cast<float4*>(kh + lo_off + kb) = klo;
    // V: MN-major, 32-byte units ^ (key % 4), 32-dim atoms of eight 4-key groups
    const int byte = (c16 & 7) * 16;
    const int vb = katom * 4096 + (key >> 2) * 512 + (key & 3) * 128 + ((((byte >> 5) ^ (key & 3)) << 5) | (byte & 31));
    *reinterpret_cast<float4*>(vh + vb) = vhi;
    *reinterpret_cast<float4*>(vh + lo_off + vb) = vlo;
  }
}

}  // namespace l3p
