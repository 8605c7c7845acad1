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
// One CTA = one q head x 128 query rows; keys in tiles of 128.  Every MMA is
// M=128 N=128 K=8: one tcgen05.mma costs the issuing thread ~44 cycles and the
// tensor core 64 cycles at N=128, so narrower MMAs would leave the tensor core
// waiting on the issuer.
//   warp 0       producer: 1-D bulk copies of pre-split K/V chunk images
//                (prefill_prep_kernel) into a 5-stage ring of 32 KB stages,
//                in the order the MMA issuer consumes them
//   warp 1       MMA issuer (one thread), per key tile j:
//                S_j = Q.K_j^T: 4 K chunks x 4 k-steps x 3 MMAs, Q hi from
//                tensor memory (TS form), Q lo from shared memory (SS form);
//                O += P_j.V_j: 4 V chunks (32 keys) x 4 k-steps x 3 MMAs, P
//                from tensor memory.  S_{j+1} is issued before P_j.V_j, so the
//                tensor core computes the next scores while the softmax
//                warps turn S_j into P_j.
//   warps 4..7   one query row per thread: Q hi into tensor memory and Q lo
//                into shared memory, online softmax on S, P in 32-key quarters
//                into a two-slot tensor-memory ring, lazy rescale of O (only
//                when the running max grows by more than 2^8), epilogue.
// Tensor memory (512 columns): Q hi [0,128) O [128,256) S [256,384)
// P slot 0 [384,448) P slot 1 [448,512) (each slot: 32 hi then 32 lo columns).
// Shared memory: Q lo image (64 KB) then the stage ring.
//   K chunk c (dims 32c..32c+31 of 128 keys): K-major, 128-byte swizzle,
//            hi 16 KB then lo 16 KB.
//   V chunk v (keys 32v..32v+31, all 128 dims): MN-major, 128-byte swizzle
//            with 32-byte units (the only MN-major layout the tensor cores
//            accept for 32-bit elements), four 32-dim atoms of eight 4-key
//            groups, hi 16 KB then lo 16 KB.
#pragma once
#include "ptx.cuh"
#include "tc.cuh"

namespace l3p {

constexpr int kPfBM = 128;  // query rows per CTA
constexpr int kPfBN = 128;  // keys per tile
constexpr int kPfHD = 128;  // head_dim of this kernel
constexpr int kPfChunkBytes = 32768;  // one K or V chunk image, hi + lo
constexpr int kPfChunkFloats = kPfChunkBytes / 4;
constexpr int kPfTileFloats = 8 * kPfChunkFloats;  // K chunks 0..3 then V chunks 0..3 of one key tile
constexpr int kPfStages = 5;
constexpr int kPfQloBytes = kPfBM * kPfHD * 4;
constexpr int kPfSmemBytes = kPfQloBytes + kPfStages * kPfChunkBytes + 1024;  // + alignment slack
constexpr float kPfRescale = 8.f;  // lazy rescale threshold (log2 units)
static_assert(kPfSmemBytes <= 232448, "prefill shared memory exceeds the per-CTA limit");

struct PrefillArgs {
  const float* q;    // [n_tok][n_heads][128], query token t at position q_pos0 + t
  float* out;        // same layout
  const float* img;  // [kvh_count][n_ktiles][kPfTileFloats] K/V chunk images (prefill_prep_kernel)
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

// The start-address field of a shared-memory descriptor holds addr >> 4 in
// 14 bits; shared addresses stay below 2^18, so byte offsets are added as
// offset >> 4 without carrying into the next field.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t byte_off) { return d + (byte_off >> 4); }

__global__ void __launch_bounds__(256, 1) prefill_tc_kernel(const PrefillArgs a) {
  extern __shared__ unsigned char pf_smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ __align__(8) uint64_t bar_kv_full[kPfStages], bar_kv_empty[kPfStages];
  __shared__ __align__(8) uint64_t bar_s_full, bar_s_free, bar_p_full[2], bar_p_free[2];
  __shared__ __align__(8) uint64_t bar_pv_done, bar_q_ready, bar_mma_idle;
  unsigned char* sbase = (unsigned char*)(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* qlo = sbase;
  unsigned char* ring = sbase + kPfQloBytes;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // heaviest query tiles first
  const int qt = a.n_qtiles - 1 - (int)blockIdx.x / a.n_qh;
  const int hq = (int)blockIdx.x % a.n_qh;
  const int h = a.kv_head_begin * a.G + hq;  // absolute q head
  const int kvh_local = hq / a.G;
  const int qbase = a.q_pos0 + qt * kPfBM;
  const int q_end = a.q_pos0 + a.n_tok;  // exclusive
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
    mbar_init(&bar_s_full, 1);
    mbar_init(&bar_s_free, 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_p_full[b], 4);
      mbar_init(&bar_p_free[b], 1);
    }
    mbar_init(&bar_pv_done, 1);
    mbar_init(&bar_q_ready, 4);
    mbar_init(&bar_mma_idle, 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = s_tmem;
  const uint32_t T_QHI = tm + 0, T_O = tm + 128, T_S = tm + 256, T_P = tm + 384;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const float* img = a.img + ((long long)kvh_local * a.n_ktiles + j0) * kPfTileFloats;
      int c = 0;  // chunks issued
      bool ok = true;
      // consumption order: K of tile 0; then per step n, K of tile n and V of tile n-1
      for (int n = 0; ok && n <= nt; ++n) {
        for (int part = 0; ok && part < 2; ++part) {
          const int t = n - part;
          if (t < 0 || t >= nt) continue;
          for (int ch = 0; ch < 4; ++ch, ++c) {
            const int s = c % kPfStages, u = c / kPfStages;
            if (u >= 1 && !mbar_wait_bounded(&bar_kv_empty[s], (uint32_t)((u - 1) & 1), a.err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bar_kv_full[s], (uint32_t)kPfChunkBytes);
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_addr(ring + s * kPfChunkBytes)),
                "l"(img + (long long)t * kPfTileFloats + (part * 4 + ch) * kPfChunkFloats),
                "r"((uint32_t)kPfChunkBytes), "r"(smem_addr(&bar_kv_full[s]))
                : "memory");
          }
        }
      }
      // no copy may still be landing when the CTA tears down
      for (int i = c > kPfStages ? c - kPfStages : 0; i < c; ++i)
        mbar_wait_bounded(&bar_kv_full[i % kPfStages], (uint32_t)((i / kPfStages) & 1), a.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t id_s = tc::idesc_tf32(kPfBM, kPfBN, false);
      constexpr uint32_t id_o = tc::idesc_tf32(kPfBM, kPfHD, true);
      const uint64_t qlo_d = tc::sdesc_sw128(smem_addr(qlo), 16, 1024);
      const uint64_t k_d = tc::sdesc_sw128(smem_addr(ring), 16, 1024);
      const uint64_t v_d = sdesc_mn_sw128_32b(smem_addr(ring));
      int c = 0;  // chunks consumed
      bool ok = mbar_wait_bounded(&bar_q_ready, 0, a.err);
      tc::fence_after_sync();
      auto next_chunk = [&](uint32_t& off) -> bool {
        const int s = c % kPfStages, u = c / kPfStages;
        off = (uint32_t)(s * kPfChunkBytes);
        if (!mbar_wait_bounded(&bar_kv_full[s], (uint32_t)(u & 1), a.err)) return false;
        tc::fence_after_sync();
        return true;
      };
      auto issue_s = [&]() -> bool {
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t off;
          if (!next_chunk(off)) return false;
          const uint64_t kh = desc_add(k_d, off), kl = desc_add(k_d, off + kPfChunkBytes / 2);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t a_col = T_QHI + ch * 32 + kk * 8;
            const uint64_t bh = desc_add(kh, kk * 32), bl = desc_add(kl, kk * 32);
            tc::mma_tf32_ts(T_S, a_col, bh, id_s, ch > 0 || kk > 0);
            tc::mma_tf32_ts(T_S, a_col, bl, id_s, true);
            tc::mma_tf32_ss(T_S, desc_add(qlo_d, ch * 16384 + kk * 32), bh, id_s, true);
          }
          tc::commit(&bar_kv_empty[c % kPfStages]);
          ++c;
        }
        tc::commit(&bar_s_full);
        return true;
      };
      auto issue_pv = [&](int jj) -> bool {
#pragma unroll 1
        for (int qq = 0; qq < 4; ++qq) {
          uint32_t off;
          if (!next_chunk(off)) return false;
          const int slot = qq & 1;
          if (!mbar_wait_bounded(&bar_p_full[slot], (uint32_t)((qq >> 1) & 1), a.err)) return false;
          tc::fence_after_sync();
          const uint64_t vh = desc_add(v_d, off), vl = desc_add(v_d, off + kPfChunkBytes / 2);
          const uint32_t p_hi = T_P + slot * 64, p_lo = p_hi + 32;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t bh = desc_add(vh, ks * 1024), bl = desc_add(vl, ks * 1024);
            tc::mma_tf32_ts(T_O, p_hi + ks * 8, bh, id_o, jj > 0 || qq > 0 || ks > 0);
            tc::mma_tf32_ts(T_O, p_hi + ks * 8, bl, id_o, true);
            tc::mma_tf32_ts(T_O, p_lo + ks * 8, bh, id_o, true);
          }
          tc::commit(&bar_kv_empty[c % kPfStages]);
          tc::commit(&bar_p_free[slot]);
          ++c;
        }
        tc::commit(&bar_pv_done);
        return true;
      };
      if (ok) ok = issue_s();
      for (int jj = 0; ok && jj < nt; ++jj) {
        if (jj + 1 < nt) {
          // S_{jj+1} overwrites S: the softmax warps must have read S_jj
          if (!mbar_wait_bounded(&bar_s_free, (uint32_t)(jj & 1), a.err)) break;
          tc::fence_after_sync();
          if (!issue_s()) break;
        }
        if (!issue_pv(jj)) break;
      }
      // every MMA of this CTA completes before tensor memory is released
      tc::commit(&bar_mma_idle);
      mbar_wait_bounded(&bar_mma_idle, 0, a.err);
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
      // Q lo: K-major 128-byte-swizzled image, 16 KB per 32 dims
      unsigned char* rp = qlo + c * 16384 + row * 128;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        *reinterpret_cast<float4*>(rp + ((i ^ (row & 7)) << 4)) =
            make_float4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
    }
    tc::wait_st();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // shared stores -> tensor-core reads
    tc::fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_q_ready);

    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < nt; ++jj) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar_s_full, (uint32_t)(jj & 1), a.err));
      if (!ok) break;
      tc::fence_after_sync();
      float sv[kPfBN];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tc::ld32(T_S + lb + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[c * 32 + i] = t[i];
      }
      tc::wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_s_free);
      const int key0 = (j0 + jj) * kPfBN;
      float mt = -INFINITY;
      if (__all_sync(0xffffffffu, valid && key0 >= kmin && key0 + kPfBN - 1 <= qpos)) {
#pragma unroll
        for (int c = 0; c < kPfBN; ++c) {
          sv[c] *= kLog2e;
          mt = fmaxf(mt, sv[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kPfBN; ++c) {
          const int key = key0 + c;
          const bool in = valid && key <= qpos && key >= kmin;
          sv[c] = in ? sv[c] * kLog2e : -INFINITY;
          mt = fmaxf(mt, sv[c]);
        }
      }
      if (jj >= 1) {
        // P_{jj-1}.V_{jj-1} complete: O is stable and both P slots are free
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar_pv_done, (uint32_t)((jj - 1) & 1), a.err));
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
      const float mneg = (m == -INFINITY) ? 0.f : -m;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        const int slot = qq & 1;
        if (qq >= 2) {
          // the slot's previous quarter (qq - 2) has been multiplied into O
          ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar_p_free[slot], 0u, a.err));
          if (!ok) break;
          tc::fence_after_sync();
        }
        float ph[32], pl[32];
        float lsum = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p = fast_exp2(sv[qq * 32 + c] + mneg);
          lsum += p;
          ph[c] = tc::tf32_hi(p);
          pl[c] = p - ph[c];
        }
        l += lsum;
        tc::st32(T_P + lb + slot * 64, ph);
        tc::st32(T_P + lb + slot * 64 + 32, pl);
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_p_full[slot]);
      }
      if (!ok) break;
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

// K/V chunk images for prefill_tc_kernel: per (owned KV head, 128-key tile),
// K chunks 0..3 then V chunks 0..3, each hi then lo, from the head-major
// cache.  Keys at or beyond n_keys read as 0.  grid (n_ktiles, kvh_count),
// 256 threads.
__global__ void prefill_prep_kernel(const float* __restrict__ kc, const float* __restrict__ vc, long long head_stride,
                                    int n_keys, int n_ktiles, float* __restrict__ img) {
  const int j = blockIdx.x, hl = blockIdx.y;
  unsigned char* base = reinterpret_cast<unsigned char*>(img + ((long long)hl * n_ktiles + j) * kPfTileFloats);
  constexpr int kHalf = kPfChunkBytes / 2;  // bytes of one hi (or lo) image
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
    const int atom = c16 >> 3, part = c16 & 7;  // 32-dim block, 16-byte piece within its 128 bytes
    // K chunk `atom`: K-major, 128-byte swizzle (16-byte piece ^ key % 8), 128 keys x 128 bytes
    const int kb = atom * kPfChunkBytes + key * 128 + ((part ^ (key & 7)) << 4);
    *reinterpret_cast<float4*>(base + kb) = khi;
    *reinterpret_cast<float4*>(base + kb + kHalf) = klo;
    // V chunk key/32: MN-major, 32-byte units ^ (key % 4), 32-dim atoms of eight 4-key groups
    const int kv = key & 31, byte = part * 16;
    const int vb = (4 + (key >> 5)) * kPfChunkBytes + atom * 4096 + (kv >> 2) * 512 + (kv & 3) * 128 +
                   ((((byte >> 5) ^ (kv & 3)) << 5) | (byte & 31));
    *reinterpret_cast<float4*>(base + vb) = vhi;
    *reinterpret_cast<float4*>(base + vb + kHalf) = vlo;
  }
}

}  // namespace l3p
