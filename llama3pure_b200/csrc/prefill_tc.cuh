// prefill_tc.cuh -- causal prompt attention on the tcgen05 tensor cores in
// 3xTF32 (sm_100a), head_dim 64 or 128.
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
// One CTA = one q head x 128 query rows; keys in tiles of 128.  Every MMA has
// N=128, K=8: one tcgen05.mma costs the issuing thread ~44 cycles and the
// tensor core 64 cycles per 128 rows at N=128, so narrower MMAs would leave
// the tensor core waiting on the issuer.
//
// CG = 2 (GQA groups of even size): the CTAs of a 2-CTA cluster take two q
// heads of the same KV head and the same query rows, and every MMA is
// cta_group::2 with M = 256 issued by the even CTA.  Each CTA stages only half
// of every K/V chunk (the B operand is split by columns across the pair), so a
// CTA streams half the bytes per flop: at M = 128 the stream needs ~42
// bytes/cycle/SM from L2, more than a ring of 1-D bulk copies (~4.5K cycles
// latency under this load) delivers.  CG = 1 is the single-CTA form.
//
// Roles (256 threads per CTA):
//   warps 0,2,3  producers (one thread each, chunks in turn): 1-D bulk
//                copies of this CTA's half of the pre-split K/V chunk images
//                (prefill_prep_kernel) into a ring of kStages stages, in the
//                order the MMA issuer consumes them
//   warp 1       even CTA: MMA issuer (one thread), per key tile j:
//                  S_j = Q.K_j^T: 4 K chunks x 4 k-steps x 3 MMAs, Q hi from
//                  tensor memory (TS form), Q lo from shared memory (SS form);
//                  O += P_j.V_j: 4 V chunks (32 keys) x 4 k-steps x 3 MMAs,
//                  P from tensor memory.  S_{j+1} is issued before P_j.V_j,
//                  so the tensor core computes the next scores while the
//                  softmax warps turn S_j into P_j.
//                odd CTA: relays each landed chunk to the even CTA's issuer
//   warps 4..7   one query row per thread: Q hi into tensor memory and Q lo
//                into shared memory, online softmax on S, P in 32-key quarters
//                into a two-slot tensor-memory ring (a quarter waits only for
//                its slot's previous quarter to be multiplied in), lazy
//                rescale of O (only when the running max grows by more than
//                2^8; only then does a warp wait for every P.V MMA issued so
//                far), epilogue through shared memory with whole-row global
//                stores.
// Barriers the issuers wait on (kv_peer, s_free, p_full, q_ready) live in the
// even CTA and count arrivals from both CTAs; barriers the issuers complete
// (kv_empty, s_full, p_free, pv_done) get one commit per CTA of the pair.
// Tensor memory (512 columns per CTA): Q hi [0,HD) O [HD,2HD) S [2HD,2HD+128)
// P slot 0 and slot 1, 64 columns each, after S (each slot: 32 hi then 32 lo
// columns).  Head_dim 256 does not fit: Q hi and O alone would take all 512
// columns.
// Shared memory: Q lo image (128 rows x HD x 4 bytes) then the stage ring.
// A key tile is HD/32 K chunks then 4 V chunks:
//   K chunk c (dims 32c..32c+31), this CTA's 128/CG keys: K-major, 128-byte
//            swizzle, hi then lo (32 KB for both CTAs of a pair).
//   V chunk v (keys 32v..32v+31), this CTA's HD/CG dims: MN-major, 128-byte
//            swizzle with 32-byte units (the only MN-major layout the tensor
//            cores accept for 32-bit elements), 32-dim atoms of eight 4-key
//            groups, hi then lo (32 * HD * 8 bytes for both CTAs).
// A stage holds the largest chunk; a V chunk of head_dim 64 fills half of one.
// CTA pairs (CG = 2) are built for head_dim 128 only.
#pragma once
#include "decode_q8.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace l3p {

constexpr int kPfBM = 128;  // query rows per CTA
constexpr int kPfBN = 128;  // keys per tile
constexpr int kPfKChunkBytes = 32768;  // one K chunk image (128 keys x 32 dims), hi + lo, both CTAs' halves
constexpr float kPfRescale = 8.f;  // lazy rescale threshold (log2 units)
constexpr int kProducers = 2;      // producer threads (warps 0, 2)

// Key-tile geometry of one head size.
template <int HD>
struct PfGeom {
  static_assert(HD == 64 || HD == 128, "tensor-core prefill: head_dim 64 or 128");
  static constexpr int kKChunks = HD / 32;          // K chunks per key tile (32 dims each)
  static constexpr int kVChunks = kPfBN / 32;       // V chunks per key tile (32 keys each)
  static constexpr int kChunks = kKChunks + kVChunks;
  static constexpr int kVChunkBytes = 32 * HD * 8;  // 32 keys x HD dims, hi + lo
  static constexpr int kTileBytes = kKChunks * kPfKChunkBytes + kVChunks * kVChunkBytes;
  static constexpr int kTileFloats = kTileBytes / 4;
  static constexpr int kQloBytes = kPfBM * HD * 4;
};

template <int CG, int HD>
struct PfCfg {
  static_assert(CG == 1 || HD == 128, "CTA pairs are built for head_dim 128");
  static constexpr int kStageBytes = kPfKChunkBytes / CG;  // this CTA's share of the largest chunk image
  static constexpr int kStageFloats = kStageBytes / 4;
  static constexpr int kKBytes = kPfKChunkBytes / CG;           // this CTA's K chunk
  static constexpr int kVBytes = PfGeom<HD>::kVChunkBytes / CG;  // this CTA's V chunk
  static constexpr int kHalfTile = PfGeom<HD>::kTileBytes / CG;  // this CTA's chunks of a key tile
  static constexpr int kStages = HD == 64 ? 6 : 5 * CG;
  static constexpr int kRows = 128 / CG;  // B rows per CTA: keys of a K chunk
  static constexpr int kSmemBytes = PfGeom<HD>::kQloBytes + kStages * kStageBytes + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 232448, "prefill shared memory exceeds the per-CTA limit");
};

struct PrefillArgs {
  const float* q;    // [n_tok][n_heads][head_dim], query token t at position q_pos0 + t
  float* out;        // same layout
  const float* img;  // [kvh_count][n_ktiles][PfGeom<HD>::kTileFloats] K/V chunk images (prefill_prep_kernel)
  int n_heads, G, kv_head_begin, n_qh;  // owned q heads = n_qh, absolute first = kv_head_begin*G
  int q_pos0, n_tok, n_qtiles, n_ktiles;
  float scale;
  int layer, is_gemma3, swa_window, swa_pattern;
  int q8;  // Q8_0 cache: q is quantised to Q8_0 per 32-value block and back (c:3569-3570)
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

template <int CG, int HD>
__global__ void __launch_bounds__(256, 1) prefill_tc_kernel(const PrefillArgs a) {
  using C = PfCfg<CG, HD>;
  using Gm = PfGeom<HD>;
  constexpr int S = C::kStages;
  constexpr int kPieces = HD / 4;         // 16-byte pieces of a q / out row
  constexpr int kRowsPerLoad = 128 / HD;  // rows one warp-wide 512-byte access covers
  constexpr int kQLoads = HD / 4;         // such accesses for a warp's 32 rows
  extern __shared__ unsigned char pf_smem_raw[];
  __shared__ uint32_t s_tmem;
  __shared__ __align__(8) uint64_t bar_kv_full[S], bar_kv_empty[S], bar_kv_peer[S];
  __shared__ __align__(8) uint64_t bar_s_full, bar_s_free, bar_p_full[2], bar_p_free[2];
  __shared__ __align__(8) uint64_t bar_pv_done, bar_q_ready, bar_mma_idle[2];
  unsigned char* sbase = (unsigned char*)(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* qlo = sbase;
  unsigned char* ring = sbase + Gm::kQloBytes;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0;
  // heaviest query tiles first; CG = 2: a cluster takes q heads 2p and 2p + 1
  const int unit = (int)blockIdx.x / CG;
  const int units_per_qt = a.n_qh / CG;
  const int qt = a.n_qtiles - 1 - unit / units_per_qt;
  const int hq = (unit % units_per_qt) * CG + (int)rank;
  const int h = a.kv_head_begin * a.G + hq;  // absolute q head
  const int kvh_local = hq / a.G;
  const int qbase = a.q_pos0 + qt * kPfBM;
  const int q_end = a.q_pos0 + a.n_tok;  // exclusive
  const int k_hi = min(qbase + kPfBM, q_end) - 1;
  const int j0 = pf_start_t(a, qbase) / kPfBN;
  const int j1 = k_hi / kPfBN;
  const int nt = j1 - j0 + 1;

  // The softmax warps fetch their Q rows before the setup barrier so the
  // latency overlaps the allocation: each warp its 32 rows, 512 contiguous
  // bytes per load (1 row of head_dim 128 or 2 rows of 64; lane = 16-byte
  // piece), all in flight at once.  Rows past the batch read the last row and
  // are zeroed later, so no load result is needed before the barrier.
  float4 qv[kQLoads];
  if (warp >= 4) {
#pragma unroll
    for (int r = 0; r < kQLoads; ++r) {
      const int rr = r * kRowsPerLoad + lane / kPieces;
      const int qpos = min(qbase + (warp - 4) * 32 + rr, q_end - 1);
      qv[r] = __ldg(reinterpret_cast<const float4*>(a.q + ((long long)(qpos - a.q_pos0) * a.n_heads + h) * HD) +
                    lane % kPieces);
    }
  }
  if (warp == 0) {
    tc::tmem_alloc_g<CG>(&s_tmem, 512);
    tc::tmem_relinquish_g<CG>();
  }
  if (tid == 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
      mbar_init(&bar_kv_peer[s], 1);
    }
    mbar_init(&bar_s_full, 1);
    mbar_init(&bar_s_free, 4 * CG);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_p_full[b], 4 * CG);
      mbar_init(&bar_p_free[b], 1);
    }
    mbar_init(&bar_pv_done, 1);
    mbar_init(&bar_q_ready, 4 * CG);
    mbar_init(&bar_mma_idle[0], 1);
    mbar_init(&bar_mma_idle[1], 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  if constexpr (CG == 2)
    cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  else
    __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = s_tmem;
  const uint32_t T_QHI = tm + 0, T_O = tm + HD, T_S = tm + 2 * HD, T_P = tm + 2 * HD + kPfBN;

  // bounded waits: cluster-scope acquire when the pair shares the barriers
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if constexpr (CG == 2)
      return mbar_wait_bounded_cluster(bar, parity, a.err);
    else
      return mbar_wait_bounded(bar, parity, a.err);
  };
  // arrive on a barrier of the issuing (even) CTA
  auto arrive_issuer = [&](uint64_t* bar) {
    if constexpr (CG == 2)
      mbar_arrive_cluster(mapa_shared(smem_addr(bar), 0));
    else
      mbar_arrive(bar);
  };
  // complete a barrier in every CTA of the pair once the MMAs issued so far are done
  auto commit_all = [&](uint64_t* bar) {
    tc::commit_g<CG>(smem_addr(bar));
    if constexpr (CG == 2) tc::commit_g<CG>(mapa_shared(smem_addr(bar), 1));
  };

  if (warp == 0 || warp == 2) {
    // ---------------- producers ----------------
    // Two threads in different warps issue chunks in turn: the bulk copies of
    // one thread complete one after another, so one thread alone cannot keep
    // the ring full.
    if (lane == 0) {
      const int me = warp >> 1;  // chunks c with c % kProducers == me
      const unsigned char* img = reinterpret_cast<const unsigned char*>(a.img) +
                                 ((long long)kvh_local * a.n_ktiles + j0) * Gm::kTileBytes + rank * C::kHalfTile;
      int c = 0;  // chunks enumerated
      bool ok = true;
      // consumption order: K of tile 0; then per step n, K of tile n and V of tile n-1
      for (int n = 0; ok && n <= nt; ++n) {
        for (int part = 0; ok && part < 2; ++part) {
          const int t = n - part;
          if (t < 0 || t >= nt) continue;
          const int n_ch = part == 0 ? Gm::kKChunks : Gm::kVChunks;
          for (int ch = 0; ch < n_ch; ++ch, ++c) {
            if (c % kProducers != me) continue;
            const int s = c % S, u = c / S;
            if (u >= 1 && !wait(&bar_kv_empty[s], (uint32_t)((u - 1) & 1))) {
              ok = false;
              break;
            }
            const uint32_t bytes = part == 0 ? C::kKBytes : C::kVBytes;
            const long long off = part == 0 ? (long long)ch * C::kKBytes
                                            : (long long)Gm::kKChunks * C::kKBytes + (long long)ch * C::kVBytes;
            mbar_arrive_expect_tx(&bar_kv_full[s], bytes);
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_addr(ring + s * C::kStageBytes)),
                "l"(img + (long long)t * Gm::kTileBytes + off), "r"(bytes), "r"(smem_addr(&bar_kv_full[s]))
                : "memory");
          }
        }
      }
      // no copy of this thread may still be landing when the CTA tears down
      for (int i = c > S ? c - S : 0; i < c; ++i)
        if (i % kProducers == me) wait(&bar_kv_full[i % S], (uint32_t)((i / S) & 1));
    }
  } else if (warp == 1 && rank == 1) {
    // ---------------- relay (odd CTA): chunk landed here -> issuer ----------------
    if (lane == 0) {
      for (int c = 0; c < Gm::kChunks * nt; ++c) {
        if (!wait(&bar_kv_full[c % S], (uint32_t)((c / S) & 1))) break;
        mbar_arrive_cluster(mapa_shared(smem_addr(&bar_kv_peer[c % S]), 0));
      }
    }
  } else if ((warp == 1 || warp == 3) && rank == 0) {
    // ---------------- MMA issuers ----------------
    // warp 1 issues S = Q.K^T, warp 3 issues O += P.V.  One thread pays ~44
    // cycles per tcgen05.mma and more per commit or barrier wait, while the
    // tensor core takes 64 cycles per N=128 MMA: a single issuer leaves it
    // idle, two issuers in different warps keep it busy.
    if (lane == 0) {
      // first chunk of each block in the ring sequence K0 K1 V0 K2 V1 ... V(nt-1)
      // (a K block holds HD/32 chunks, a V block 4)
      constexpr int nK = Gm::kKChunks, nKV = Gm::kChunks;
      auto k_chunk0 = [&](int t) { return t == 0 ? 0 : nK + (t - 1) * nKV; };
      auto v_chunk0 = [&](int t) { return t + 1 < nt ? 2 * nK + t * nKV : nK + t * nKV; };
      auto chunk_ready = [&](int c, uint32_t& off) -> bool {
        const int s = c % S, u = c / S;
        off = (uint32_t)(s * C::kStageBytes);
        if (!wait(&bar_kv_full[s], (uint32_t)(u & 1))) return false;
        if (CG == 2 && !wait(&bar_kv_peer[s], (uint32_t)(u & 1))) return false;
        tc::fence_after_sync();
        return true;
      };
      if (warp == 1) {
        constexpr uint32_t id_s = tc::idesc_tf32(kPfBM * CG, kPfBN, false);
        const uint64_t qlo_d = tc::sdesc_sw128(smem_addr(qlo), 16, 1024);
        const uint64_t k_d = tc::sdesc_sw128(smem_addr(ring), 16, 1024);
        bool ok = wait(&bar_q_ready, 0);
        tc::fence_after_sync();
        for (int t = 0; ok && t < nt; ++t) {
          if (t >= 1) {
            // S_t overwrites S: the softmax warps must have read S_{t-1}
            if (!wait(&bar_s_free, (uint32_t)((t - 1) & 1))) break;
            tc::fence_after_sync();
          }
#pragma unroll 1
          for (int ch = 0; ok && ch < nK; ++ch) {
            const int c = k_chunk0(t) + ch;
            uint32_t off;
            if (!(ok = chunk_ready(c, off))) break;
            const uint64_t kh = desc_add(k_d, off), kl = desc_add(k_d, off + C::kStageBytes / 2);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t a_col = T_QHI + ch * 32 + kk * 8;
              const uint64_t bh = desc_add(kh, kk * 32), bl = desc_add(kl, kk * 32);
              tc::mma_tf32_ts_g<CG>(T_S, a_col, bh, id_s, ch > 0 || kk > 0);
              tc::mma_tf32_ts_g<CG>(T_S, a_col, bl, id_s, true);
              tc::mma_tf32_ss_g<CG>(T_S, desc_add(qlo_d, ch * 16384 + kk * 32), bh, id_s, true);
            }
            commit_all(&bar_kv_empty[c % S]);
          }
          if (ok) commit_all(&bar_s_full);
        }
        // every MMA of this issuer completes before tensor memory is released
        tc::commit_g<CG>(smem_addr(&bar_mma_idle[0]));
        wait(&bar_mma_idle[0], 0);
      } else {
        constexpr uint32_t id_o = tc::idesc_tf32(kPfBM * CG, HD, true);
        const uint64_t v_d = sdesc_mn_sw128_32b(smem_addr(ring));
        bool ok = true;
        for (int t = 0; ok && t < nt; ++t) {
#pragma unroll 1
          for (int qq = 0; ok && qq < Gm::kVChunks; ++qq) {
            const int c = v_chunk0(t) + qq, slot = qq & 1;
            uint32_t off;
            if (!(ok = chunk_ready(c, off))) break;
            if (!(ok = wait(&bar_p_full[slot], (uint32_t)((qq >> 1) & 1)))) break;
            tc::fence_after_sync();
            const uint64_t vh = desc_add(v_d, off), vl = desc_add(v_d, off + C::kVBytes / 2);
            const uint32_t p_hi = T_P + slot * 64, p_lo = p_hi + 32;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint64_t bh = desc_add(vh, ks * 1024), bl = desc_add(vl, ks * 1024);
              tc::mma_tf32_ts_g<CG>(T_O, p_hi + ks * 8, bh, id_o, t > 0 || qq > 0 || ks > 0);
              tc::mma_tf32_ts_g<CG>(T_O, p_hi + ks * 8, bl, id_o, true);
              tc::mma_tf32_ts_g<CG>(T_O, p_lo + ks * 8, bh, id_o, true);
            }
            commit_all(&bar_kv_empty[c % S]);
            commit_all(&bar_p_free[slot]);
          }
          if (ok) commit_all(&bar_pv_done);
        }
        tc::commit_g<CG>(smem_addr(&bar_mma_idle[1]));
        wait(&bar_mma_idle[1], 0);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax warpgroup: thread = query row ----------------
    const int row = (warp - 4) * 32 + lane;
    const int qpos = qbase + row;
    const bool valid = qpos < q_end;
    const int kmin = valid ? pf_start_t(a, qpos) : 0;
    const uint32_t lb = (uint32_t)((warp - 4) * 32) << 16;
    // Rows to threads through the Q lo region: 16-byte piece i of row r at
    // piece i ^ (r % 8) of the row's HD * 4 bytes (conflict-free both ways).
#pragma unroll
    for (int r = 0; r < kQLoads; ++r) {
      const int rr = (warp - 4) * 32 + r * kRowsPerLoad + lane / kPieces;
      *reinterpret_cast<float4*>(qlo + rr * (HD * 4) + (((lane % kPieces) ^ (rr & 7)) << 4)) =
          qbase + rr < q_end ? qv[r] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < kPieces; ++i)
      qv[i] = *reinterpret_cast<const float4*>(qlo + row * (HD * 4) + ((i ^ (row & 7)) << 4));
    // every softmax warp has its row before the Q lo image overwrites the region
    asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) {
      float hi[32], lo[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 t = qv[c * 8 + i];
        lo[4 * i] = t.x * a.scale;
        lo[4 * i + 1] = t.y * a.scale;
        lo[4 * i + 2] = t.z * a.scale;
        lo[4 * i + 3] = t.w * a.scale;
      }
      if (a.q8) {
        // dims 32c..32c+31 are one Q8_0 block: d = amax/127 as truncated fp16,
        // q = round-half-away(x*127/amax); the attention sees q * d, exactly
        // what the reference's int8 dot products compute with
        // (quantize_to_q8_0_cache c:1535-1570, dot_q8_0_q8_0_cache c:1574-1597)
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(lo[i]));
        const float d = amax / 127.0f;
        const float inv = d > 0.0f ? 127.0f / amax : 0.0f;
        const float dq = fp16_to_f32(fp32_to_fp16_trunc(d));
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          int qi = (int)roundf(lo[i] * inv);
          qi = qi > 127 ? 127 : (qi < -128 ? -128 : qi);
          lo[i] = (float)qi * dq;
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float x = lo[i];
        hi[i] = tc::tf32_hi(x);
        lo[i] = x - hi[i];
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
    if (lane == 0) arrive_issuer(&bar_q_ready);

    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < nt; ++jj) {
      ok = __all_sync(0xffffffffu, wait(&bar_s_full, (uint32_t)(jj & 1)));
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
      if (lane == 0) arrive_issuer(&bar_s_free);
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
      const float m_new = fmaxf(m, mt);
      const bool grow = m_new > m + kPfRescale;  // true on the first finite score (m = -inf)
      float alpha = 1.f;
      if (grow) {
        alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
        l *= alpha;
        m = m_new;
      }
      if (jj >= 1 && __any_sync(0xffffffffu, grow)) {
        // rescale O (warp-wide tensor-memory access; rows that keep their max
        // use 1).  Every P.V MMA issued so far must be complete; the next one
        // waits for this warp's P.  Warps that keep their max skip the wait.
        ok = __all_sync(0xffffffffu, wait(&bar_pv_done, (uint32_t)((jj - 1) & 1)));
        if (!ok) break;
        tc::fence_after_sync();
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
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
        if (jj >= 1 || qq >= 2) {
          // the slot's previous quarter (this tile's qq - 2, or the previous
          // tile's qq + 2) has been multiplied into O: p_free[slot] completes
          // once per quarter in the slot, the previous one is number
          // 2 * jj + qq / 2 - 1
          ok = __all_sync(0xffffffffu, wait(&bar_p_free[slot], (uint32_t)((qq >> 1) ^ 1)));
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
        if (lane == 0) arrive_issuer(&bar_p_full[slot]);
      }
      if (!ok) break;
    }
    // ---------------- epilogue ----------------
    if (ok) ok = __all_sync(0xffffffffu, wait(&bar_pv_done, (uint32_t)((nt - 1) & 1)));
    if (ok) {
      tc::fence_after_sync();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      // O rows go through shared memory (the Q lo image is dead once the last
      // S is done) so that global stores are whole 512-byte rows.  16-byte
      // piece i of row r sits at piece i ^ (r % 8): conflict-free for the
      // row-per-thread writes and the row-per-warp reads.
      unsigned char* srow = qlo + row * (HD * 4);
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        float ov[32];
        tc::ld32(T_O + lb + c * 32, ov);
        tc::wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<float4*>(srow + (((c * 8 + i) ^ (row & 7)) << 4)) =
              make_float4(ov[4 * i] * inv, ov[4 * i + 1] * inv, ov[4 * i + 2] * inv, ov[4 * i + 3] * inv);
      }
      __syncwarp();
#pragma unroll 4
      for (int r = 0; r < kQLoads; ++r) {
        const int rr = (warp - 4) * 32 + r * kRowsPerLoad + lane / kPieces;
        const int pc = lane % kPieces;
        const int pos = qbase + rr;
        if (pos < q_end)
          *reinterpret_cast<float4*>(a.out + ((long long)(pos - a.q_pos0) * a.n_heads + h) * HD + 4 * pc) =
              *reinterpret_cast<const float4*>(qlo + rr * (HD * 4) + ((pc ^ (rr & 7)) << 4));
      }
    }
  }
  tc::fence_before_sync();
  if constexpr (CG == 2)
    cluster_sync_all();  // no CTA leaves while its peer may still signal it or read its memory
  else
    __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc_g<CG>(tm, 512);
  }
}

// K/V chunk images for prefill_tc_kernel<CG, HD>: per (owned KV head, 128-key
// tile), per CTA half r of the pair: the HD/32 K chunks then the 4 V chunks,
// each hi then lo, from the head-major cache (fp32 kc/vc, or the Q8_0 arrays
// k8/ksc, v8/vsc when k8 is set).  K chunk c of half r holds keys
// [r*128/CG, (r+1)*128/CG) of dims 32c..32c+31; V chunk v of half r holds
// keys 32v..32v+31 of dims [r*HD/CG, (r+1)*HD/CG).  Keys at or beyond n_keys
// read as 0.  grid (n_ktiles, kvh_count), 256 threads.
template <int CG, int HD>
__global__ void prefill_prep_kernel(const float* __restrict__ kc, const float* __restrict__ vc, long long head_stride,
                                    int n_keys, int n_ktiles, float* __restrict__ img, const int8_t* __restrict__ k8,
                                    const int8_t* __restrict__ v8, const uint16_t* __restrict__ ksc,
                                    const uint16_t* __restrict__ vsc) {
  using C = PfCfg<CG, HD>;
  using Gm = PfGeom<HD>;
  const int j = blockIdx.x, hl = blockIdx.y;
  unsigned char* base = reinterpret_cast<unsigned char*>(img) + ((long long)hl * n_ktiles + j) * Gm::kTileBytes;
  constexpr int kVRows = HD / CG;               // dims of a V chunk per CTA half
  constexpr int kVBase = Gm::kKChunks * C::kKBytes;  // V chunks after the K chunks of a half
  for (int idx = threadIdx.x; idx < kPfBN * HD / 4; idx += blockDim.x) {
    const int key = idx / (HD / 4), c16 = idx % (HD / 4);  // 16-byte piece of the row
    const int pos = j * kPfBN + key;
    float4 kx = make_float4(0.f, 0.f, 0.f, 0.f), vx = kx;
    if (pos < n_keys) {
      const long long e = hl * head_stride + (long long)pos * HD + 4 * c16;
      if (k8) {
        // Q8_0 cache: the values the reference's dot products use, d * int8 (exact)
        const char4 kq = *reinterpret_cast<const char4*>(k8 + e);
        const char4 vq = *reinterpret_cast<const char4*>(v8 + e);
        const float dk = fp16_to_f32(ksc[e / 32]), dv = fp16_to_f32(vsc[e / 32]);
        kx = make_float4((float)kq.x * dk, (float)kq.y * dk, (float)kq.z * dk, (float)kq.w * dk);
        vx = make_float4((float)vq.x * dv, (float)vq.y * dv, (float)vq.z * dv, (float)vq.w * dv);
      } else {
        kx = *reinterpret_cast<const float4*>(kc + e);
        vx = *reinterpret_cast<const float4*>(vc + e);
      }
    }
    const float4 khi = make_float4(tc::tf32_hi(kx.x), tc::tf32_hi(kx.y), tc::tf32_hi(kx.z), tc::tf32_hi(kx.w));
    const float4 klo = make_float4(kx.x - khi.x, kx.y - khi.y, kx.z - khi.z, kx.w - khi.w);
    const float4 vhi = make_float4(tc::tf32_hi(vx.x), tc::tf32_hi(vx.y), tc::tf32_hi(vx.z), tc::tf32_hi(vx.w));
    const float4 vlo = make_float4(vx.x - vhi.x, vx.y - vhi.y, vx.z - vhi.z, vx.w - vhi.w);
    const int part = c16 & 7;  // 16-byte piece within its 128-byte (32-dim) block
    // K chunk c16/8, half key/kRows: K-major, 128-byte swizzle (piece ^ key % 8)
    const int kr = key / C::kRows, kl = key % C::kRows;
    const int kb = kr * C::kHalfTile + (c16 >> 3) * C::kKBytes + kl * 128 + ((part ^ (kl & 7)) << 4);
    *reinterpret_cast<float4*>(base + kb) = khi;
    *reinterpret_cast<float4*>(base + kb + C::kKBytes / 2) = klo;
    // V chunk key/32, half dim/kVRows: MN-major, 32-byte units ^ (key % 4),
    // 32-dim atoms of eight 4-key groups
    const int dim = 4 * c16, vr = dim / kVRows, atom = (dim % kVRows) >> 5;
    const int kv = key & 31, byte = part * 16;
    const int vb = vr * C::kHalfTile + kVBase + (key >> 5) * C::kVBytes + atom * 4096 + (kv >> 2) * 512 +
                   (kv & 3) * 128 + ((((byte >> 5) ^ (kv & 3)) << 5) | (byte & 31));
    *reinterpret_cast<float4*>(base + vb) = vhi;
    *reinterpret_cast<float4*>(base + vb + C::kVBytes / 2) = vlo;
  }
}

}  // namespace l3p
