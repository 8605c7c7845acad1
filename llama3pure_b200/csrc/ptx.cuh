// ptx.cuh -- inline-PTX helpers for sm_100a: mbarriers with bounded waits and
// 1-D bulk asynchronous copies (global -> shared, completed on an mbarrier).
//
// No multicast form of any copy is used anywhere in this library.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace l3p {

// Error bits a kernel may set in the context's error word.
enum : int { kErrTimeout = 1, kErrBadArg = 2 };

// A bounded wait gives up after this many failed try_wait probes (each probe
// may itself block for a hardware-defined interval), sets kErrTimeout and
// lets the kernel finish without the data.
constexpr uint32_t kMaxWaitProbes = 1u << 24;

// Waits on another GPU (the NVLink groups) are bounded by time, not probes:
// a member that never arrives costs this long, then the error word is set.
constexpr unsigned long long kGroupWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Make mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for phase `parity` of `bar` to complete, giving up after
// kMaxWaitProbes probes.  Returns false on timeout and records it in *err
// (a plain store: the error word may live in mapped host memory).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kMaxWaitProbes; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) *reinterpret_cast<volatile int*>(err) = kErrTimeout;
  return false;
}

// ---- thread-block cluster helpers (CTA pairs of the tensor-core prefill)

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t cta_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cta_addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its cluster address (this CTA's or a peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// mbar_wait_bounded with cluster-scope acquire: for barriers that CTAs of the
// cluster (or tensor-core commits issued by a peer) complete.
__device__ __forceinline__ bool mbar_wait_bounded_cluster(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kMaxWaitProbes; ++i)
    if (mbar_try_wait_cluster(bar, parity)) return true;
  if (err) *reinterpret_cast<volatile int*>(err) = kErrTimeout;
  return false;
}

// Every thread of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// System-scope ordering for flags and counters that other GPUs read or write
// over NVLink.
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Low-latency packets between GPUs: a float and the call number e that wrote
// it, in one 64-bit word stored and loaded with relaxed system-scope accesses,
// which cannot tear -- a receiver that reads e in a packet has its value
// without any fence or flag.
__device__ __forceinline__ void ll_store(unsigned long long* p, float v, unsigned e) {
  const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Values of packets p[0], p[stride], ... p[(n-1)*stride] once all carry call e
// (all loads of a poll in flight together); false after kGroupWaitNs.
template <int MAXN>
__device__ __forceinline__ bool ll_wait(const unsigned long long* p, long long stride, int n, unsigned e,
                                        float (&v)[MAXN], int* err) {
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    unsigned long long w[MAXN];
#pragma unroll
    for (int m = 0; m < MAXN; ++m)
      if (m < n) w[m] = ll_load(p + m * stride);
    bool all = true;
#pragma unroll
    for (int m = 0; m < MAXN; ++m)
      if (m < n) {
        all = all && (unsigned)(w[m] >> 32) == e;
        v[m] = __uint_as_float((unsigned)w[m]);
      }
    if (all) return true;
    if (globaltimer_ns() - t0 > kGroupWaitNs) {
      *reinterpret_cast<volatile int*>(err) = kErrTimeout;
      return false;
    }
    __nanosleep(20);
  }
}

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float4 lds128(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

}  // namespace l3p
