// seq_xchg.cuh -- sequence-sharded decode across GPUs without a collective
// library: the partial (m, l, o) triples of the GPUs that share a KV-head
// range are read straight out of each other's memory over NVLink.
//
// The reference has no multi-device path (c:3327-3328 parallelises over KV
// heads inside one process); this file is new.
//
// Layout of a context's exchange region (one cudaMalloc, exported by CUDA IPC
// and mapped by every peer of the group):
//   flags   [kXchgMaxParts] uint32 at byte 0: flags[s] = the last step for
//           which member s has published its partials (written by member s)
//   step    uint32 at byte 64: this member's own step counter (only its own
//           merge kernel reads and writes it)
//   parts   from byte 256, [n_layers][n_heads*hd + 2*n_heads] float: per layer
//           the normalised partial output of every q head ([n_heads][hd]),
//           then its (m, l) pairs ([n_heads][2]), written by this context's
//           own decode (partial mode)
// Each decode_seq step: the partial decode of this GPU's positions writes
// the layer's slot (a normal split-K launch), then seq_merge_kernel (one CTA)
//   1. (after griddepcontrol.wait: the partials are complete) advances the
//      step counter and stores the step into flags[me] of every peer -- a
//      release store at system scope;
//   2. waits (at most kGroupWaitNs) until every peer's step has arrived in its
//      own flags, else sets kErrTimeout in the error word and returns;
//   3. for each owned q head reads the n_parts triples -- its own locally, the
//      peers' over NVLink -- and writes the log-sum-exp merge to `out`.
// The step counter lives on the device, so a captured CUDA graph replays
// correctly.  Members run the same sequence of steps; merge kernels of one
// member never overlap (each decode waits for the merge before it), and a
// member that is ahead can only be writing a later layer's slot, never one a
// slower member still reads.
#pragma once
#include "decode.cuh"
#include "limits.cuh"

namespace l3p {

struct XchgArgs {
  const float* parts[kXchgMaxParts];    // this layer's slot in every member's region (own included)
  unsigned* peer_flags[kXchgMaxParts];  // flags array of every member (own included)
  unsigned* my_flags;                   // this member's flags; its step counter at my_flags + 16
  int n_parts, part;                    // group size and this member's index
  int hd, n_heads, row_begin, n_rows;   // owned q heads [row_begin, row_begin + n_rows)
  float* out;                           // [n_heads][hd]
  int* err;
};

// grid: ONE CTA of kXchgThreads threads (warp w merges q heads w, w + warps, ...).
constexpr int kXchgThreads = 512;
static __global__ void __launch_bounds__(kXchgThreads) seq_merge_kernel(const XchgArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // this GPU's partials are written
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    unsigned* step = a.my_flags + 16;
    const unsigned e = *step + 1;
    *step = e;
    __threadfence_system();  // the partials (written by the kernel before) precede the flags
    for (int s = 0; s < a.n_parts; ++s)
      if (s != a.part) st_release_sys(a.peer_flags[s] + a.part, e);
    int ok = 1;
    for (int s = 0; s < a.n_parts && ok; ++s) {
      if (s == a.part) continue;
      const unsigned long long t0 = globaltimer_ns();
      // steps only grow: a member already further on has published this step too
      while ((int)(ld_acquire_sys(a.my_flags + s) - e) < 0) {
        if (globaltimer_ns() - t0 > kGroupWaitNs) {
          *reinterpret_cast<volatile int*>(a.err) = kErrTimeout;
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;

  // every thread issues all its loads -- (m, l) of its head and its float4
  // of the output from every member -- before using any, so the merge costs
  // one NVLink round trip, not one per member or per element
  const int hd4 = a.hd / 4;
  for (int idx = threadIdx.x; idx < a.n_rows * hd4; idx += kXchgThreads) {
    const int h = a.row_begin + idx / hd4;
    const long long o4 = (long long)h * hd4 + idx % hd4;                   // float4 of the output
    const long long ml = (long long)a.n_heads * a.hd / 2 + h;              // float2 (m, l) of head h
    float2 mlp[kXchgMaxParts];
    float4 op[kXchgMaxParts];
#pragma unroll
    for (int p = 0; p < kXchgMaxParts; ++p) {
      if (p < a.n_parts) {
        mlp[p] = __ldcv(reinterpret_cast<const float2*>(a.parts[p]) + ml);
        op[p] = __ldcv(reinterpret_cast<const float4*>(a.parts[p]) + o4);
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int p = 0; p < kXchgMaxParts; ++p)
      if (p < a.n_parts) M = fmaxf(M, mlp[p].x);
    float L = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < kXchgMaxParts; ++p) {
      if (p < a.n_parts && mlp[p].x != -INFINITY) {  // empty ranges carry m = -inf and weigh nothing
        const float w = mlp[p].y * fast_exp2(mlp[p].x - M);
        L += w;
        O.x = fmaf(op[p].x, w, O.x);
        O.y = fmaf(op[p].y, w, O.y);
        O.z = fmaf(op[p].z, w, O.z);
        O.w = fmaf(op[p].w, w, O.w);
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    reinterpret_cast<float4*>(a.out)[o4] = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
  }
}

}  // namespace l3p
