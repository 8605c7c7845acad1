// seq_xchg.cuh -- sequence-sharded decode across GPUs without a collective
// library: the partial (m, l, o) triples of the GPUs that share a KV-head
// range are read straight out of each other's memory over NVLink.
//
// The reference has no multi-device path (c:3327-3328 parallelises over KV
// heads inside one process); this file is new.
//
// Layout of a context's exchange region (one cudaMalloc, exported by CUDA IPC
// and mapped by every peer of the group):
//   header  [0, 256): u32 step counter at byte 64 (this member's calls so far;
//           only its own merge kernel reads and writes it), u32 exit ticket of
//           the merge kernel's CTAs at byte 68
//   parts   from byte 256, [n_layers][slot_floats] float: per layer the
//           normalised partial output of every q head ([n_heads][hd]), then
//           its (m, l) pairs ([n_heads][2]), written by this context's own
//           decode (partial mode) and read only by its own merge kernel
//   inbox   after the parts, [2][n_parts][slot_floats] u64 packets: member
//           s's partial of the current call, sent by member s
// Each decode_seq step: the partial decode of this GPU's positions writes the
// layer's part slot (a normal split-K launch), then seq_merge_kernel (one
// thread per owned output element)
//   1. (after griddepcontrol.wait: the partial is complete) sends the owned
//      rows of its partial to slot [e&1][me] of every member's inbox, itself
//      included, e = its step counter + 1;
//   2. waits (at most kGroupWaitNs, else kErrTimeout) for every member's
//      packets in its own inbox and writes the log-sum-exp merge, members in
//      order (the same bits on every member), to `out`;
//   3. the last CTA to finish stores e into its step counter.
// Every value travels as one 64-bit packet (float | e << 32), stored and
// loaded with relaxed system-scope 64-bit accesses, which cannot tear: a
// packet that carries e carries its value, so no fence or flag orders
// anything (a system-scope fence after peer stores measured ~4.6 us on B200).
// The step counter lives on the device, so a captured CUDA graph replays
// correctly.  Members run the same sequence of steps; two inbox slots
// suffice, since a member cannot finish call e + 1 (and so send call e + 2)
// before every member has sent call e + 1, which each does only after its own
// merge of call e.
#pragma once
#include "decode.cuh"
#include "limits.cuh"

namespace l3p {

constexpr int kXchgMaxRows = 128;  // owned q heads of a sequence-group member at most

struct XchgArgs {
  const float* mine;                        // this layer's partial in this member's part slot
  unsigned long long* inbox[kXchgMaxParts];  // every member's inbox (own included)
  unsigned* my_step;                        // this member's step counter
  long long slot_floats;                    // packets of one member's slot
  int n_parts, part;                        // group size and this member's index
  int hd, n_heads, row_begin, n_rows;       // owned q heads [row_begin, row_begin + n_rows)
  float* out;                               // [n_heads][hd]
  int* err;
};


// grid: ceil(n_rows * hd / kXchgThreads) CTAs of kXchgThreads threads; CTA c
// sends and merges output elements [c * kXchgThreads, (c + 1) * kXchgThreads)
// of the owned rows, one per thread (a thread's packet polls then overlap no
// other of its own), and CTA 0 also sends the (m, l) pairs.
constexpr int kXchgThreads = 512;
static __global__ void __launch_bounds__(kXchgThreads) seq_merge_kernel(const XchgArgs a) {
  pdl_launch_dependents();
  pdl_wait();  // this GPU's partial is written
  __shared__ unsigned s_e;
  constexpr int kHeads = kXchgThreads / 64 + 1;  // owned heads a CTA's elements touch (head_dim >= 64)
  __shared__ float s_m[kXchgMaxParts][kHeads], s_l[kXchgMaxParts][kHeads];
  if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile unsigned*>(a.my_step) + 1u;
  __syncthreads();
  const unsigned e = s_e;
  const long long par = e & 1u;
  const int N = a.n_parts;
  const long long ml0 = (long long)a.n_heads * a.hd;  // (m, l) pairs after the outputs
  const int n_o = a.n_rows * a.hd;
  const int idx = blockIdx.x * kXchgThreads + threadIdx.x;  // this thread's output element
  const int h_first = blockIdx.x * kXchgThreads / a.hd;     // first owned head of this CTA
  // 1. this member's partial to every member's inbox (itself included)
  if (idx < n_o) {
    const long long src = (long long)a.row_begin * a.hd + idx;
    const float v = a.mine[src];
    for (int m = 0; m < N; ++m) ll_store(a.inbox[m] + (par * N + a.part) * a.slot_floats + src, v, e);
  }
  if (blockIdx.x == 0)
    for (int t = threadIdx.x; t < 2 * a.n_rows; t += kXchgThreads) {
      const long long src = ml0 + 2ll * a.row_begin + t;
      const float v = a.mine[src];
      for (int m = 0; m < N; ++m) ll_store(a.inbox[m] + (par * N + a.part) * a.slot_floats + src, v, e);
    }
  // 2. every member's (m, l) of the heads this CTA merges
  const unsigned long long* in = a.inbox[a.part] + par * N * a.slot_floats;
  const int h_count = min(kHeads, a.n_rows - h_first);
  bool ok = true;
  if (threadIdx.x < N * h_count) {
    const int m = threadIdx.x / h_count, hh = threadIdx.x % h_count;
    float v[2];
    ok = ll_wait<2>(in + m * a.slot_floats + ml0 + 2ll * (a.row_begin + h_first + hh), 1, 2, e, v, a.err);
    s_m[m][hh] = v[0];
    s_l[m][hh] = v[1];
  }
  ok = __syncthreads_and(ok);
  // 3. this thread's output element, members in order (the same bits on every member)
  if (ok && idx < n_o) {
    const int hh = idx / a.hd - h_first;
    const long long off = (long long)a.row_begin * a.hd + idx;
    float o[kXchgMaxParts];
    if (ll_wait<kXchgMaxParts>(in + off, a.slot_floats, N, e, o, a.err)) {
      float M = -INFINITY;
#pragma unroll
      for (int m = 0; m < kXchgMaxParts; ++m)
        if (m < N) M = fmaxf(M, s_m[m][hh]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int m = 0; m < kXchgMaxParts; ++m) {
        if (m < N && s_m[m][hh] != -INFINITY) {  // empty ranges carry m = -inf and weigh nothing
          const float w = s_l[m][hh] * fast_exp2(s_m[m][hh] - M);
          L += w;
          O = fmaf(o[m], w, O);
        }
      }
      a.out[off] = L > 0.f ? O / L : 0.f;
    }
  }
  // 4. the last CTA to leave ends this call on this member (the next call
  // reads the step after this grid has completed)
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(a.my_step + 1, 1u) == gridDim.x - 1) {
    a.my_step[1] = 0u;
    *reinterpret_cast<volatile unsigned*>(a.my_step) = e;
  }
}

}  // namespace l3p
