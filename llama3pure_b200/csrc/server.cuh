// server.cuh -- the host-call server: one resident decode grid that serves
// the single-token host-pointer calls (l3p_attn_step, l3p_attn_decode) of a
// context, so that a call costs no kernel launch and no stream
// synchronisation.
//
// The reference calls its attention once per layer and token from the host
// (llama3pure-c-engine.c:3299-3359); this is the device side of that call
// when the host and the GPU talk through memory instead of launches.
//
// Inbox (device memory), written by one host->device copy per call:
//   [0, 4)  header packets: layer, position, command (kSrvExit / kSrvDecode /
//           kSrvStep), padding
//   then    the owned q rows [kvh_count * G][hd], then the owned K rows
//           [kvh_count][hd], then the owned V rows
// Every entry is a 64-bit packet: the 32-bit value in the low half, the call
// number c in the high half.  A copy lands in no particular order, but a
// packet that carries c carries its value, so nothing else orders the inbox.
// (Reading the inputs out of mapped host memory instead cost 2-7 us per PCIe
// round trip on B200 boxes, four round trips per call.)
// Outbox (mapped pinned host memory): the output [n_heads][hd] as floats,
// then one flag per merger [units][merge_k]: the last call whose slice of
// the output it has written, stored after a system-scope fence.
// Per call c, for each owned KV head:
//   1. its fetcher (split 0 of the head's first q-head group) waits for the
//      header and the head's packets of call c, copies the q rows into device
//      memory (slot c & 1) and, for a step, stores the new K/V row into the
//      cache; then it publishes go[head] = (c, instance) after a fence;
//   2. every CTA of the head (the fetcher included) runs decode_f32_cta over
//      the call's layer and position: split-K parts, designated mergers on
//      flags tagged c (scratch slot c & 1); each merger writes its slice of
//      the output, fences at system scope and raises its outbox flag to c;
//   3. the host, which polls the flags, reads the output once every flag
//      carries c.
// Call c + 1 is posted only after the host has every flag of call c, that is
// after every merger of call c has read every partial of call c and the
// fetchers have read every packet of call c: the two scratch slots, the q
// slots and the inbox are never written while their readers run.
// Every wait is bounded: a fetcher with no call for idle_ns publishes the exit
// command and its head's CTAs leave; a CTA that sees no go word for idle_ns +
// kGroupWaitNs sets kErrTimeout and leaves.  The grid is launched
// cooperatively, so all its CTAs are resident and the merge waits end.
#pragma once
#include "decode.cuh"

namespace l3p {

enum : unsigned { kSrvExit = 0, kSrvDecode = 1, kSrvStep = 2 };
constexpr int kSrvHeader = 4;  // header packets of the inbox

struct ServerArgs {
  const unsigned long long* inbox;  // header, then q | K | V packets of the owned rows
  float* out;                       // outbox output (mapped host memory) [n_heads][hd]
  unsigned* done;                   // outbox flags (mapped host memory) [units][merge_k]
  float* q_dev[2];                  // device copies of the owned q rows, by call parity ([n_heads][hd])
  unsigned long long* go;           // per owned KV head: call | instance << 32
  int* go_desc;                     // per owned KV head: layer, position, command
  float* ws_o[2];                   // split scratch by call parity
  float* ws_ml[2];
  unsigned* flags[2];               // designated-merger flags by call parity
  unsigned first_call;              // the first call this instance serves
  unsigned instance;                // go words of earlier instances never match
  unsigned long long idle_ns;       // a fetcher with no call for this long ends its head
  // builds with L3P_DECODE_TRACE: stamps of call c in slot c % trace_slots
  // (trace_stride words per slot, 8 per CTA): the decode body's stages 0-5,
  // 6 = the call seen (fetcher: header; others: go word), 7 = go published
  unsigned long long* trace;
  int trace_slots, trace_stride;
};

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// grid and block as decode_f32_kernel's for one layer and one token (z = 1),
// launched cooperatively; `a` holds the context's fields and the plan.
template <int HD, int GT>
__global__ void __launch_bounds__(DecodeCfg<HD, GT>::kThreads, DecodeCfg<HD, GT>::kCtasPerSm)
    decode_server_kernel(const DecodeArgs a, const ServerArgs s) {
  using C = DecodeCfg<HD, GT>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int s_call[3];  // layer, position, command of the current call
  const int kvh_local = blockIdx.y / a.n_hg;
  const bool fetcher = blockIdx.x == 0 && blockIdx.y % a.n_hg == 0;
  const int gq = a.G * HD;                                    // q values of one KV head
  const long long n_q = (long long)gridDim.y / a.n_hg * gq;   // owned q values
  const long long n_kv = (long long)gridDim.y / a.n_hg * HD;  // owned K (and V) values
  for (unsigned c = s.first_call;; ++c) {
    const unsigned long long want = (unsigned long long)s.instance << 32 | c;
    unsigned long long* const tr = s.trace ? s.trace + (size_t)(c % s.trace_slots) * s.trace_stride : nullptr;
    __syncthreads();  // the previous call is done with shared memory and s_call
    if (fetcher) {
      if (threadIdx.x == 0) {
        int layer = 0, pos = 0, cmd = kSrvExit;
        const unsigned long long t0 = globaltimer_ns();
        while (true) {
          const unsigned long long h0 = ll_load(s.inbox), h1 = ll_load(s.inbox + 1), h2 = ll_load(s.inbox + 2);
          if ((unsigned)(h0 >> 32) == c && (unsigned)(h1 >> 32) == c && (unsigned)(h2 >> 32) == c) {
            trace_stamp(tr, 6);
            layer = (int)(unsigned)h0;
            pos = (int)(unsigned)h1;
            cmd = (int)(unsigned)h2;
            break;
          }
          if (globaltimer_ns() - t0 > s.idle_ns) break;  // idle: this head's CTAs leave
          __nanosleep(32);
        }
        s_call[0] = layer;
        s_call[1] = pos;
        s_call[2] = cmd;
      }
      __syncthreads();
      int cmd = s_call[2];
      if (cmd != kSrvExit) {
        // the head's q rows into device memory, and for a step its new K/V
        // row into the cache, each value once its packet carries c
        const int layer = s_call[0], pos = s_call[1];
        const bool append = cmd == kSrvStep && pos >= a.seq_begin && pos < a.seq_begin + a.cap;
        const long long row = (long long)layer * a.layer_stride + (long long)kvh_local * a.head_stride +
                              (long long)(pos - a.seq_begin) * HD;
        const unsigned long long* in = s.inbox + kSrvHeader;
        float* qd = s.q_dev[c & 1] + ((long long)a.kv_head_begin + kvh_local) * gq;
        const int n_in = gq + (cmd == kSrvStep ? 2 * HD : 0);  // a decode sends no K/V rows
        bool ok = true;
        for (int i = threadIdx.x; i < n_in && ok; i += C::kThreads) {
          const unsigned long long* p = i < gq        ? in + (long long)kvh_local * gq + i
                                        : i < gq + HD ? in + n_q + (long long)kvh_local * HD + (i - gq)
                                                      : in + n_q + n_kv + (long long)kvh_local * HD + (i - gq - HD);
          float v[1];
          ok = ll_wait<1>(p, 1, 1, c, v, a.err);
          if (!ok) break;
          if (i < gq)
            qd[i] = v[0];
          else if (append)
            (i < gq + HD ? a.kc_w + row + (i - gq) : a.vc + row + (i - gq - HD))[0] = v[0];
        }
        if (!__syncthreads_and(ok)) cmd = kSrvExit;  // a packet never came: the error word is set
      }
      if (threadIdx.x == 0) {
        s.go_desc[3 * kvh_local] = s_call[0];
        s.go_desc[3 * kvh_local + 1] = s_call[1];
        s.go_desc[3 * kvh_local + 2] = cmd;
        s_call[2] = cmd;
        fence_acq_rel_gpu();  // the rows (every thread's stores, ordered by the barrier) before go
        st_relaxed_gpu_u64(s.go + kvh_local, want);
        trace_stamp(tr, 7);
      }
    } else {
      if (threadIdx.x == 0) {
        int cmd = kSrvExit;
        const unsigned long long t0 = globaltimer_ns();
        while (true) {
          if (ld_acquire_gpu_u64(s.go + kvh_local) == want) {
            trace_stamp(tr, 6);
            s_call[0] = s.go_desc[3 * kvh_local];
            s_call[1] = s.go_desc[3 * kvh_local + 1];
            cmd = s.go_desc[3 * kvh_local + 2];
            break;
          }
          if (globaltimer_ns() - t0 > s.idle_ns + kGroupWaitNs) {
            *reinterpret_cast<volatile int*>(a.err) = kErrTimeout;
            break;
          }
          __nanosleep(64);
        }
        s_call[2] = cmd;
      }
    }
    __syncthreads();
    if (s_call[2] == kSrvExit) return;
    DecodeArgs b = a;
    b.layer0 = s_call[0];
    b.pos0 = s_call[1];
    b.q = s.q_dev[c & 1];
    b.out = s.out;
    b.ws_o = s.ws_o[c & 1];
    b.ws_ml = s.ws_ml[c & 1];
    b.flags = s.flags[c & 1];
    b.flag_tag = c;
    b.trace = tr;
    decode_f32_cta<HD, GT>(b, smem_raw);
    if ((int)blockIdx.x < a.merge_k) {  // a merger (part < merge_k): its slice of the output is written
      __syncthreads();
      if (threadIdx.x == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(s.done + blockIdx.y * a.merge_k + blockIdx.x), "r"(c)
                     : "memory");
      }
    }
  }
}

}  // namespace l3p
