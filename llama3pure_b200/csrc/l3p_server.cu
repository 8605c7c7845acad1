// l3p_server.cu -- the host side of the host-call server (server.cuh):
// l3p_attn_set_host_server, and the l3p_attn_step / l3p_attn_decode calls it
// serves.  A call packs its rows into 64-bit packets tagged with its number,
// copies them into the device inbox with one asynchronous copy, and polls the
// mergers' flags in the outbox; the resident grid does the rest.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <ctime>

#include "ctx.h"
#include "server.cuh"

using namespace l3p;
using namespace l3p_api;

namespace {

constexpr long long kDefaultIdleUs = 20000;  // an idle instance leaves after 20 ms
constexpr int kCheckEveryUs = 100;           // a waiting call looks at the stream this often
constexpr int kMaxRelaunches = 4;            // per call

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Device buffer of the server: the inbox, q copies by call parity, go words,
// their descriptors and the designated-merger flags by call parity.
struct SrvLayout {
  size_t inbox_off, q_off, go_off, desc_off, flags_off, bytes;
  long long qd, inbox_words, flag_words;
};

SrvLayout srv_layout(const l3p_attn_ctx* ctx) {
  SrvLayout l{};
  l.qd = (long long)ctx->cfg.n_heads * ctx->hd;
  l.inbox_words = kSrvHeader + l.qd + 2ll * ctx->cfg.n_kv_heads * ctx->hd;
  l.flag_words = (long long)ctx->kvh_count * ctx->n_hg * kMaxSplits;
  l.inbox_off = 0;
  l.q_off = align_up((size_t)l.inbox_words * 8, 256);
  l.go_off = align_up(l.q_off + 2 * l.qd * sizeof(float), 256);
  l.desc_off = align_up(l.go_off + (size_t)ctx->kvh_count * 8, 256);
  l.flags_off = align_up(l.desc_off + (size_t)ctx->kvh_count * 3 * sizeof(int), 256);
  l.bytes = l.flags_off + 2 * (size_t)l.flag_words * sizeof(unsigned);
  return l;
}

// Outbox: [qd] output floats, then the mergers' flags.
size_t outbox_bytes(const l3p_attn_ctx* ctx) {
  const SrvLayout l = srv_layout(ctx);
  return (size_t)l.qd * 4 + (size_t)l.flag_words * 4;
}

#ifdef L3P_DECODE_TRACE
long long realtime_ns() {
  timespec t;
  clock_gettime(CLOCK_REALTIME, &t);
  return (long long)t.tv_sec * 1000000000ll + t.tv_nsec;
}
// Slot metadata of served call c (trace ordinal, grid x, y, z, layer,
// position) and the host's times in the slot's last CTA row: [0] before the
// call's packets are written, [2] the copy issued, [3] every flag seen, [1]
// the output read (CLOCK_REALTIME ns).
void trace_call(l3p_attn_ctx* ctx, unsigned c, int gx, int gy, int layer, int pos, int what) {
  if (!ctx->trace_host) return;
  const int ts = (int)(c % kTraceSlots);
  unsigned long long* row = ctx->trace_host + (size_t)ts * kTraceCtas * 8 + (size_t)(kTraceCtas - 1) * 8;
  if (what == 0) {
    long long* m = ctx->trace_meta[ts];
    m[0] = (long long)c, m[1] = gx, m[2] = gy, m[3] = 1, m[4] = layer, m[5] = pos;
    ctx->trace_count = std::max<unsigned long long>(ctx->trace_count, std::min<unsigned long long>(c, kTraceSlots));
  }
  row[what] = (unsigned long long)realtime_ns();
}
#else
void trace_call(l3p_attn_ctx*, unsigned, int, int, int, int, int) {}
#endif

unsigned next_call(l3p_attn_ctx* ctx) {
  if (ctx->srv_next == 0) ctx->srv_next = 1;  // 0 is no call (and no flag tag)
  return ctx->srv_next++;
}

void pack(unsigned long long* dst, const float* src, size_t n, unsigned long long tag) {
  const unsigned* u = reinterpret_cast<const unsigned*>(src);
  for (size_t i = 0; i < n; ++i) dst[i] = tag | u[i];
}

// Posts call c: the header and (not for kSrvExit) the owned rows as packets
// into the staging buffer, then one copy into the device inbox.  The staging
// buffer is free: the previous call's packets have all been read on the
// device (the host has its flags), and a re-post waits for the copy stream.
int post(l3p_attn_ctx* ctx, unsigned c, int layer, int pos, unsigned cmd, const float* q, const float* k,
         const float* v) {
  unsigned long long* st = ctx->srv_stage;
  const unsigned long long tag = (unsigned long long)c << 32;
  st[0] = tag | (unsigned)layer;
  st[1] = tag | (unsigned)pos;
  st[2] = tag | cmd;
  st[3] = tag;
  size_t n = kSrvHeader;
  if (cmd != kSrvExit) {
    int r0, r1;
    owned_rows(ctx, &r0, &r1);
    const size_t row0 = (size_t)r0 * ctx->hd, nrow = (size_t)(r1 - r0) * ctx->hd;
    const size_t kv0 = (size_t)ctx->cfg.kv_head_begin * ctx->hd, nkv = (size_t)ctx->kvh_count * ctx->hd;
    pack(st + n, q + row0, nrow, tag);
    n += nrow;
    if (cmd == kSrvStep) {
      pack(st + n, k + kv0, nkv, tag);
      pack(st + n + nkv, v + kv0, nkv, tag);
      n += 2 * nkv;
    }
  }
  const SrvLayout l = srv_layout(ctx);
  L3P_CUDA(ctx, cudaMemcpyAsync(ctx->srv_dev + l.inbox_off, st, n * 8, cudaMemcpyHostToDevice, ctx->srv_copy));
  return L3P_OK;
}

// Launches an instance whose first call is `first`, with the geometry of `g`.
int launch_server(l3p_attn_ctx* ctx, const ServerGeom& g, unsigned first) {
  const SrvLayout l = srv_layout(ctx);
  DecodeArgs a{};
  decode_common_args(ctx, &a);
  a.nsplit = g.nsplit;
  a.merge_k = g.merge_k;
  a.counters = ctx->counters;  // unused: the server merges through tagged flags
  ServerArgs s{};
  s.inbox = reinterpret_cast<const unsigned long long*>(ctx->srv_dev + l.inbox_off);
  s.out = reinterpret_cast<float*>(ctx->srv_outbox_dev);
  s.done = reinterpret_cast<unsigned*>(ctx->srv_outbox_dev + (size_t)l.qd * 4);
  for (int p = 0; p < 2; ++p) {
    s.q_dev[p] = reinterpret_cast<float*>(ctx->srv_dev + l.q_off) + p * l.qd;
    s.ws_o[p] = ctx->ws_o + p * (ctx->ws_o_floats / kScratchSlots);
    s.ws_ml[p] = ctx->ws_ml + p * (ctx->ws_ml_floats / kScratchSlots);
    s.flags[p] = reinterpret_cast<unsigned*>(ctx->srv_dev + l.flags_off) + p * l.flag_words;
  }
  s.go = reinterpret_cast<unsigned long long*>(ctx->srv_dev + l.go_off);
  s.go_desc = reinterpret_cast<int*>(ctx->srv_dev + l.desc_off);
  s.first_call = first;
  s.instance = ++ctx->srv_instance;
  s.idle_ns = ctx->srv_idle_ns;
#ifdef L3P_DECODE_TRACE
  if (ctx->trace_dev && (long long)g.nsplit * g.units < kTraceCtas) {
    s.trace = ctx->trace_dev;
    s.trace_slots = kTraceSlots;
    s.trace_stride = kTraceCtas * 8;
  }
#endif
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(g.nsplit, g.units, 1);
  lc.blockDim = dim3(g.threads, 1, 1);
  lc.dynamicSmemBytes = g.smem;
  lc.stream = ctx->stream;
  // every CTA resident at once: the fetchers, the go waits and the merges
  // wait for one another
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  void* args[] = {&a, &s};
  L3P_CUDA(ctx, cudaLaunchKernelExC(&lc, g.fn, args));
  ++ctx->launches;
  ++ctx->srv_restarts;
  ctx->srv_running = true;
  ctx->srv_nsplit = g.nsplit;
  return L3P_OK;
}

int alloc_server(l3p_attn_ctx* ctx) {
  if (ctx->srv_dev) return L3P_OK;
  const SrvLayout l = srv_layout(ctx);
  const size_t ob = outbox_bytes(ctx);
  if (cudaHostAlloc(&ctx->srv_outbox, ob, cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(&ctx->srv_outbox_dev, ctx->srv_outbox, 0) != cudaSuccess ||
      cudaHostAlloc(&ctx->srv_stage, (size_t)l.inbox_words * 8, cudaHostAllocDefault) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->srv_copy, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->srv_dev, l.bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(ctx, L3P_E_NOMEM, "host-call server buffers (%zu device, %zu mapped bytes)", l.bytes, ob);
  }
  memset(ctx->srv_outbox, 0, ob);
  L3P_CUDA(ctx, cudaMemset(ctx->srv_dev, 0, l.bytes));
  L3P_CUDA(ctx, cudaDeviceSynchronize());
  return L3P_OK;
}

}  // namespace

namespace l3p_api {

int stop_server(l3p_attn_ctx* ctx) {
  if (!ctx->srv_running) return L3P_OK;
  ctx->srv_running = false;
  // every fetcher still resident passes the exit on
  if (int rc = post(ctx, next_call(ctx), 0, 0, kSrvExit, nullptr, nullptr, nullptr)) return rc;
  L3P_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  L3P_CUDA(ctx, cudaStreamSynchronize(ctx->srv_copy));
  return read_err(ctx);
}

int server_call(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k, const float* v, float* out) {
  DeviceScope dev(ctx->cfg.device);
  ServerGeom g;
  if (int rc = server_geom(ctx, pos, &g)) return rc;
  if (ctx->srv_running && g.nsplit != ctx->srv_nsplit)  // re-planned: a new instance with the new split
    if (int rc = stop_server(ctx)) return rc;
  using clock = std::chrono::steady_clock;
  auto now_ns = [] {
    return (long long)std::chrono::duration_cast<std::chrono::nanoseconds>(clock::now().time_since_epoch()).count();
  };
  if (ctx->srv_running && now_ns() - ctx->srv_last_ns > (long long)(ctx->srv_idle_ns / 2) &&
      cudaStreamQuery(ctx->stream) == cudaSuccess) {  // the instance has left after an idle spell
    ctx->srv_running = false;
    if (int rc = read_err(ctx)) return rc;
  }
  const unsigned cmd = k ? kSrvStep : kSrvDecode;
  unsigned c = next_call(ctx);
  trace_call(ctx, c, g.nsplit, g.units, layer, pos, 0);
  if (int rc = post(ctx, c, layer, pos, cmd, q, k, v)) return rc;
  trace_call(ctx, c, g.nsplit, g.units, layer, pos, 2);
  if (!ctx->srv_running)
    if (int rc = launch_server(ctx, g, c)) return rc;

  // the call is done when every merger's flag carries c
  const SrvLayout l = srv_layout(ctx);
  const volatile unsigned* done = reinterpret_cast<const volatile unsigned*>(ctx->srv_outbox + (size_t)l.qd * 4);
  const size_t n_done = (size_t)g.units * g.merge_k;
  const auto t0 = clock::now();
  auto next_check = t0 + std::chrono::microseconds(kCheckEveryUs);
  const auto limit = t0 + std::chrono::nanoseconds(ctx->srv_idle_ns + 2 * kGroupWaitNs);
  int relaunches = 0;
  size_t i = 0;
  unsigned misses = 0;
  while (i < n_done) {
    if (done[i] == c) {
      ++i;
      continue;
    }
    if (++misses % 256) continue;
    const auto now = clock::now();
    if (now < next_check) continue;
    next_check = now + std::chrono::microseconds(kCheckEveryUs);
    const cudaError_t e = cudaStreamQuery(ctx->stream);
    if (e == cudaErrorNotReady) {
      if (now > limit) {  // resident but silent: end it, report the wait
        stop_server(ctx);
        return fail(ctx, L3P_E_TIMEOUT, "the host-call server did not answer call %u", c);
      }
      continue;
    }
    if (e != cudaSuccess) return fail(ctx, L3P_E_CUDA, "host-call server: %s", cudaGetErrorString(e));
    // the instance has left (idle before the call reached every fetcher, or a
    // device error): report an error, else post the call again to a new one
    ctx->srv_running = false;
    if (int rc = read_err(ctx)) return rc;
    if (++relaunches > kMaxRelaunches) return fail(ctx, L3P_E_CUDA, "the host-call server keeps leaving");
    L3P_CUDA(ctx, cudaStreamSynchronize(ctx->srv_copy));  // the staging buffer is free
    c = next_call(ctx);
    if (int rc = post(ctx, c, layer, pos, cmd, q, k, v)) return rc;
    if (int rc = launch_server(ctx, g, c)) return rc;
    i = 0;
  }
  // the flags were stored after the output (system-scope fence on the device)
  __atomic_thread_fence(__ATOMIC_ACQUIRE);
  trace_call(ctx, c, g.nsplit, g.units, layer, pos, 3);
  int r0, r1;
  owned_rows(ctx, &r0, &r1);
  const size_t row0 = (size_t)r0 * ctx->hd, nrow = (size_t)(r1 - r0) * ctx->hd;
  memcpy(out + row0, reinterpret_cast<const float*>(ctx->srv_outbox) + row0, nrow * 4);
  ctx->srv_last_ns = now_ns();
  trace_call(ctx, c, g.nsplit, g.units, layer, pos, 1);
  return read_err(ctx);
}

}  // namespace l3p_api

L3P_API int l3p_attn_set_host_server(l3p_attn_ctx* ctx, int enable, long long idle_us) {
  if (!ctx) return L3P_E_INVAL;
  if (idle_us < 0) return fail(ctx, L3P_E_INVAL, "idle time %lld us", idle_us);
  CtxScope dev(ctx);  // stops a resident instance
  if (!enable) {
    ctx->srv_on = false;
    return L3P_OK;
  }
  if (ctx->q8) return fail(ctx, L3P_E_UNSUPPORTED, "the host-call server serves fp32 caches only");
  if (ctx->cfg.seq_begin != 0)
    return fail(ctx, L3P_E_UNSUPPORTED, "the host-call server needs the whole sequence on this context");
  ServerGeom g;
  if (int rc = server_geom(ctx, 0, &g)) return rc;
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->cfg.device);
  if (!coop) return fail(ctx, L3P_E_UNSUPPORTED, "the device has no cooperative launch");
  L3P_CUDA(ctx, cudaFuncSetAttribute(g.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, g.smem));
  if (int rc = alloc_server(ctx)) return rc;
  ctx->srv_idle_ns = (unsigned long long)(idle_us > 0 ? idle_us : kDefaultIdleUs) * 1000ull;
  ctx->srv_on = true;
  return L3P_OK;
}
