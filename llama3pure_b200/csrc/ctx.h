// ctx.h -- the library context and the helpers its translation units share
// (l3p_attn.cu, l3p_preattn.cu, l3p_wo.cu, l3p_groups.cu).  Private: not part
// of the C ABI.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <deque>
#include <initializer_list>
#include <string>
#include <vector>

#include "limits.cuh"
#include "llama3pure_attn.h"

#define L3P_API extern "C" __attribute__((visibility("default")))

namespace l3p {
struct DecodeArgs;
}

struct l3p_attn_ctx {
  l3p_attn_config cfg{};
  int hd = 0, G = 0, GT = 1, n_hg = 1;
  int kvh_count = 0, seq_count = 0;
  float scale = 1.f;
  int num_sms = 148;
  float* kc = nullptr;  // fp32 cache: [n_layers][kvh_count][seq_count][hd]
  float* vc = nullptr;
  bool q8 = false;      // Q8_0 cache (kv_format L3P_KV_Q8_0) instead of kc/vc:
  int8_t* k8 = nullptr;  //   int8 values, same layout as kc
  int8_t* v8 = nullptr;
  uint16_t* ksc = nullptr;  //   fp16 block scales [n_layers][kvh_count][seq_count][hd/32]
  uint16_t* vsc = nullptr;
  long long layer_elems = 0, head_elems = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  // split-K scratch: partial outputs, (m, l) pairs and per-unit tickets
  float* ws_o = nullptr;
  float* ws_ml = nullptr;
  unsigned* counters = nullptr;
  long long ws_o_floats = 0, ws_ml_floats = 0, n_counters = 0;
  // device staging for the host-pointer entry points
  float* st_buf = nullptr;
  size_t st_floats = 0;
  // pinned, device-mapped host staging for the single-token host calls: the
  // inputs cross in one copy and the kernel writes the output straight into it
  float* hst = nullptr;
  float* hst_dev = nullptr;
  size_t hst_floats = 0;
  // prefill: pre-split K/V tile images for the tensor-core kernel
  float* pf_img = nullptr;
  size_t pf_img_floats = 0;
  bool prefill_tc = false;  // head_dim 128 uses the tcgen05 kernel (L3P_PREFILL_PATH=ffma forces the other)
  int prefill_cg = 1;       // CTAs per tcgen05 prefill unit: 2 (CTA pairs) when the GQA group is even
  // device error word in mapped pinned host memory
  int* err_host = nullptr;
  int* err_dev = nullptr;
  long long launches = 0;
  // clusters of 2^i CTAs of this context's decode kernel that fit on the GPU at once
  int max_clusters[5] = {0, 0, 0, 0, 0};
  // L3P_DECODE_PLAN="nsplit:cluster" pins the decomposition (tests use it to
  // exercise every merge path); 0 = automatic
  int force_nsplit = 0, force_cluster = 0;
  // overlap mode: decode launches carry programmatic stream serialisation
  bool overlap = false;
  // split-K plans of recent launches, by (tiles, units, rows per tile, CTAs per SM)
  struct PlanEntry {
    long long n_tiles = -1, units = -1;
    int rows = 0, ctas_per_sm = 0, nsplit = 1, cluster = 1;
  } plan_cache[4];
  unsigned plan_cache_next = 0;
  // one-wave decode launches merge through the last-arriving part (ticket)
  // instead of designated mergers (L3P_DECODE_MERGE=ticket)
  bool ticket_merge = false;
  // split scratch is used in kScratchSlots rotating slices so that launches
  // overlapping on the GPU never share partials or tickets
  unsigned long long launch_seq = 0;
  // cache rows stored by the fused append of recent decode launches, per
  // layer: (launch_seq of the launch, position); see launch_decode
  std::vector<std::deque<std::pair<unsigned long long, int>>> recent_stores;
  // pre-attention step (l3p_attn_set_rope): (cos, sin) per position and pair,
  // [seq_len][hd/2], for dense layers and for Gemma3 SWA layers (the same
  // array when the model has one table), QK-norm weights [2][n_layers][hd]
  // (q then k; null = no QK-norm) and the rotated rows of the raw entry points
  float2* rope_tab = nullptr;
  float2* rope_tab_swa = nullptr;
  float* qk_norm = nullptr;
  float rms_eps = 1e-5f;
  float* rope_buf = nullptr;
  size_t rope_buf_floats = 0;
  // wo projection (l3p_attn_set_wo): per layer the owned columns of the
  // weight rows in the device layout of wo.cuh, and the attention output
  // buffer of the combined host call
  struct WoLayer {
    bool set = false;  // l3p_attn_set_wo has been called for the layer
    int type = 0;      // GGUF type number (0 is F32)
    int rows = 0;
    long long row_bytes = 0;
    int sc_stride = 0;  // bytes per row of Q8_0 scales
    uint8_t* w = nullptr;
    uint8_t* wsc = nullptr;
  };
  std::vector<WoLayer> wo;
  float* wo_x = nullptr;
  int wo_ctas_per_sm[l3p::kWoKernelCount] = {};  // per wo GEMV kernel (l3p_wo.cu's table)
  // sequence group over NVLink (l3p_attn_seq_group_*): this context's exchange
  // region (flags, then per-layer partial slots; seq_xchg.cuh), the members'
  // regions mapped into this process, and the step counter
  int xg_parts = 0, xg_part = 0;
  bool xg_ready = false;
  uint8_t* xg_region = nullptr;
  void* xg_peer[l3p::kXchgMaxParts] = {};
  long long xg_slot_floats = 0;
  // tensor-parallel group over NVLink (l3p_attn_tp_group_*): flags, step
  // counter, then two slots of [members][dim] partial projections
  int tp_members = 0, tp_member = 0, tp_dim = 0;
  bool tp_ready = false;
  uint8_t* tp_region = nullptr;
  void* tp_peer[l3p::kXchgMaxParts] = {};
  // decode trace (builds with L3P_DECODE_TRACE only): mapped pinned stamps of
  // the last kTraceSlots decode launches and their grids, written to the file
  // named by $L3P_TRACE_FILE when the context is destroyed
  unsigned long long* trace_host = nullptr;
  unsigned long long* trace_dev = nullptr;
  long long trace_meta[64][6] = {};  // launch seq, grid x, y, z, layer0, pos0
  unsigned long long trace_count = 0;
  // host-call server (l3p_attn_set_host_server, l3p_server.cu): a resident
  // decode grid on `stream` that takes the single-token host calls through a
  // mailbox in mapped pinned memory (server.cuh)
  bool srv_on = false;       // the host calls go through the server
  bool srv_running = false;  // an instance may be resident on `stream`
  unsigned srv_next = 1;     // number of the next call (never 0)
  unsigned srv_instance = 0;
  unsigned long long srv_idle_ns = 0;
  int srv_nsplit = 0;        // split-K of the running instance
  unsigned long long* srv_stage = nullptr;  // pinned: the packets of the next call's inbox copy
  cudaStream_t srv_copy = nullptr;           // the inbox copies
  uint8_t* srv_outbox = nullptr;             // mapped pinned: output floats, then the mergers' flags
  uint8_t* srv_outbox_dev = nullptr;
  uint8_t* srv_dev = nullptr;  // device: inbox, q copies, go words, descriptors, flags
  long long srv_restarts = 0;       // instances launched
  long long srv_last_ns = 0;        // steady-clock time the last served call ended
  std::string last_error;
};

namespace l3p_api {

#ifdef L3P_DECODE_TRACE
constexpr int kTraceSlots = 64;    // decode launches whose stamps are kept
constexpr int kTraceCtas = 4096;   // CTAs per traced launch at most
#endif

// Records the message of a failing entry point and returns its code.
inline int fail(l3p_attn_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return code;
}

#define L3P_CUDA(ctx, call)                                                                  \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      return l3p_api::fail((ctx), L3P_E_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                           __LINE__);                                                        \
  } while (0)

// Makes the context's device current for the duration of an entry point and
// restores the caller's device afterwards.
struct DeviceScope {
  int prev = -1;
  bool changed = false;
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) changed = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceScope() {
    if (changed) cudaSetDevice(prev);
  }
};

// l3p_server.cu: ends the context's host-call server instance, if one is
// resident, and waits for it to leave the GPU.
int stop_server(l3p_attn_ctx* ctx);
// l3p_server.cu: one l3p_attn_step (k, v non-null) or l3p_attn_decode call
// through the server, which it starts when none is resident.
int server_call(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k, const float* v, float* out);

// DeviceScope for the entry points that launch work or touch the context's
// memory: a resident host-call server would hold every SM, so it is stopped
// first (the next host call starts it again).
struct CtxScope : DeviceScope {
  explicit CtxScope(l3p_attn_ctx* ctx) : DeviceScope(ctx->cfg.device) {
    if (ctx->srv_running) stop_server(ctx);
  }
};

inline cudaStream_t pick_stream(l3p_attn_ctx* ctx, void* s) { return s ? static_cast<cudaStream_t>(s) : ctx->stream; }

// With overlap mode, a launch may start while the kernel before it on the
// stream still runs (programmatic dependent launch); every kernel so launched
// reads nothing the earlier kernel writes before its griddepcontrol.wait.
inline void pdl_attr(const l3p_attn_ctx* ctx, cudaLaunchConfig_t& lc, cudaLaunchAttribute (&attr)[1]) {
  if (!ctx->overlap) return;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
}

// l3p_attn.cu
int check_aligned(l3p_attn_ctx* ctx, std::initializer_list<const void*> ptrs);
int ensure_staging(l3p_attn_ctx* ctx, size_t floats);
int ensure_host_staging(l3p_attn_ctx* ctx, size_t floats);
int check_layer(l3p_attn_ctx* ctx, int layer);
int check_pos_full(l3p_attn_ctx* ctx, int pos);
int read_err(l3p_attn_ctx* ctx);
int finish_host_call(l3p_attn_ctx* ctx);
void owned_rows(const l3p_attn_ctx* ctx, int* row_lo, int* row_hi);
// Decode core shared by the single-layer, multi-layer, prefill and partial
// entry points.  z-slices are layers (layer_step=1) or tokens (pos_step=1).
unsigned long long* trace_slot(l3p_attn_ctx* ctx, int gx, int gy, int gz, int layer, int pos);
int launch_decode(l3p_attn_ctx* ctx, int layer0, int layer_step, int pos0, int pos_step, int nz, const float* q,
                  float* out, float* part_o, float* part_ml, cudaStream_t s, const float* k_new = nullptr,
                  const float* v_new = nullptr, bool allow_overlap = false);
// Cache rows of n_tok tokens.  The next kernel launches when the rows are written.
int launch_append(l3p_attn_ctx* ctx, int layer, int pos0, int n_tok, const float* k, const float* v, cudaStream_t s);
int launch_prefill_tc(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q, float* out,
                      cudaStream_t s);

// Decode geometry of the host-call server for a call at `pos`: the plan's
// split-K (clamped so that the grid is resident at once), the designated
// mergers, and the kernel (null when the context's cache has no server).
struct ServerGeom {
  int nsplit = 1, merge_k = 1, units = 0, threads = 0, smem = 0;
  const void* fn = nullptr;
};
int server_geom(l3p_attn_ctx* ctx, int pos, ServerGeom* g);
// The context's fields of a decode launch: cache, strides, geometry, scale,
// error word (everything but the call's layer, position, q, outputs and plan).
void decode_common_args(const l3p_attn_ctx* ctx, l3p::DecodeArgs* a);

// l3p_preattn.cu
int check_rope(l3p_attn_ctx* ctx);
int step_raw_core(l3p_attn_ctx* ctx, int layer, int pos, const float* q, const float* k, const float* v, float* out,
                  cudaStream_t s, bool allow_overlap);
int prefill_raw_core(l3p_attn_ctx* ctx, int layer, int start_pos, int n_tok, const float* q, const float* k,
                     const float* v, float* out, cudaStream_t s);

// l3p_wo.cu
int launch_wo(l3p_attn_ctx* ctx, int layer, const float* x, float* y, cudaStream_t s, bool tp = false);
int check_wo(l3p_attn_ctx* ctx, int layer);

}  // namespace l3p_api
