// moe_api.cu -- the extern "C" entry points declared in include/moe_block.h and include/moe_ep.h, and the
// library counters behind moe_stats_get.
//
// Host-side launch code replacing the MoE part of forward() (qwen.cu:429-448) and moe() (qwen.cu:345-363), and the
// expert-parallel stages. Every compute entry point validates the shape and the workspace size before launching
// anything and returns cudaErrorInvalidValue on a violation; none allocates memory or synchronises the stream (except
// moe_workspace_error, which reads the error word back). The setup helpers moe_device_alloc / moe_ipc_* of the
// expert-parallel exchange buffers are the only calls that allocate or map memory.
#include <algorithm>
#include <atomic>
#include <climits>
#include <cstring>

#include <cstdlib>

#include <nvtx3/nvToolsExt.h>

#include "moe_common.cuh"
#include "../../include/moe_ep.h"
#include "moe_decode.h"
#include "moe_ep.h"
#include "moe_fused.h"
#include "moe_lean.h"
#include "moe_prefill.h"

using namespace moe;

namespace {
// One NVTX range per entry-point call, named after the entry point (visible in Nsight timelines; with no tool
// attached NVTX calls return at once).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace

namespace {

bool shape_ok(const moe_layer_weights* w) {
  if (!w) return false;
  const int H = w->H, E = w->E, K = w->TOPK, I = w->I, Is = w->Is, G = w->G;
  if (H <= 0 || E <= 0 || K <= 0 || I <= 0 || Is <= 0 || G <= 0) return false;
  if (H % 256 || I % 128 || Is % 128) return false;
  if (G != 32 && G != 64 && G != 128) return false;
  if (H % G || I % G) return false;
  if (K > 8 || E > 256 || K > E) return false;
  if (H > 4096 || I > 2048 || Is > 2048) return false;
  // the optional int8 shared expert: all four arrays, one group size (a multiple of 32) dividing H and Is
  const int n8 = (w->shared_gate_up_q8 != nullptr) + (w->shared_gate_up_s8 != nullptr) +
                 (w->shared_down_q8 != nullptr) + (w->shared_down_s8 != nullptr);
  if (n8 != 0 && n8 != 4) return false;
  if (n8 == 4) {
    const int g8 = w->shared_group;
    if (g8 <= 0 || g8 % 32 || H % g8 || Is % g8) return false;
  }
  return true;
}

bool weights_present(const moe_layer_weights* w, bool router, bool routed, bool shared) {
  if (router && (!w->router || !w->rms2)) return false;
  if (routed && (!w->exp_gu_q || !w->exp_gu_s || !w->exp_dn_q || !w->exp_dn_s)) return false;
  if (shared && (!w->shared_gate_up || !w->shared_down || !w->shared_gate)) return false;
  return true;
}

BlockArgs make_args(const moe_layer_weights* w, void* ws, const WsLayout& L, int T) {
  BlockArgs a;
  memset(&a, 0, sizeof a);
  uint8_t* b = static_cast<uint8_t*>(ws);
  a.w = *w;
  a.T = T;
  a.ticket = reinterpret_cast<uint32_t*>(b + L.ticket);
  a.err = reinterpret_cast<uint32_t*>(b + L.err);
  a.logits = reinterpret_cast<float*>(b + L.logits);
  a.idx = reinterpret_cast<int32_t*>(b + L.idx);
  a.wts = reinterpret_cast<float*>(b + L.wts);
  a.gate = reinterpret_cast<float*>(b + L.gate);
  a.nuniq = reinterpret_cast<int32_t*>(b + L.nuniq);
  a.uniq = reinterpret_cast<int32_t*>(b + L.uniq);
  a.uoff = reinterpret_cast<int32_t*>(b + L.uoff);
  a.upairs = reinterpret_cast<int32_t*>(b + L.upairs);
  a.inter = reinterpret_cast<uint16_t*>(b + L.inter);
  a.sinter = reinterpret_cast<uint16_t*>(b + L.sinter);
  a.routed = reinterpret_cast<float*>(b + L.routed);
  a.sout = reinterpret_cast<uint16_t*>(b + L.sout);
  if (L.maxT >= kPrefillMinT) {
    a.bits = reinterpret_cast<uint32_t*>(b + L.bits);
    a.wpre = reinterpret_cast<uint32_t*>(b + L.wpre);
    a.counts = reinterpret_cast<int32_t*>(b + L.counts);
    a.offsets = reinterpret_cast<int32_t*>(b + L.offsets);
    a.tiles = b + L.tiles;
    a.ntiles = reinterpret_cast<int32_t*>(b + L.ntiles);
    a.tiles2 = b + L.tiles2;
    a.ntiles2 = reinterpret_cast<int32_t*>(b + L.ntiles2);
    a.sorted = reinterpret_cast<int32_t*>(b + L.sorted);
    a.slot = reinterpret_cast<float*>(b + L.slot);
    a.nwp = L.nwp;
    a.max_tiles = L.max_tiles;
    a.max_tiles2 = L.max_tiles2;
  }
  return a;
}

WsLayout layout_for(const moe_layer_weights* w, int T) { return ws_layout(w->H, w->E, w->TOPK, w->I, w->Is, T); }

// The decode kernels stage one chunk of tokens in shared memory; larger T runs chunk by chunk.
int chunk_tokens(const moe_layer_weights* w) { return decode_max_tokens(w->H, w->TOPK, w->I, w->Is); }

// T >= kPrefillMinT takes the prefill path (tcgen05 GEMMs, the reference's tile numerics) unless the environment
// sets MOE_B200_PREFILL=0 (read once per process), which keeps the decode kernels, chunk by chunk.
// moe_set_prefill_min_tokens moves the threshold (0 restores the default).
std::atomic<int> g_prefill_min{0};
int prefill_min_tokens() {
  int v = g_prefill_min.load(std::memory_order_relaxed);
  if (v == 0) {
    const char* e = getenv("MOE_B200_PREFILL");
    v = (e && e[0] == '0') ? INT_MAX : kPrefillMinT;
  }
  return v;
}
bool use_prefill(const moe_layer_weights* w, int T) {
  return T >= kPrefillMinT && T >= prefill_min_tokens() && prefill_supported(*w);
}
// Tokens the workspace layout of one call is computed for.
int layout_tokens(const moe_layer_weights* w, int T) { return use_prefill(w, T) ? T : std::min(T, chunk_tokens(w)); }

int check_common(const moe_layer_weights* w, void* ws, size_t bytes, int T) {
  if (!shape_ok(w) || !ws || T < 1) return (int)cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(ws) % 256) return (int)cudaErrorInvalidValue;
  if (bytes < layout_for(w, layout_tokens(w, T)).total) return (int)cudaErrorInvalidValue;
  return 0;
}

}  // namespace

// Counters of moe_stats_get (relaxed atomics: each is a tally, nothing is ordered by them).
namespace moe {
namespace {
std::atomic<uint64_t> g_launches{0}, g_block_calls{0}, g_pack_bytes{0};
}  // namespace
void note_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
void note_block_call() { g_block_calls.fetch_add(1, std::memory_order_relaxed); }
void note_pack_bytes(uint64_t n) { g_pack_bytes.fetch_add(n, std::memory_order_relaxed); }
}  // namespace moe

extern "C" {

void moe_stats_get(moe_stats* out) {
  if (!out) return;
  out->launches = moe::g_launches.load(std::memory_order_relaxed);
  out->block_calls = moe::g_block_calls.load(std::memory_order_relaxed);
  out->pack_bytes = moe::g_pack_bytes.load(std::memory_order_relaxed);
}

void moe_stats_reset(void) {
  moe::g_launches.store(0, std::memory_order_relaxed);
  moe::g_block_calls.store(0, std::memory_order_relaxed);
  moe::g_pack_bytes.store(0, std::memory_order_relaxed);
}

int moe_check_shape(const moe_layer_weights* w) { return shape_ok(w) ? 0 : (int)cudaErrorInvalidValue; }

size_t moe_workspace_bytes(const moe_layer_weights* w, int max_T) {
  if (!shape_ok(w) || max_T < 1) return 0;
  return layout_for(w, max_T).total;
}

int moe_workspace_init(void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  if (!workspace || workspace_bytes == 0) return (int)cudaErrorInvalidValue;
  return (int)cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream);
}

int moe_workspace_error(void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  if (!workspace || workspace_bytes < 512) return -(int)cudaErrorInvalidValue;
  const WsLayout L = ws_layout(256, 1, 1, 128, 128, 1);  // ticket/err offsets do not depend on the geometry
  uint32_t* errp = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + L.err);
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, errp, sizeof v, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(errp, 0, sizeof v, (cudaStream_t)stream);
  if (e != cudaSuccess) return -(int)e;
  return (int)v;
}

namespace {
// The fused single-launch decode kernel serves T <= kFusedMaxT unless the environment sets MOE_B200_FUSED=0
// (read once per process), which selects the three-kernel path.
bool fused_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("MOE_B200_FUSED");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

int block_forward_impl(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, float* hidden,
                       const uint16_t* attn_out, uint16_t* normed, const uint16_t* next_rms1, int T,
                       void* const* events, cudaStream_t s) {
  int rc = check_common(w, workspace, workspace_bytes, T);
  if (rc) return rc;
  if (!hidden || !attn_out || !normed || !weights_present(w, true, true, true)) return (int)cudaErrorInvalidValue;
  note_block_call();
  if (use_prefill(w, T)) {
    BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
    a.hidden = hidden;
    a.attn_out = attn_out;
    a.normed = normed;
    a.next_rms1 = next_rms1;
    cudaError_t e = events ? record_event(events[0], s) : cudaSuccess;
    if (e == cudaSuccess) e = prefill_block(a, s, events);
    return (int)e;
  }
  int fs = 0, frows = 0;
  size_t fsmem = 0;
  const bool lean = lean_config(*w, T);
  if (lean || (fused_enabled() && fused_config(*w, T, &fs, &fsmem, &frows))) {
    const WsLayout L = layout_for(w, T);
    BlockArgs a = make_args(w, workspace, L, T);
    a.hidden = hidden;
    a.attn_out = attn_out;
    a.normed = normed;
    a.next_rms1 = next_rms1;
    unsigned long long* gbar = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(workspace) + L.gbar);
    cudaError_t e = events ? record_event(events[0], s) : cudaSuccess;
    if (e == cudaSuccess)
      e = lean ? launch_lean_decode(a, gbar, next_rms1 != nullptr, s) : launch_fused_decode(a, gbar, next_rms1 != nullptr, s);
    for (int k = 1; k < 4 && events && e == cudaSuccess; ++k) e = record_event(events[k], s);
    return (int)e;
  }
  const int chunk = chunk_tokens(w);
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int Tc = std::min(chunk, T - t0);
    const WsLayout L = layout_for(w, Tc);
    BlockArgs a = make_args(w, workspace, L, Tc);
    const int64_t off = (int64_t)t0 * w->H;
    a.hidden = hidden + off;
    a.attn_out = attn_out + off;
    a.normed = normed + off;
    a.next_rms1 = next_rms1;
    const bool first = t0 == 0, last = t0 + chunk >= T;
    cudaError_t e = first && events ? record_event(events[0], s) : cudaSuccess;
    if (e == cudaSuccess) e = launch_route(a, true, true, s);
    if (e == cudaSuccess && last && events) e = record_event(events[1], s);
    if (e == cudaSuccess) e = launch_gate_up(a, true, true, s);
    if (e == cudaSuccess && last && events) e = record_event(events[2], s);
    if (e == cudaSuccess) e = launch_down_combine(a, 1 | 2 | 4 | (next_rms1 ? 8 : 0), s);
    if (e == cudaSuccess && last && events) e = record_event(events[3], s);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}
}  // namespace

int moe_block_forward(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, float* hidden,
                      const uint16_t* attn_out, uint16_t* normed, const uint16_t* next_rms1, int T,
                      moe_stream_t stream) {
  NvtxRange nvtx("moe_block_forward");
  return block_forward_impl(w, workspace, workspace_bytes, hidden, attn_out, normed, next_rms1, T, nullptr,
                            (cudaStream_t)stream);
}

int moe_block_forward_events(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, float* hidden,
                             const uint16_t* attn_out, uint16_t* normed, const uint16_t* next_rms1, int T,
                             void* const* events, moe_stream_t stream) {
  NvtxRange nvtx("moe_block_forward_events");
  if (!events) return (int)cudaErrorInvalidValue;
  return block_forward_impl(w, workspace, workspace_bytes, hidden, attn_out, normed, next_rms1, T, events,
                            (cudaStream_t)stream);
}

int moe_event_create(void** ev) {
  if (!ev) return (int)cudaErrorInvalidValue;
  return (int)cudaEventCreate(reinterpret_cast<cudaEvent_t*>(ev));
}

int moe_event_destroy(void* ev) { return (int)cudaEventDestroy(static_cast<cudaEvent_t>(ev)); }

int moe_event_elapsed_ms(void* start, void* stop, float* ms) {
  if (!ms) return (int)cudaErrorInvalidValue;
  return (int)cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(stop));
}

int moe_router_topk(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const uint16_t* normed,
                    float* logits, int32_t* idx, float* wts, int T, moe_stream_t stream) {
  NvtxRange nvtx("moe_router_topk");
  int rc = check_common(w, workspace, workspace_bytes, T);
  if (rc) return rc;
  if (!normed || !logits || !idx || !wts || !w->router) return (int)cudaErrorInvalidValue;
  if (use_prefill(w, T)) {
    BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
    a.normed = const_cast<uint16_t*>(normed);
    a.logits = logits;
    a.idx = idx;
    a.wts = wts;
    return (int)prefill_router(a, (cudaStream_t)stream);
  }
  const int chunk = chunk_tokens(w);
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int Tc = std::min(chunk, T - t0);
    BlockArgs a = make_args(w, workspace, layout_for(w, Tc), Tc);
    a.normed = const_cast<uint16_t*>(normed) + (int64_t)t0 * w->H;
    a.logits = logits + (int64_t)t0 * w->E;
    a.idx = idx + (int64_t)t0 * w->TOPK;
    a.wts = wts + (int64_t)t0 * w->TOPK;
    cudaError_t e = launch_route(a, false, false, (cudaStream_t)stream);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

int moe_routed_experts(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const uint16_t* normed,
                       const int32_t* idx, const float* wts, float* routed, uint16_t* inter_out, int T,
                       moe_stream_t stream) {
  NvtxRange nvtx("moe_routed_experts");
  int rc = check_common(w, workspace, workspace_bytes, T);
  if (rc) return rc;
  if (!normed || !idx || !wts || !routed || !weights_present(w, false, true, false)) return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  if (use_prefill(w, T)) {
    BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
    a.normed = const_cast<uint16_t*>(normed);
    a.idx = const_cast<int32_t*>(idx);
    a.wts = const_cast<float*>(wts);
    a.routed = routed;
    return (int)prefill_routed(a, inter_out, s);
  }
  const int chunk = chunk_tokens(w);
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int Tc = std::min(chunk, T - t0);
    BlockArgs a = make_args(w, workspace, layout_for(w, Tc), Tc);
    a.normed = const_cast<uint16_t*>(normed) + (int64_t)t0 * w->H;
    a.idx = const_cast<int32_t*>(idx) + (int64_t)t0 * w->TOPK;
    a.wts = const_cast<float*>(wts) + (int64_t)t0 * w->TOPK;
    a.routed = routed + (int64_t)t0 * w->H;
    if (inter_out) a.inter = inter_out + (int64_t)t0 * w->TOPK * w->I;
    cudaError_t e = launch_route_table(a, s);
    if (e == cudaSuccess) e = launch_gate_up(a, true, false, s);
    if (e == cudaSuccess) e = launch_down_combine(a, 1, s);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

int moe_shared_expert(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const uint16_t* normed,
                      uint16_t* sout, int T, moe_stream_t stream) {
  NvtxRange nvtx("moe_shared_expert");
  int rc = check_common(w, workspace, workspace_bytes, T);
  if (rc) return rc;
  if (!normed || !sout || !weights_present(w, false, false, true)) return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  if (use_prefill(w, T)) {
    BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
    a.normed = const_cast<uint16_t*>(normed);
    a.sout = sout;
    return (int)prefill_shared(a, s);
  }
  const int chunk = chunk_tokens(w);
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int Tc = std::min(chunk, T - t0);
    BlockArgs a = make_args(w, workspace, layout_for(w, Tc), Tc);
    a.normed = const_cast<uint16_t*>(normed) + (int64_t)t0 * w->H;
    a.sout = sout + (int64_t)t0 * w->H;
    cudaError_t e = launch_gate_up(a, false, true, s);
    if (e == cudaSuccess) e = launch_down_combine(a, 2, s);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

int moe_workspace_trace(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, int T, moe_trace* out) {
  if (!shape_ok(w) || !workspace || !out || T < 1 || (T > chunk_tokens(w) && !use_prefill(w, T)))
    return (int)cudaErrorInvalidValue;
  const int Tc = T;
  const WsLayout L = layout_for(w, Tc);
  if (workspace_bytes < L.total) return (int)cudaErrorInvalidValue;
  const BlockArgs a = make_args(w, workspace, L, Tc);
  out->logits = a.logits;
  out->idx = a.idx;
  out->wts = a.wts;
  out->routed = a.routed;
  out->sout = a.sout;
  out->gate = a.gate;
  const bool pf = use_prefill(w, T);
  out->sorted = pf ? a.sorted : nullptr;
  out->offsets = pf ? a.offsets : nullptr;
  return 0;
}

int moe_set_prefill_min_tokens(int T) {
  if (T < 0) return (int)cudaErrorInvalidValue;
  g_prefill_min.store(T, std::memory_order_relaxed);
  return 0;
}

const char* moe_version(void) { return "moe_b200 0.1 sm_100a"; }

}  // extern "C"

// ------------------------------------------------------------------ expert-parallel stages (include/moe_ep.h)

namespace {
bool ep_geometry_ok(const moe_layer_weights* w, int world) {
  if (!shape_ok(w) || world < 1 || world > kEpMaxWorld || w->E % world) return false;
  const int El = w->E / world;
  return El % 16 == 0 && El >= w->TOPK;
}
}  // namespace

extern "C" {

size_t moe_ep_record_bytes(const moe_layer_weights* w) {
  if (!shape_ok(w)) return 0;
  return (size_t)ep_record_bytes(w->H, w->TOPK);
}

int moe_ep_dispatch(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const float* hidden,
                    const uint16_t* attn_out, uint16_t* normed, int T, int world, void* send, int32_t* send_count,
                    int32_t* tok_pos, moe_stream_t stream) {
  NvtxRange nvtx("moe_ep_dispatch");
  if (!ep_geometry_ok(w, world) || !workspace || T < 1) return (int)cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 || workspace_bytes < layout_for(w, T).total)
    return (int)cudaErrorInvalidValue;
  if (!hidden || !attn_out || !normed || !send || !send_count || !tok_pos || !w->router || !w->rms2 ||
      !w->shared_gate || reinterpret_cast<uintptr_t>(send) % 16)
    return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
  a.hidden = const_cast<float*>(hidden);
  a.attn_out = attn_out;
  a.normed = normed;
  cudaError_t e = prefill_norm(a, s);
  if (e == cudaSuccess) e = prefill_router(a, s);
  if (e == cudaSuccess) e = ep_plan_pack(a, world, static_cast<uint8_t*>(send), send_count, tok_pos, s);
  return (int)e;
}

int moe_ep_experts(const moe_layer_weights* w_local, void* workspace, size_t workspace_bytes, const void* recv, int R,
                   uint16_t* part, moe_stream_t stream) {
  NvtxRange nvtx("moe_ep_experts");
  if (!shape_ok(w_local) || !prefill_supported(*w_local) || !workspace || R < 0) return (int)cudaErrorInvalidValue;
  if (!weights_present(w_local, false, true, false)) return (int)cudaErrorInvalidValue;
  if (R == 0) return 0;
  const WsLayout L = layout_for(w_local, std::max(R, kPrefillMinT));
  if (reinterpret_cast<uintptr_t>(workspace) % 256 || workspace_bytes < L.total) return (int)cudaErrorInvalidValue;
  if (!recv || !part || reinterpret_cast<uintptr_t>(recv) % 16 || reinterpret_cast<uintptr_t>(part) % 16)
    return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  BlockArgs a = make_args(w_local, workspace, L, R);
  a.normed = static_cast<uint16_t*>(const_cast<void*>(recv));
  a.xstride = ep_record_bytes(w_local->H, w_local->TOPK) / 2;
  a.routed16 = part;
  cudaError_t e = prefill_bits_clear(a, s);
  if (e == cudaSuccess) e = ep_mark(a, static_cast<const uint8_t*>(recv), nullptr, 0, s);
  if (e == cudaSuccess) e = prefill_routed_marked(a, s);
  return (int)e;
}

int moe_ep_combine(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, float* hidden,
                   const uint16_t* attn_out, const uint16_t* sout, uint16_t* normed, const uint16_t* next_rms1,
                   int T, int world, const int32_t* tok_pos, const uint16_t* ret, moe_stream_t stream) {
  NvtxRange nvtx("moe_ep_combine");
  if (!ep_geometry_ok(w, world) || !workspace || T < 1) return (int)cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 || workspace_bytes < layout_for(w, T).total)
    return (int)cudaErrorInvalidValue;
  if (!hidden || !attn_out || !sout || !normed || !tok_pos || !ret) return (int)cudaErrorInvalidValue;
  BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
  a.hidden = hidden;
  a.attn_out = attn_out;
  a.sout = const_cast<uint16_t*>(sout);
  a.normed = normed;
  a.next_rms1 = next_rms1;
  a.ep_pos = tok_pos;
  a.ep_ret = ret;
  a.ep_world = world;
  return (int)prefill_combine(a, (cudaStream_t)stream);
}

size_t moe_ep_recv_bytes(const moe_layer_weights* w, int world, int cap) {
  if (!ep_geometry_ok(w, world) || cap < 1) return 0;
  return ws_align((size_t)world * cap * ep_record_bytes(w->H, w->TOPK)) + ws_align(sizeof(int32_t) * world);
}

size_t moe_ep_rcount_offset(const moe_layer_weights* w, int world, int cap) {
  if (!ep_geometry_ok(w, world) || cap < 1) return 0;
  return ws_align((size_t)world * cap * ep_record_bytes(w->H, w->TOPK));
}

size_t moe_ep_ret_bytes(const moe_layer_weights* w, int world, int cap) {
  if (!ep_geometry_ok(w, world) || cap < 1) return 0;
  return (size_t)world * cap * w->H * sizeof(uint16_t);
}

static bool peers_ok(const moe_ep_peers* p, int world) {
  if (!p || p->rank < 0 || p->rank >= world || p->cap < 1) return false;
  for (int d = 0; d < world; ++d)
    if (!p->recv[d] || !p->rcount[d] || !p->ret[d] || reinterpret_cast<uintptr_t>(p->recv[d]) % 16 ||
        reinterpret_cast<uintptr_t>(p->ret[d]) % 16)
      return false;
  return true;
}

static EpPeers to_peers(const moe_ep_peers* p) {
  EpPeers q;
  memset(&q, 0, sizeof q);
  for (int d = 0; d < kEpMaxWorld; ++d) {
    q.recv[d] = static_cast<uint8_t*>(p->recv[d]);
    q.rcount[d] = p->rcount[d];
    q.ret[d] = p->ret[d];
  }
  q.rank = p->rank;
  q.cap = p->cap;
  return q;
}

int moe_ep_dispatch_peers(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const float* hidden,
                          const uint16_t* attn_out, uint16_t* normed, int T, int world, const moe_ep_peers* peers,
                          int32_t* send_count, int32_t* tok_pos, moe_stream_t stream) {
  NvtxRange nvtx("moe_ep_dispatch_peers");
  if (!ep_geometry_ok(w, world) || !workspace || T < 1 || !peers_ok(peers, world) || T > peers->cap)
    return (int)cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 || workspace_bytes < layout_for(w, T).total)
    return (int)cudaErrorInvalidValue;
  if (!hidden || !attn_out || !normed || !send_count || !tok_pos || !w->router || !w->rms2 || !w->shared_gate)
    return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  BlockArgs a = make_args(w, workspace, layout_for(w, T), T);
  a.hidden = const_cast<float*>(hidden);
  a.attn_out = attn_out;
  a.normed = normed;
  cudaError_t e = prefill_norm(a, s);
  if (e == cudaSuccess) e = prefill_router(a, s);
  if (e == cudaSuccess) e = ep_plan_pack_peers(a, world, to_peers(peers), send_count, tok_pos, s);
  return (int)e;
}

int moe_ep_experts_peers(const moe_layer_weights* w_local, void* workspace, size_t workspace_bytes, int world,
                         const moe_ep_peers* peers, moe_stream_t stream) {
  NvtxRange nvtx("moe_ep_experts_peers");
  if (!shape_ok(w_local) || !prefill_supported(*w_local) || !workspace || world < 1 || world > kEpMaxWorld ||
      !peers_ok(peers, world) || !weights_present(w_local, false, true, false))
    return (int)cudaErrorInvalidValue;
  const int R = world * peers->cap;
  const WsLayout L = layout_for(w_local, std::max(R, kPrefillMinT));
  if (reinterpret_cast<uintptr_t>(workspace) % 256 || workspace_bytes < L.total) return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  const EpPeers q = to_peers(peers);
  BlockArgs a = make_args(w_local, workspace, L, R);
  a.normed = reinterpret_cast<uint16_t*>(q.recv[q.rank]);
  a.xstride = ep_record_bytes(w_local->H, w_local->TOPK) / 2;
  cudaError_t e = prefill_bits_clear(a, s);
  if (e == cudaSuccess) e = ep_mark(a, q.recv[q.rank], q.rcount[q.rank], q.cap, s);
  if (e == cudaSuccess) e = prefill_routed_marked_gemms(a, s);
  if (e == cudaSuccess) e = ep_return_peers(a, world, q, s);
  return (int)e;
}

int moe_device_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return (int)cudaErrorInvalidValue;
  return (int)cudaMalloc(ptr, bytes);
}

int moe_device_free(void* ptr) { return (int)cudaFree(ptr); }

int moe_ipc_handle(void* ptr, void* handle64) {
  if (!ptr || !handle64) return (int)cudaErrorInvalidValue;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e == cudaSuccess) memcpy(handle64, &h, sizeof h);
  return (int)e;
}

int moe_ipc_open(const void* handle64, void** ptr) {
  if (!ptr || !handle64) return (int)cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof h);
  return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

int moe_ipc_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }

}  // extern "C"
