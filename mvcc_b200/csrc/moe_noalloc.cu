// moe_noalloc.cu -- moe_router_topk_noalloc: router + top-k for callers that cannot allocate device memory.
//
// Some hosts cannot hand this library a workspace: a serving runtime or plugin host that owns all device memory
// through its own allocator and reserves it at start-up, so nothing may call cudaMalloc after initialisation, and
// that has no workspace of ours to pass. For them this entry point runs the router kernel with its scratch (the
// self-wrapping ticket counter, the error word and the unique-expert table) in a fixed array in the library's own
// device memory instead of a caller-owned workspace. Logits, indices and weights still go to the caller's buffers.
//
// The array is a file-scope static __device__ object: every GPU that loads the library holds it (8 KiB) until the
// process exits. Host code cannot use the array's name as a device address (it is a host-side stand-in), so each
// call looks the address up with cudaGetSymbolAddress on the current device and checks the result; nothing is
// cached, so a device reset cannot leave a stale address behind. The first call on a device also loads the
// library's device code there, so it should come before any stream capture. All calls share the array and it keeps
// the last call's contents; each call clears the ticket and error word before its launches. Calls that overlap on the
// GPU (concurrent streams, or several host threads) race on the array and must be serialised by the caller.
//
// The router always runs the decode kernels (route_kernel: GEMV + the reference's top-k), chunk by chunk, whatever
// the prefill threshold. moe_router_topk_noalloc_error reads the array's error word back (and clears it) for the
// current device; the route kernel's own top-k cannot produce the invalid-expert index the word records, so it
// stays zero unless the kernels misbehave.
#include <cstring>

#include "moe_common.cuh"
#include "moe_decode.h"

namespace {

constexpr size_t kScratchBytes = 8192;  // the stated maximum; see moe_router_topk_noalloc

static __device__ __align__(256) uint8_t g_router_scratch[kScratchBytes];

// Scratch sections, in bytes from the start of the array.
struct ScratchLayout {
  size_t ticket, err, nuniq, uniq, uoff, upairs, total;
};

ScratchLayout scratch_layout(int E, int pairs) {
  ScratchLayout L;
  size_t o = 0;
  L.ticket = o; o = moe::ws_align(o + 16 * sizeof(uint32_t));
  L.err = o;    o = moe::ws_align(o + sizeof(uint32_t));
  L.nuniq = o;  o = moe::ws_align(o + sizeof(int32_t));
  L.uniq = o;   o = moe::ws_align(o + sizeof(int32_t) * (size_t)E);
  L.uoff = o;   o = moe::ws_align(o + sizeof(int32_t) * ((size_t)E + 1));
  L.upairs = o; o = moe::ws_align(o + sizeof(int32_t) * (size_t)pairs);
  L.total = o;
  return L;
}

// Device address of g_router_scratch on the current device.
cudaError_t scratch_address(uint8_t** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_router_scratch);
  if (e != cudaSuccess) return e;
  *out = static_cast<uint8_t*>(p);
  return cudaSuccess;
}

bool shape_ok(const moe_layer_weights* w) {
  if (!w || !w->router) return false;
  return moe_check_shape(w) == 0;
}

}  // namespace

extern "C" int moe_router_topk_noalloc(const moe_layer_weights* w, const uint16_t* normed, float* logits,
                                       int32_t* idx, float* wts, int T, moe_stream_t stream) {
  if (!shape_ok(w) || !normed || !logits || !idx || !wts || T < 1) return (int)cudaErrorInvalidValue;
  const int chunk = moe::decode_max_tokens(w->H, w->TOPK, w->I, w->Is);
  const ScratchLayout L = scratch_layout(w->E, chunk * w->TOPK);
  if (L.total > kScratchBytes) return (int)cudaErrorInvalidValue;  // larger than the static scratch
  uint8_t* base = nullptr;
  cudaError_t e = scratch_address(&base);
  if (e != cudaSuccess) return (int)e;
  const cudaStream_t s = (cudaStream_t)stream;
  e = cudaMemsetAsync(base, 0, L.nuniq, s);  // ticket and error word start at zero
  if (e != cudaSuccess) return (int)e;
  for (int t0 = 0; t0 < T; t0 += chunk) {
    const int Tc = T - t0 < chunk ? T - t0 : chunk;
    moe::BlockArgs a;
    memset(&a, 0, sizeof a);
    a.w = *w;
    a.T = Tc;
    a.normed = const_cast<uint16_t*>(normed) + (int64_t)t0 * w->H;
    a.logits = logits + (int64_t)t0 * w->E;
    a.idx = idx + (int64_t)t0 * w->TOPK;
    a.wts = wts + (int64_t)t0 * w->TOPK;
    a.ticket = reinterpret_cast<uint32_t*>(base + L.ticket);
    a.err = reinterpret_cast<uint32_t*>(base + L.err);
    a.nuniq = reinterpret_cast<int32_t*>(base + L.nuniq);
    a.uniq = reinterpret_cast<int32_t*>(base + L.uniq);
    a.uoff = reinterpret_cast<int32_t*>(base + L.uoff);
    a.upairs = reinterpret_cast<int32_t*>(base + L.upairs);
    e = moe::launch_route(a, false, false, s);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

extern "C" int moe_router_topk_noalloc_error(moe_stream_t stream) {
  uint8_t* base = nullptr;
  cudaError_t e = scratch_address(&base);
  if (e != cudaSuccess) return -(int)e;
  uint32_t* errp = reinterpret_cast<uint32_t*>(base + scratch_layout(1, 1).err);  // offset independent of the shape
  uint32_t v = 0;
  const cudaStream_t s = (cudaStream_t)stream;
  e = cudaMemcpyAsync(&v, errp, sizeof v, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(errp, 0, sizeof v, s);
  if (e != cudaSuccess) return -(int)e;
  return (int)v;
}
