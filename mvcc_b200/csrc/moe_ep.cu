// moe_ep.cu -- dispatch plan/pack and receive-side unpack of the expert-parallel MoE layer.
//
// The experts are sharded over `world` ranks, rank d owning the E / world consecutive experts starting at
// d * E / world. A token goes once to every rank that owns at least one of its TOPK experts, as one record: its
// normed activations plus, per slot, the expert's id on that rank (-1 when the slot's expert lives elsewhere) and
// the routing weight. The receiving rank runs its experts over the records (the prefill GEMMs) and returns one
// partial row per record (its slots summed in slot order in fp32, then rounded to bf16: half the bytes of an fp32
// row on the return exchange); the source sums the partials of a token in rank order in fp32 (moe_prefill.cu's
// combine).
// The exchange either packs the records into one send buffer grouped by destination (for an all-to-all library
// call), or, in peer mode, stores each record straight into the destination rank's receive buffer and each partial
// row straight into the source rank's return buffer through peer-memory mappings (NVLink), every such store
// followed by a system-scope fence so that a collective barrier after the kernel publishes it.
// The reference runs the block on one GPU (qwen.cu:429-448); this split has no counterpart there.
#include "moe_device.cuh"
#include "moe_ep.h"

namespace moe {

constexpr int kPlanThreads = 1024;
constexpr int kPackThreads = 128;

__device__ __forceinline__ uint32_t dest_mask(const int32_t* idx, int K, int E, int El) {
  uint32_t m = 0;
  for (int k = 0; k < K; ++k) {
    const int e = idx[k];
    if ((unsigned)e < (unsigned)E) m |= 1u << (e / El);
  }
  return m;
}

// One CTA: per-destination counts of the tokens in a contiguous token range per thread, block scans, then each
// token's record index per destination (-1 = not sent).
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const BlockArgs a, int world, int32_t* tok_pos,
                                                               int32_t* send_count, int peer_mode, EpPeers peers) {
  __shared__ int sm[32];
  const int T = a.T, K = a.w.TOPK, E = a.w.E, El = E / world, tid = threadIdx.x;
  const int per = (T + kPlanThreads - 1) / kPlanThreads;
  const int t0 = min(T, tid * per), t1 = min(T, t0 + per);
  int c[kEpMaxWorld];
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) c[d] = 0;
  for (int t = t0; t < t1; ++t) {
    const uint32_t m = dest_mask(a.idx + (int64_t)t * K, K, E, El);
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) c[d] += (m >> d) & 1u;
  }
  int run[kEpMaxWorld], off[kEpMaxWorld];
  int o = 0;
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) {
    int tot;
    run[d] = block_excl_scan(c[d], sm, &tot);
    off[d] = peer_mode ? d * peers.cap : o;
    o += tot;
    if (tid == 0 && d < world) {
      send_count[d] = tot;
      if (peer_mode) {
        peers.rcount[d][peers.rank] = tot;
        __threadfence_system();
      }
    }
  }
  for (int t = t0; t < t1; ++t) {
    const uint32_t m = dest_mask(a.idx + (int64_t)t * K, K, E, El);
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) {
      if (d >= world) break;
      const bool on = (m >> d) & 1u;
      tok_pos[(int64_t)t * world + d] = on ? off[d] + run[d] : -1;
      run[d] += on;
    }
  }
}

// One CTA per token: its normed row (held in registers) and per-destination meta into each of its records.
__global__ void __launch_bounds__(kPackThreads) ep_pack_kernel(const BlockArgs a, int world, int rec_bytes,
                                                               uint8_t* send, const int32_t* tok_pos, int peer_mode,
                                                               EpPeers peers) {
  const int t = blockIdx.x, tid = threadIdx.x, H = a.w.H, K = a.w.TOPK, E = a.w.E, El = E / world;
  const int nv = H / 8;  // 16-byte chunks of a row (H <= 4096: at most 4 per thread)
  const uint4* src = reinterpret_cast<const uint4*>(a.normed + (int64_t)t * H);
  uint4 v[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tid + r * kPackThreads;
    if (i < nv) v[r] = src[i];
  }
  int e = -1;
  float wt = 0.f;
  if (tid < K) {
    e = a.idx[(int64_t)t * K + tid];
    wt = a.wts[(int64_t)t * K + tid];
  }
  for (int d = 0; d < world; ++d) {
    const int pos = tok_pos[(int64_t)t * world + d];
    if (pos < 0) continue;
    uint8_t* rec = peer_mode ? peers.recv[d] + ((int64_t)peers.rank * peers.cap + (pos - d * peers.cap)) * rec_bytes
                             : send + (int64_t)pos * rec_bytes;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = tid + r * kPackThreads;
      if (i < nv) reinterpret_cast<uint4*>(rec)[i] = v[r];
    }
    if (tid < K) {
      const bool here = (unsigned)e < (unsigned)E && e / El == d;
      reinterpret_cast<int32_t*>(rec + 2 * H)[tid] = here ? e - d * El : -1;
      reinterpret_cast<float*>(rec + 2 * H + 4 * K)[tid] = wt;
    }
  }
  if (peer_mode) __threadfence_system();
}

// One thread per (record, slot): meta into a.idx / a.wts, local slots into the pair bitmaps.
__global__ void __launch_bounds__(256) ep_mark_kernel(const BlockArgs a, const uint8_t* recv, int rec_bytes,
                                                      const int32_t* rcount, int cap) {
  const int K = a.w.TOPK, H = a.w.H, P = a.T * K;
  const int p = blockIdx.x * 256 + threadIdx.x;
  if (p >= P) return;
  const int r = p / K, k = p - r * K;
  if (rcount) {  // rows past a source's count hold no record
    const int src = r / cap;
    if (r - src * cap >= __ldcg(rcount + src)) {
      a.idx[p] = -1;
      a.wts[p] = 0.f;
      return;
    }
  }
  const uint8_t* rec = recv + (int64_t)r * rec_bytes;
  const int e = reinterpret_cast<const int32_t*>(rec + 2 * H)[k];
  a.idx[p] = e;
  a.wts[p] = reinterpret_cast<const float*>(rec + 2 * H + 4 * K)[k];
  if (e == -1) return;
  if ((unsigned)e >= (unsigned)a.w.E) {
    atomicOr(a.err, (uint32_t)MOE_ERR_EXPERT_INDEX);
    return;
  }
  atomicOr(a.bits + (int64_t)e * a.nwp + (p >> 5), 1u << (p & 31));
}

// One CTA per record row r = src * cap + j of the receive buffer (peer mode): rows with a record sum their valid
// slots in slot order (as prefill_combine_kernel's mode 1) and store the row, rounded to bf16, into rank src's
// return buffer.
__global__ void __launch_bounds__(256) ep_return_kernel(const BlockArgs a, int world, EpPeers peers) {
  const int r = blockIdx.x, tid = threadIdx.x, H = a.w.H, K = a.w.TOPK;
  const int src = r / peers.cap, j = r - src * peers.cap;
  if (j >= __ldcg(peers.rcount[peers.rank] + src)) return;
  bool ok[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) ok[k] = k < K && (unsigned)a.idx[(int64_t)r * K + k] < (unsigned)a.w.E;
  uint2* dst = reinterpret_cast<uint2*>(peers.ret[src] + ((int64_t)peers.rank * peers.cap + j) * H);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int i = tid + q * 256;
    if (i >= H / 4) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (!ok[k]) continue;
      const float4 v = __ldcs(reinterpret_cast<const float4*>(a.slot + ((int64_t)r * K + k) * H) + i);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    dst[i] = make_uint2((uint32_t)f2bf(acc.x) | ((uint32_t)f2bf(acc.y) << 16),
                        (uint32_t)f2bf(acc.z) | ((uint32_t)f2bf(acc.w) << 16));
  }
  __threadfence_system();
}

static const EpPeers kNoPeers = {};

cudaError_t ep_plan_pack(const BlockArgs& a, int world, uint8_t* send, int32_t* send_count, int32_t* tok_pos,
                         cudaStream_t s) {
  ep_plan_kernel<<<1, kPlanThreads, 0, s>>>(a, world, tok_pos, send_count, 0, kNoPeers);
  cudaError_t e = launched(cudaGetLastError());
  if (e != cudaSuccess) return e;
  ep_pack_kernel<<<a.T, kPackThreads, 0, s>>>(a, world, ep_record_bytes(a.w.H, a.w.TOPK), send, tok_pos, 0,
                                              kNoPeers);
  return launched(cudaGetLastError());
}

cudaError_t ep_plan_pack_peers(const BlockArgs& a, int world, const EpPeers& peers, int32_t* send_count,
                               int32_t* tok_pos, cudaStream_t s) {
  ep_plan_kernel<<<1, kPlanThreads, 0, s>>>(a, world, tok_pos, send_count, 1, peers);
  cudaError_t e = launched(cudaGetLastError());
  if (e != cudaSuccess) return e;
  ep_pack_kernel<<<a.T, kPackThreads, 0, s>>>(a, world, ep_record_bytes(a.w.H, a.w.TOPK), nullptr, tok_pos, 1,
                                              peers);
  return launched(cudaGetLastError());
}

cudaError_t ep_mark(const BlockArgs& a, const uint8_t* recv, const int32_t* rcount, int cap, cudaStream_t s) {
  const int P = a.T * a.w.TOPK;
  ep_mark_kernel<<<(P + 255) / 256, 256, 0, s>>>(a, recv, ep_record_bytes(a.w.H, a.w.TOPK), rcount, cap);
  return launched(cudaGetLastError());
}

cudaError_t ep_return_peers(const BlockArgs& a, int world, const EpPeers& peers, cudaStream_t s) {
  ep_return_kernel<<<world * peers.cap, 256, 0, s>>>(a, world, peers);
  return launched(cudaGetLastError());
}

}  // namespace moe
