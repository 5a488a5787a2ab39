// moe_fused.cu -- fused persistent decode kernel of the MoE block for T <= 8 tokens: one cooperative launch does
// qwen.cu:429-448 end to end.
//
// One CTA per SM, 16 warps. Weight bytes move with bulk asynchronous copies (cp.async.bulk, completion counted on
// shared-memory mbarriers) issued by one thread, a few large contiguous copies per CTA, so no warp stalls issuing
// loads and every byte is requested as soon as its dependency allows:
//   entry     bulk copies of the routing-independent weights this CTA owns: router rows (rows 2c, 2c + 1 -> CTA c;
//             the shared gate vector is row E), shared-expert gate/up row pairs (pairs 4c .. 4c + 3 -> CTA c) and
//             the shared-expert down rows of the CTA's output rows [h0, h1);
//   phase R   RMSNorm of every token (every CTA, into shared memory), router logits of the CTA's rows -> global;
//             arrive at grid barrier 1; the shared-expert gate/up pairs while the barrier settles; wait;
//   phase G   every CTA runs the reference's top-k on all logits itself (one warp per token, warp reductions) and
//             one warp builds the unique-expert table; the CTA's share of the routed gate/up jobs (contiguous row
//             ranges of each unique expert) and its down rows (rows [h0, h1) of every unique expert) form a list
//             of chunks that stream through a ring of shared-memory stages: gate/up chunks are consumed one job
//             per warp, `inter` -> global; the last warp to finish a stage refills it with the next chunk, so the
//             down rows arrive while phase G still runs; grid barrier 2;
//   phase D   stage every pair's `inter` and the shared `sinter`; each warp reduces one output row h over every
//             unique expert (weighted per pair) and the shared expert, and applies the gated residual combine;
//             the last CTA to finish (ticket) optionally applies the next layer's RMSNorm.
// Grid barriers use a monotone 64-bit arrival counter in the workspace (each launch adds exactly 2 x G arrivals,
// so the targets follow from its value at launch start) and bounded spins; stage waits are bounded by the global
// timer. A wait that gives up records MOE_ERR_BARRIER in the error word; the CTA skips the remaining work, still
// arrives at the grid barriers, and before returning waits (bounded) for every copy it issued. The launch is
// cooperative, so all CTAs are co-resident, and a programmatic dependent launch: the entry (barrier setup and the
// weight copies) overlaps the previous kernel's tail, everything that reads its outputs or the workspace follows
// griddepcontrol.wait, and phase D lets the next kernel start its own entry. Per-job reductions and numerics are
// those of the three-kernel path (moe_decode.cu).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "moe_fused.h"
#include "moe_sync.cuh"

namespace moe {

constexpr int kFW = 16;
constexpr int kFThreads = kFW * 32;
constexpr int kSgu = 4;                            // shared gate/up pairs per CTA (Is <= 4 x grid)
constexpr int kRouterRows = 2;                     // router rows per CTA (E + 1 <= 2 x grid)
constexpr int kMaxStages = 6;                      // ring stages
constexpr int kMaxChunks = 96;                     // gate/up + down chunks of one CTA

struct FusedArgs {
  BlockArgs a;
  unsigned long long* gbar;  // grid-barrier arrival counter
  int stages;                // ring stages
  int stage_bytes;           // bytes per stage
  int cjobs;                 // gate/up jobs (row pairs) per chunk, at most kFW
  int kd;                    // experts per down chunk
  int rows_per_cta;          // output rows h per CTA (at most kFW)
  int next_norm;             // apply the next layer's RMSNorm
};

// Shared-memory carve-up (bytes), identical on host and device.
struct FusedSmem {
  size_t xs, sinter, router, sgu, sdn, acc, ring, total;
};

__host__ __device__ inline size_t f_align(size_t x) { return (x + 127) & ~(size_t)127; }
__host__ __device__ inline int a16(int x) { return (x + 15) & ~15; }

__host__ __device__ inline FusedSmem fused_smem(int T, int H, int TOPK, int I, int Is, int rows_per_cta,
                                                 int stage_bytes, int stages) {
  FusedSmem L;
  size_t o = 0;
  const size_t xs = (size_t)T * H * 4, inter = (size_t)T * TOPK * inter_stride(I) * 2;
  L.xs = o;     o = f_align(o + (xs > inter ? xs : inter));
  L.sinter = o; o = f_align(o + (size_t)T * Is * 2);
  L.router = o; o = f_align(o + (size_t)kRouterRows * H * 2);
  L.sgu = o;    o = f_align(o + (size_t)kSgu * 2 * H * 2);
  L.sdn = o;    o = f_align(o + (size_t)rows_per_cta * Is * 2);
  L.acc = o;    o = f_align(o + (size_t)kFW * T * 32 * 4);
  L.ring = o;   o = f_align(o + (size_t)stages * stage_bytes);
  L.total = o;
  return L;
}

// Layout of one stage. Gate/up chunk of n <= C consecutive jobs, in one expert or running on into the next (two
// segments): gate rows [C][H/2], up rows [C][H/2], then the gate and the up scale rows, each segment's copied as the
// 16-byte aligned superset of its [n_k][H/G] fp16, the second segment's after the first's. Down chunk of n <= kd experts: rows
// [kd][rpc][I/2], then per expert its scale rows [rpc][I/G] fp16 as an aligned superset.
__host__ __device__ inline int gate_scale_region(int C, int H, int G) { return a16(C * (H / G) * 2) + 64; }
__host__ __device__ inline int down_scale_region(int rpc, int I, int G) { return a16(rpc * (I / G) * 2) + 32; }
__host__ __device__ inline int gate_stage_bytes(int C, int H, int G) {
  return 2 * C * (H / 2) + 2 * gate_scale_region(C, H, G);
}
__host__ __device__ inline int down_stage_bytes(int kd, int rpc, int I, int G) {
  return kd * rpc * (I / 2) + kd * down_scale_region(rpc, I, G);
}

// The unique-expert table in one warp (same contents and order as build_unique in moe_decode.cu): the P <= 64 pairs
// sorted by (expert, pair index) with a bitonic network over 64 keys (element i in lane i % 32, register i / 32);
// uniq[u] the ascending experts, uoff[u] their first sorted position, upairs/ptok the sorted pairs and their tokens.
// Invalid indices sort last and are dropped.
__device__ void table_warp(const int32_t* idx_s, int P, int E, int K, int* uniq_s, int* uoff_s, int* upairs_s,
                           int* ptok_s, int* pu_s, int* nuniq_s) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  uint32_t v0, v1;
  {
    const int e0 = lane < P ? idx_s[lane] : -1, e1 = lane + 32 < P ? idx_s[lane + 32] : -1;
    v0 = (lane < P && e0 >= 0 && e0 < E) ? ((uint32_t)e0 << 6) | (uint32_t)lane : 0xffffffffu;
    v1 = (lane + 32 < P && e1 >= 0 && e1 < E) ? ((uint32_t)e1 << 6) | (uint32_t)(lane + 32) : 0xffffffffu;
  }
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint32_t o0, o1;
      if (j == 32) {
        o0 = v1;
        o1 = v0;
      } else {
        o0 = __shfl_xor_sync(0xffffffffu, v0, j);
        o1 = __shfl_xor_sync(0xffffffffu, v1, j);
      }
      const int i0 = lane, i1 = lane + 32;
      const bool keep_lo0 = ((i0 & j) == 0) == ((i0 & k) == 0), keep_lo1 = ((i1 & j) == 0) == ((i1 & k) == 0);
      v0 = keep_lo0 ? min(v0, o0) : max(v0, o0);
      v1 = keep_lo1 ? min(v1, o1) : max(v1, o1);
    }
  }
  // v0 / v1 hold sorted positions lane / lane + 32
  const bool valid0 = v0 != 0xffffffffu, valid1 = v1 != 0xffffffffu;
  const int e0 = (int)(v0 >> 6), e1 = (int)(v1 >> 6);
  int prev0 = __shfl_up_sync(0xffffffffu, e0, 1);
  int prev1 = __shfl_up_sync(0xffffffffu, e1, 1);
  const int last0 = __shfl_sync(0xffffffffu, e0, 31);
  if (lane == 0) {
    prev0 = -1;
    prev1 = last0;
  }
  const bool f0 = valid0 && e0 != prev0, f1 = valid1 && e1 != prev1;
  const uint32_t b0 = __ballot_sync(0xffffffffu, f0), b1 = __ballot_sync(0xffffffffu, f1);
  const uint32_t le = 0xffffffffu >> (31 - lane);
  const int u0 = __popc(b0 & le) - 1, u1 = __popc(b0) + __popc(b1 & le) - 1;
  const int nvalid = __popc(__ballot_sync(0xffffffffu, valid0)) + __popc(__ballot_sync(0xffffffffu, valid1));
  if (f0) {
    uniq_s[u0] = e0;
    uoff_s[u0] = lane;
  }
  if (f1) {
    uniq_s[u1] = e1;
    uoff_s[u1] = lane + 32;
  }
  if (valid0) {
    const int p = (int)(v0 & 63);
    upairs_s[lane] = p;
    ptok_s[lane] = p / K;
    pu_s[lane] = u0;
  }
  if (valid1) {
    const int p = (int)(v1 & 63);
    upairs_s[lane + 32] = p;
    ptok_s[lane + 32] = p / K;
    pu_s[lane + 32] = u1;
  }
  if (lane == 0) {
    const int U = __popc(b0) + __popc(b1);
    *nuniq_s = U;
    uoff_s[U] = nvalid;
  }
}

// ------------------------------------------------------------------ per-job arithmetic (three-kernel path order)

// One routed gate/up row pair (gate row i and up row I + i of unique expert uix) for every pair routed to it; same
// reduction as compute_routed in moe_decode.cu.
__device__ __forceinline__ void fused_gate_job(const BlockArgs& a, const float* xs, const uint8_t* grow,
                                               const uint8_t* urow, const uint16_t* gsc, const uint16_t* usc, int uix,
                                               int i, const int* uoff_s, const int* upairs_s, const int* ptok_s,
                                               int gshift, const Nib8Magic& M) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, I = a.w.I, nch = H >> 5;
  for (int p = uoff_s[uix]; p < uoff_s[uix + 1]; ++p) {
    const int pair = upairs_s[p];
    const float* xt = xs + ptok_s[p] * H;
    float g = 0.f, u = 0.f;
    for (int c = lane; c < nch; c += 32) {
      const uint4 gq = *reinterpret_cast<const uint4*>(grow + c * 16);
      const uint4 uq = *reinterpret_cast<const uint4*>(urow + c * 16);
      const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w}, uw[4] = {uq.x, uq.y, uq.z, uq.w};
      Nib8Acc ag, au;
      nib8_zero(ag);
      nib8_zero(au);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        u64 x01, x23, x45, x67;
        lds_pairs(xt + ((q * 2) * nch + c) * 4, x01, x23);
        lds_pairs(xt + ((q * 2 + 1) * nch + c) * 4, x45, x67);
        nib8x2(gw[q], x01, x23, x45, x67, M, ag);
        nib8x2(uw[q], x01, x23, x45, x67, M, au);
      }
      g = fmaf(nib8_fold(ag), h2f(gsc[c >> gshift]), g);
      u = fmaf(nib8_fold(au), h2f(usc[c >> gshift]), u);
    }
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) a.inter[(int64_t)pair * I + i] = f2bf(silu(g) * u);
    __syncwarp();
  }
}

// Two gate/up jobs of the same unique expert (rows i0 and i1) on one warp: the activation loads are shared, each
// job's arithmetic is that of fused_gate_job.
__device__ __forceinline__ void fused_gate_job2(const BlockArgs& a, const float* xs, const uint8_t* grow0,
                                                const uint8_t* urow0, const uint16_t* gsc0, const uint16_t* usc0,
                                                const uint8_t* grow1, const uint8_t* urow1, const uint16_t* gsc1,
                                                const uint16_t* usc1, int uix, int i0, int i1, const int* uoff_s,
                                                const int* upairs_s, const int* ptok_s, int gshift,
                                                const Nib8Magic& M) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, I = a.w.I, nch = H >> 5;
  for (int p = uoff_s[uix]; p < uoff_s[uix + 1]; ++p) {
    const int pair = upairs_s[p];
    const float* xt = xs + ptok_s[p] * H;
    float g0 = 0.f, u0 = 0.f, g1 = 0.f, u1 = 0.f;
    for (int c = lane; c < nch; c += 32) {
      const uint4 gq0 = *reinterpret_cast<const uint4*>(grow0 + c * 16);
      const uint4 uq0 = *reinterpret_cast<const uint4*>(urow0 + c * 16);
      const uint4 gq1 = *reinterpret_cast<const uint4*>(grow1 + c * 16);
      const uint4 uq1 = *reinterpret_cast<const uint4*>(urow1 + c * 16);
      const uint32_t gw0[4] = {gq0.x, gq0.y, gq0.z, gq0.w}, uw0[4] = {uq0.x, uq0.y, uq0.z, uq0.w};
      const uint32_t gw1[4] = {gq1.x, gq1.y, gq1.z, gq1.w}, uw1[4] = {uq1.x, uq1.y, uq1.z, uq1.w};
      Nib8Acc ag0, au0, ag1, au1;
      nib8_zero(ag0);
      nib8_zero(au0);
      nib8_zero(ag1);
      nib8_zero(au1);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        u64 x01, x23, x45, x67;
        lds_pairs(xt + ((q * 2) * nch + c) * 4, x01, x23);
        lds_pairs(xt + ((q * 2 + 1) * nch + c) * 4, x45, x67);
        nib8x2(gw0[q], x01, x23, x45, x67, M, ag0);
        nib8x2(uw0[q], x01, x23, x45, x67, M, au0);
        nib8x2(gw1[q], x01, x23, x45, x67, M, ag1);
        nib8x2(uw1[q], x01, x23, x45, x67, M, au1);
      }
      g0 = fmaf(nib8_fold(ag0), h2f(gsc0[c >> gshift]), g0);
      u0 = fmaf(nib8_fold(au0), h2f(usc0[c >> gshift]), u0);
      g1 = fmaf(nib8_fold(ag1), h2f(gsc1[c >> gshift]), g1);
      u1 = fmaf(nib8_fold(au1), h2f(usc1[c >> gshift]), u1);
    }
    g0 = warp_sum(g0);
    u0 = warp_sum(u0);
    g1 = warp_sum(g1);
    u1 = warp_sum(u1);
    if (lane == 0) {
      a.inter[(int64_t)pair * I + i0] = f2bf(silu(g0) * u0);
      a.inter[(int64_t)pair * I + i1] = f2bf(silu(g1) * u1);
    }
    __syncwarp();
  }
}

// d += sum over the 4 signed bytes of w (k ascending) of byte * x[i], as gemv_i8_kernel's char4 loop
// (kernels.cuh:250-256) accumulates one 32-input chunk.
__device__ __forceinline__ float i8x4_dot(uint32_t w, const float* x, float d) {
#pragma unroll
  for (int i = 0; i < 4; ++i) d = fmaf((float)((int32_t)(w << (24 - 8 * i)) >> 24), x[i], d);
  return d;
}

// Shared-memory slot of a 16-byte aligned superset of `rows` scale rows of `bytes` each.
__host__ __device__ inline int scale_slot(int rows, int bytes) { return a16(rows * bytes) + 16; }

// Chunk list entry: kind 0 = gate/up jobs i0 .. i0 + n - 1 of unique expert a; kind 1 = down rows of unique experts
// a .. a + n - 1.
struct Chunk {
  int kind, a, i0, n;
};

__global__ void __launch_bounds__(kFThreads, 1) moe_fused_decode_kernel(FusedArgs f) {
  extern __shared__ __align__(128) uint8_t smem[];
  const BlockArgs& a = f.a;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, H = a.w.H, E = a.w.E, K = a.w.TOPK, I = a.w.I, Is = a.w.Is, G = a.w.G;
  const int P = T * K, nch = H >> 5, nvs = Is >> 3;
  const int grid = gridDim.x, cta = blockIdx.x;
  const int S = f.stages, SB = f.stage_bytes, C = f.cjobs, rpc = f.rows_per_cta;
  const FusedSmem L = fused_smem(T, H, K, I, Is, rpc, SB, S);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  uint16_t* sinter_s = reinterpret_cast<uint16_t*>(smem + L.sinter);
  uint8_t* router_s = smem + L.router;
  uint8_t* sgu_s = smem + L.sgu;
  uint8_t* sdn_s = smem + L.sdn;
  float* acc_s = reinterpret_cast<float*>(smem + L.acc);
  uint8_t* ring = smem + L.ring;
  __shared__ __align__(8) uint64_t full_b[kMaxStages];
  __shared__ __align__(8) uint64_t rbar, sbar;
  __shared__ int cnt_s[kMaxStages], issued_s[kMaxStages];
  __shared__ Chunk chunk_s[kMaxChunks];
  __shared__ float red[32];
  __shared__ int32_t idx_s[64];
  __shared__ float wts_s[64];
  __shared__ int uniq_s[64], uoff_s[65], upairs_s[64], ptok_s[64], pu_s[64];
  __shared__ int nuniq_s, nchunks_s, ngate_s, ok_s, is_last, abort_s;
  __shared__ unsigned long long base_s;
  const int h0 = cta * rpc, h1 = min(H, h0 + rpc);
  const int rowb = H >> 1, sgb = (H / G) * 2;   // gate/up: row bytes, scale bytes per row
  const int drowb = I >> 1, dsb = (I / G) * 2;  // down: row bytes, scale bytes per row
  const int nrows = E + 1;
  const uint8_t* gscale = reinterpret_cast<const uint8_t*>(a.w.exp_gu_s);
  const uint8_t* dscale = reinterpret_cast<const uint8_t*>(a.w.exp_dn_s);
  // int8 shared expert (optional): rows, scales, scale bytes per row of gate/up and down, 32-input chunks per group
  const bool sh8 = a.w.shared_gate_up_q8 != nullptr;
  const uint8_t* q8g = reinterpret_cast<const uint8_t*>(a.w.shared_gate_up_q8);
  const uint8_t* s8g = reinterpret_cast<const uint8_t*>(a.w.shared_gate_up_s8);
  const uint8_t* q8d = reinterpret_cast<const uint8_t*>(a.w.shared_down_q8);
  const uint8_t* s8d = reinterpret_cast<const uint8_t*>(a.w.shared_down_s8);
  const int g8 = sh8 ? a.w.shared_group : 32;
  const int sgs8 = (H / g8) * 2, dss8 = (Is / g8) * 2, cshift8 = __ffs(g8) - 6;

  // Entry: barriers and the routing-independent weight copies touch only this CTA's shared memory and read only
  // weights, so under programmatic dependent launch they overlap the previous kernel's tail; everything after
  // griddepcontrol.wait may read that kernel's outputs (hidden) and reuses the workspace.
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_b[s], 1);
      cnt_s[s] = 0;
      issued_s[s] = 0;
    }
    mbar_init(&rbar, 1);
    mbar_init(&sbar, 1);
    abort_s = 0;
    mbar_fence_init();
    // ---- entry: routing-independent weights of this CTA
    // router rows [r0, r1) of this CTA, contiguous in the router matrix up to row E (the shared gate vector)
    const int r0 = min(nrows, kRouterRows * cta), r1 = min(nrows, r0 + kRouterRows), re = min(r1, E);
    expect_tx(&rbar, (uint32_t)((r1 - r0) * H * 2));
    if (re > r0) bulk_g2s(router_s, a.w.router + (int64_t)r0 * H, (re - r0) * H * 2, &rbar);
    if (r1 > re) bulk_g2s(router_s + (size_t)(re - r0) * H * 2, a.w.shared_gate, H * 2, &rbar);
    // shared-expert pairs [j0, j1): gate rows j0 .. j1 - 1 and up rows Is + j0 .. Is + j1 - 1, one copy each
    const int j0 = min(Is, kSgu * cta), j1 = min(Is, j0 + kSgu);
    if (sh8) {
      // int8 shared expert: gate q rows [kSgu][H], up q rows [kSgu][H], then their scale rows (aligned supersets);
      // down q rows [rpc][Is], then their scale rows
      uint32_t tx = 0;
      if (j1 > j0)
        tx += 2 * (j1 - j0) * H + span_bytes(s8g + (int64_t)j0 * sgs8, (j1 - j0) * sgs8) +
              span_bytes(s8g + (int64_t)(Is + j0) * sgs8, (j1 - j0) * sgs8);
      if (h0 < h1) tx += (h1 - h0) * Is + span_bytes(s8d + (int64_t)h0 * dss8, (h1 - h0) * dss8);
      expect_tx(&sbar, tx);
      if (j1 > j0) {
        bulk_g2s(sgu_s, q8g + (int64_t)j0 * H, (j1 - j0) * H, &sbar);
        bulk_g2s(sgu_s + (size_t)kSgu * H, q8g + (int64_t)(Is + j0) * H, (j1 - j0) * H, &sbar);
        bulk_span(sgu_s + (size_t)2 * kSgu * H, s8g + (int64_t)j0 * sgs8, (j1 - j0) * sgs8, &sbar);
        bulk_span(sgu_s + (size_t)2 * kSgu * H + scale_slot(kSgu, sgs8), s8g + (int64_t)(Is + j0) * sgs8,
                  (j1 - j0) * sgs8, &sbar);
      }
      if (h0 < h1) {
        bulk_g2s(sdn_s, q8d + (int64_t)h0 * Is, (h1 - h0) * Is, &sbar);
        bulk_span(sdn_s + (size_t)rpc * Is, s8d + (int64_t)h0 * dss8, (h1 - h0) * dss8, &sbar);
      }
    } else {
      expect_tx(&sbar, (uint32_t)(2 * (j1 - j0) * H * 2 + (h0 < h1 ? (h1 - h0) * Is * 2 : 0)));
      if (j1 > j0) {
        bulk_g2s(sgu_s, a.w.shared_gate_up + (int64_t)j0 * H, (j1 - j0) * H * 2, &sbar);
        bulk_g2s(sgu_s + (size_t)kSgu * H * 2, a.w.shared_gate_up + (int64_t)(Is + j0) * H, (j1 - j0) * H * 2,
                 &sbar);
      }
      if (h0 < h1) bulk_g2s(sdn_s, a.w.shared_down + (int64_t)h0 * Is, (h1 - h0) * Is * 2, &sbar);
    }
  }
  uint2 pre_w[2];  // the norm weights: read only weights, so requested before griddepcontrol.wait
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = tid + r * kFThreads;
    if (i < H / 4) pre_w[r] = reinterpret_cast<const uint2*>(a.w.rms2)[i];
  }
  cta_sync();
  pdl_wait();
  unsigned long long gb = 0;  // thread 0: the barrier counter at entry, consumed before the first arrival
  if (tid == 0) gb = ld_relaxed_u64(f.gbar);
  float4 pre_h[2];  // token 0's activations, requested before the norm's reduction needs them
  uint2 pre_d[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = tid + r * kFThreads;
    if (i < H / 4) {
      pre_h[r] = reinterpret_cast<const float4*>(a.hidden)[i];
      pre_d[r] = reinterpret_cast<const uint2*>(a.attn_out)[i];
    }
  }

  // ---- phase R: RMSNorm of every token into xs (fp32, permuted); CTA 0 writes `normed`
  for (int t = 0; t < T; ++t) {
    const float4* hr = reinterpret_cast<const float4*>(a.hidden + (int64_t)t * H);
    const uint2* dr = reinterpret_cast<const uint2*>(a.attn_out + (int64_t)t * H);
    float4 hv[2];
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {  // H <= 4096 = 2 x 512 threads x 4
      const int i = tid + r * kFThreads;
      if (i < H / 4) {
        const uint2 d = t == 0 ? pre_d[r] : dr[i];
        hv[r] = t == 0 ? pre_h[r] : hr[i];
        hv[r].x += lo_bf(d.x);
        hv[r].y += hi_bf(d.x);
        hv[r].z += lo_bf(d.y);
        hv[r].w += hi_bf(d.y);
        ss += hv[r].x * hv[r].x;
        ss += hv[r].y * hv[r].y;
        ss += hv[r].z * hv[r].z;
        ss += hv[r].w * hv[r].w;
      }
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)H + a.w.eps);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = tid + r * kFThreads;
      if (i < H / 4) {
        const uint2 wr = pre_w[r];
        const uint32_t y0 = f2bf(hv[r].x * inv * lo_bf(wr.x)), y1 = f2bf(hv[r].y * inv * hi_bf(wr.x));
        const uint32_t y2 = f2bf(hv[r].z * inv * lo_bf(wr.y)), y3 = f2bf(hv[r].w * inv * hi_bf(wr.y));
        *reinterpret_cast<float4*>(xs + t * H + xperm(i * 4, nch)) =
            make_float4(bf2f(y0), bf2f(y1), bf2f(y2), bf2f(y3));
        if (cta == 0)
          reinterpret_cast<uint2*>(a.normed + (int64_t)t * H)[i] = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
      }
    }
  }
  cta_sync();

  // Router rows (warps 0..1): gemv_bf16 order per lane over its 32-k chunks, butterfly sum.
  if (warp < kRouterRows) {
    const int row = kRouterRows * cta + warp;
    if (row < nrows) {
      const bool ok = __all_sync(0xffffffffu, bar_wait(&rbar, 0));
      if (!ok) {
        if (lane == 0) {
          atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
          abort_s = 1;
        }
      } else {
        const uint8_t* wrow = router_s + (size_t)warp * H * 2;
        for (int t = 0; t < T; ++t) {
          const float4* xs4 = reinterpret_cast<const float4*>(xs + t * H);
          float acc = 0.f;
          for (int c = lane; c < nch; c += 32) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x[8];
              x_word(xs4, nch, c, q, x);
              acc = dot_bf16_word(*reinterpret_cast<const uint4*>(wrow + c * 64 + q * 16), x, acc);
            }
          }
          acc = warp_sum(acc);
          if (lane == 0) {
            if (row < E) a.logits[(int64_t)t * E + row] = a.w.router_bias ? acc + a.w.router_bias[row] : acc;
            else a.gate[t] = sigmoid(acc);
          }
          __syncwarp();
        }
      }
    }
  }
  if (tid == 0) base_s = (gb / grid) * grid;
  grid_arrive(f.gbar);

  // Shared-expert gate/up pairs of this CTA while the router barrier settles (warps 2..5).
  if (warp >= 2 && warp < 2 + kSgu) {
    const int r = warp - 2, j = kSgu * cta + r;
    if (j < Is) {
      const bool ok = __all_sync(0xffffffffu, bar_wait(&sbar, 0));
      if (!ok) {
        if (lane == 0) {
          atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
          abort_s = 1;
        }
      } else if (sh8) {
        // gemv_i8_kernel's numerics: per 32-input chunk an fp32 dot of the raw int8 values, scaled once by the
        // chunk's group scale
        const uint8_t* grow = sgu_s + (size_t)r * H;
        const uint8_t* urow = sgu_s + (size_t)(kSgu + r) * H;
        const uint16_t* gsc = reinterpret_cast<const uint16_t*>(sgu_s + (size_t)2 * kSgu * H +
                                                                span_delta(s8g + (int64_t)(kSgu * cta) * sgs8) + r * sgs8);
        const uint16_t* usc = reinterpret_cast<const uint16_t*>(
            sgu_s + (size_t)2 * kSgu * H + scale_slot(kSgu, sgs8) + span_delta(s8g + (int64_t)(Is + kSgu * cta) * sgs8) +
            r * sgs8);
        for (int t = 0; t < T; ++t) {
          const float4* xs4 = reinterpret_cast<const float4*>(xs + t * H);
          float g = 0.f, u = 0.f;
          for (int c = lane; c < nch; c += 32) {
            const uint4 ga = *reinterpret_cast<const uint4*>(grow + c * 32);
            const uint4 gb = *reinterpret_cast<const uint4*>(grow + c * 32 + 16);
            const uint4 ua = *reinterpret_cast<const uint4*>(urow + c * 32);
            const uint4 ub = *reinterpret_cast<const uint4*>(urow + c * 32 + 16);
            const uint32_t gw[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
            const uint32_t uw[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
            float dg = 0.f, du = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x[8];
              x_word(xs4, nch, c, q, x);
              dg = i8x4_dot(gw[2 * q], x, dg);
              dg = i8x4_dot(gw[2 * q + 1], x + 4, dg);
              du = i8x4_dot(uw[2 * q], x, du);
              du = i8x4_dot(uw[2 * q + 1], x + 4, du);
            }
            g = fmaf(dg, h2f(gsc[c >> cshift8]), g);
            u = fmaf(du, h2f(usc[c >> cshift8]), u);
          }
          g = warp_sum(g);
          u = warp_sum(u);
          if (lane == 0) a.sinter[(int64_t)t * Is + j] = f2bf(silu(bf2f(f2bf(g))) * bf2f(f2bf(u)));
          __syncwarp();
        }
      } else {
        const uint8_t* grow = sgu_s + (size_t)r * H * 2;
        const uint8_t* urow = sgu_s + (size_t)(kSgu + r) * H * 2;
        for (int t = 0; t < T; ++t) {
          const float4* xs4 = reinterpret_cast<const float4*>(xs + t * H);
          float g = 0.f, u = 0.f;
          for (int c = lane; c < nch; c += 32) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float x[8];
              x_word(xs4, nch, c, q, x);
              g = dot_bf16_word(*reinterpret_cast<const uint4*>(grow + c * 64 + q * 16), x, g);
              u = dot_bf16_word(*reinterpret_cast<const uint4*>(urow + c * 64 + q * 16), x, u);
            }
          }
          g = warp_sum(g);
          u = warp_sum(u);
          if (lane == 0) a.sinter[(int64_t)t * Is + j] = f2bf(silu(bf2f(f2bf(g))) * bf2f(f2bf(u)));
          __syncwarp();
        }
      }
    }
  }
  const unsigned long long base = base_s;
  if (!grid_wait(f.gbar, base + grid, a.err, &ok_s) && tid == 0) abort_s = 1;

  // ---- phase G: top-k per token (warp t), unique-expert table and chunk list (warp 0)
  if (warp < T) topk_warp_redux(a.logits + (int64_t)warp * E, E, K, idx_s + warp * K, wts_s + warp * K);
  cta_sync();
  if (warp == 0) {
    table_warp(idx_s, P, E, K, uniq_s, uoff_s, upairs_s, ptok_s, pu_s, &nuniq_s);
    __syncwarp();
    if (lane == 0) {
      const int U = nuniq_s, J = U * I;
      const int cj0 = cta * J / grid, cj1 = (cta + 1) * J / grid;  // J <= 64 x 2048: no overflow
      int n = 0;
      for (int j = cj0; j < cj1 && n < kMaxChunks;) {
        const int uix = j / I, i0 = j - uix * I;
        const int m = min(C, cj1 - j);  // may run on into the next expert (C <= I)
        chunk_s[n++] = Chunk{0, uix, i0, m};
        j += m;
      }
      ngate_s = n;
      if (h0 < h1)
        for (int b = 0; b < U && n < kMaxChunks; b += f.kd) chunk_s[n++] = Chunk{1, b, 0, min(f.kd, U - b)};
      nchunks_s = n;
    }
  }
  cta_sync();
  const int U = nuniq_s, nchunks = nchunks_s, ngate = ngate_s;

  // Issues chunk c into stage c % S; called by all 32 lanes of one warp, which spread the copies over lanes.
  auto issue = [&](int c) {
    const int s = c % S;
    uint8_t* st = ring + (size_t)s * SB;
    const Chunk ch = chunk_s[c];
    fence_proxy_async_smem();  // this stage's earlier generic reads before the async-proxy writes
    if (ch.kind == 0) {
      // segment k: n_k jobs of unique expert a + k from row r_k, at stage position pos_k; lanes 4k .. 4k + 3 copy its
      // gate rows, up rows, gate scales, up scales
      const int n1 = min(ch.n, I - ch.i0), seg = (lane >> 2) & 1, part = lane & 3;
      const int nk = seg ? ch.n - n1 : n1, rk = seg ? 0 : ch.i0, pos = seg ? n1 : 0;
      const int64_t g0 = nk > 0 ? (int64_t)uniq_s[ch.a + seg] * 2 * I + rk : 0, u0 = g0 + I;
      const int64_t gA = (int64_t)uniq_s[ch.a] * 2 * I + ch.i0;  // segment 0's first gate row
      const uint32_t gsp0 = span_bytes(gscale + gA * sgb, n1 * sgb), usp0 = span_bytes(gscale + (gA + I) * sgb, n1 * sgb);
      const uint32_t mine = (lane < 8 && nk > 0)
                                ? (part < 2 ? (uint32_t)(nk * rowb)
                                            : span_bytes(gscale + (part == 2 ? g0 : u0) * sgb, nk * sgb))
                                : 0u;
      const uint32_t tx = __reduce_add_sync(0xffffffffu, mine);
      if (lane == 0) expect_tx(&full_b[s], tx);
      __syncwarp();
      if (lane < 8 && nk > 0) {
        uint8_t* sc0 = st + 2 * C * rowb;
        if (part == 0) bulk_g2s(st + pos * rowb, a.w.exp_gu_q + g0 * rowb, nk * rowb, &full_b[s]);
        else if (part == 1) bulk_g2s(st + (C + pos) * rowb, a.w.exp_gu_q + u0 * rowb, nk * rowb, &full_b[s]);
        else if (part == 2) bulk_span(sc0 + (seg ? gsp0 : 0), gscale + g0 * sgb, nk * sgb, &full_b[s]);
        else bulk_span(sc0 + gate_scale_region(C, H, G) + (seg ? usp0 : 0), gscale + u0 * sgb, nk * sgb, &full_b[s]);
      }
    } else {
      const int nr = h1 - h0, b = lane >> 1;
      const int64_t r0 = b < ch.n ? (int64_t)uniq_s[ch.a + b] * H + h0 : 0;
      const uint32_t mine = (b < ch.n && (lane & 1) == 0) ? (uint32_t)(nr * drowb) + span_bytes(dscale + r0 * dsb, nr * dsb) : 0u;
      const uint32_t tx = __reduce_add_sync(0xffffffffu, mine);
      if (lane == 0) expect_tx(&full_b[s], tx);
      __syncwarp();
      if (b < ch.n) {
        if ((lane & 1) == 0) bulk_g2s(st + (size_t)b * rpc * drowb, a.w.exp_dn_q + r0 * drowb, nr * drowb, &full_b[s]);
        else
          bulk_span(st + (size_t)f.kd * rpc * drowb + (size_t)b * down_scale_region(rpc, I, G), dscale + r0 * dsb,
                    nr * dsb, &full_b[s]);
      }
    }
    if (lane == 0) issued_s[s] += 1;
    __syncwarp();
  };
  // Called by every warp once it is done with chunk c: the last of the kFW warps refills the stage with chunk c + S.
  auto release = [&](int c) {
    __syncwarp();
    int refill = 0;
    if (lane == 0) {
      const int s = c % S;
      __threadfence_block();
      const int old = atomicAdd(&cnt_s[s], 1);
      if (old == kFW - 1) {
        cnt_s[s] = 0;
        __threadfence_block();
        refill = c + S < nchunks && !vload(&abort_s);
      }
    }
    if (__shfl_sync(0xffffffffu, refill, 0)) issue(c + S);
    __syncwarp();
  };
  // Waits for chunk c's bytes (every lane); false, and the CTA aborts, if the wait gives up.
  auto wait_chunk = [&](int c) -> bool {
    const bool ok = __all_sync(0xffffffffu, bar_wait(&full_b[c % S], (uint32_t)((c / S) & 1)));
    if (!ok && lane == 0) {
      atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
      abort_s = 1;
    }
    __syncwarp();
    return ok;
  };

  // first fill of the ring: warp 0 issues the gate/up chunks, the last warp the down chunks, concurrently; the
  // consumers synchronise on the stage barriers, not on a CTA barrier
  if (!vload(&abort_s)) {
    if (warp == 0)
      for (int c = 0; c < min(S, ngate); ++c) issue(c);
    else if (warp == kFW - 1)
      for (int c = ngate; c < min(S, nchunks); ++c) issue(c);
  }
  if (cta == 0) {
    for (int p = tid; p < P; p += kFThreads) {
      a.idx[p] = idx_s[p];
      a.wts[p] = wts_s[p];
      a.upairs[p] = upairs_s[p];
    }
    for (int u = tid; u < U; u += kFThreads) a.uniq[u] = uniq_s[u];
    for (int u = tid; u <= U; u += kFThreads) a.uoff[u] = uoff_s[u];
    if (tid == 0) *a.nuniq = U;
  }

  // Routed gate/up: jobs w and w + kFW of each gate/up chunk on warp w (two at once when both exist).
  const Nib8Magic M = nib8_magic();
  const int gshift = __ffs(G) - 6, dshift = __ffs(G) - 5;
  bool live = !vload(&abort_s);
  for (int c = 0; c < ngate; ++c) {
    if (live) live = wait_chunk(c);
    const Chunk ch = chunk_s[c];
    if (live && warp < ch.n) {
      const uint8_t* st = ring + (size_t)(c % S) * SB;
      const int n1 = min(ch.n, I - ch.i0);
      const int64_t gA = (int64_t)uniq_s[ch.a] * 2 * I + ch.i0;
      const int64_t gB = ch.n > n1 ? (int64_t)uniq_s[ch.a + 1] * 2 * I : 0;
      const uint32_t gsp0 = span_bytes(gscale + gA * sgb, n1 * sgb), usp0 = span_bytes(gscale + (gA + I) * sgb, n1 * sgb);
      const uint8_t* sc0 = st + 2 * C * rowb;
      // gate/up rows and scales of chunk job k
      auto job = [&](int k, const uint16_t*& gsc, const uint16_t*& usc, int& uix, int& row) {
        const bool second = k >= n1;
        const int64_t gk = second ? gB : gA;
        const int kk = second ? k - n1 : k;
        gsc = reinterpret_cast<const uint16_t*>(sc0 + (second ? gsp0 : 0) + span_delta(gscale + gk * sgb) + kk * sgb);
        usc = reinterpret_cast<const uint16_t*>(sc0 + gate_scale_region(C, H, G) + (second ? usp0 : 0) +
                                                span_delta(gscale + (gk + I) * sgb) + kk * sgb);
        uix = ch.a + (second ? 1 : 0);
        row = second ? kk : ch.i0 + kk;
      };
      const uint16_t *gs0, *us0, *gs1, *us1;
      int ux0, r0, ux1 = -1, r1 = 0;
      job(warp, gs0, us0, ux0, r0);
      const int w1 = warp + kFW;
      if (w1 < ch.n) job(w1, gs1, us1, ux1, r1);
      if (ux1 == ux0) {
        fused_gate_job2(a, xs, st + warp * rowb, st + (C + warp) * rowb, gs0, us0, st + w1 * rowb,
                        st + (C + w1) * rowb, gs1, us1, ux0, r0, r1, uoff_s, upairs_s, ptok_s, gshift, M);
      } else {
        fused_gate_job(a, xs, st + warp * rowb, st + (C + warp) * rowb, gs0, us0, ux0, r0, uoff_s, upairs_s, ptok_s,
                       gshift, M);
        if (ux1 >= 0)
          fused_gate_job(a, xs, st + w1 * rowb, st + (C + w1) * rowb, gs1, us1, ux1, r1, uoff_s, upairs_s, ptok_s,
                         gshift, M);
      }
    }
    release(c);
  }
  grid_arrive(f.gbar);
  if (!grid_wait(f.gbar, base + 2 * (unsigned long long)grid, a.err, &ok_s) && tid == 0) abort_s = 1;
  cta_sync();

  // the next kernel on the stream may start its entry on SMs this grid frees from here on
  pdl_launch_dependents();

  // ---- phase D: stage inter (bf16, permuted) and sinter; reduce this warp's output row over the down chunks
  const int nchd = I >> 4, Ld = min(32, nchd), PI = inter_stride(I);
  uint16_t* inter_s = reinterpret_cast<uint16_t*>(smem + L.xs);
  for (int idx = tid; idx < P * I / 8; idx += kFThreads) {
    const int p = (idx * 8) / I, k = idx * 8 - p * I;
    *reinterpret_cast<uint4*>(inter_s + (size_t)p * PI + iperm(k, Ld)) =
        __ldcg(reinterpret_cast<const uint4*>(a.inter) + idx);
  }
  for (int idx = tid; idx < T * Is / 8; idx += kFThreads)
    reinterpret_cast<uint4*>(sinter_s)[idx] = __ldcg(reinterpret_cast<const uint4*>(a.sinter) + idx);
  cta_sync();

  float* acc_w = acc_s + (size_t)warp * T * 32;
  for (int t = 0; t < T; ++t) acc_w[t * 32 + lane] = 0.f;
  const int hw = h0 + warp;
  live = !vload(&abort_s);
  for (int c = ngate; c < nchunks; ++c) {
    if (live) live = wait_chunk(c);
    const Chunk ch = chunk_s[c];
    if (live && hw < h1) {
      // the chunk's pairs are contiguous in sorted order; four partials at a time are independent, then they are
      // accumulated in pair order (the order of the three-kernel path)
      const uint8_t* st = ring + (size_t)(c % S) * SB;
      const int pa = uoff_s[ch.a], pb = uoff_s[ch.a + ch.n];
      for (int p0 = pa; p0 < pb; p0 += 4) {
        float part[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          part[q] = 0.f;
          const int p = p0 + q;
          if (p < pb) {
            const int b = pu_s[p] - ch.a;
            const int64_t r0 = (int64_t)uniq_s[ch.a + b] * H + h0;
            const uint8_t* wr = st + ((size_t)b * rpc + warp) * drowb;
            const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + (size_t)f.kd * rpc * drowb +
                                                                   (size_t)b * down_scale_region(rpc, I, G) +
                                                                   span_delta(dscale + r0 * dsb) + warp * dsb);
            const uint8_t* xr = reinterpret_cast<const uint8_t*>(inter_s + (size_t)upairs_s[p] * PI);
            for (int cc = lane; cc < nchd; cc += 32) {
              const int j = cc >> 5;
              const uint2 wq = *reinterpret_cast<const uint2*>(wr + cc * 8);
              u64 x01, x23, x45, x67;
              Nib8Acc A;
              nib8_zero(A);
              inter_pairs<false>(xr + (size_t)((j * 2) * Ld + lane) * 16, x01, x23, x45, x67);
              nib8x2(wq.x, x01, x23, x45, x67, M, A);
              inter_pairs<false>(xr + (size_t)((j * 2 + 1) * Ld + lane) * 16, x01, x23, x45, x67);
              nib8x2(wq.y, x01, x23, x45, x67, M, A);
              part[q] = fmaf(nib8_fold(A), h2f(sc[cc >> dshift]), part[q]);
            }
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = p0 + q;
          if (p < pb) {
            float* slotacc = acc_w + ptok_s[p] * 32 + lane;
            *slotacc = fmaf(wts_s[upairs_s[p]], part[q], *slotacc);
          }
        }
      }
    }
    release(c);
  }
  bool sdn_ok = live && hw < h1;
  if (sdn_ok) {
    sdn_ok = __all_sync(0xffffffffu, bar_wait(&sbar, 0));
    if (!sdn_ok && lane == 0) {  // this warp's output row is not written: the call's results are invalid
      atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
      abort_s = 1;
    }
  }
  if (sdn_ok) {
    float routed_t = 0.f, shared_t = 0.f;
    for (int t = 0; t < T; ++t) {
      const float v = warp_sum(acc_w[t * 32 + lane]);
      if (lane == t) routed_t = v;
    }
    const uint8_t* srow = sdn_s + (size_t)(hw - h0) * Is * (sh8 ? 1 : 2);
    const uint16_t* dsc8 = reinterpret_cast<const uint16_t*>(sdn_s + (size_t)rpc * Is +
                                                             span_delta(s8d + (int64_t)h0 * dss8) + (hw - h0) * dss8);
    for (int t = 0; t < T && sh8; ++t) {
      // gemv_i8_kernel over the Is shared intermediates: lane l takes inputs 32 l .. 32 l + 31 of each 1024
      float acc = 0.f;
      for (int k0 = lane * 32; k0 < Is; k0 += 1024) {
        const uint4 wa = *reinterpret_cast<const uint4*>(srow + k0);
        const uint4 wb = *reinterpret_cast<const uint4*>(srow + k0 + 16);
        const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        float d = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 xv = *reinterpret_cast<const uint4*>(sinter_s + t * Is + k0 + q * 8);
          const float x[8] = {lo_bf(xv.x), hi_bf(xv.x), lo_bf(xv.y), hi_bf(xv.y),
                              lo_bf(xv.z), hi_bf(xv.z), lo_bf(xv.w), hi_bf(xv.w)};
          d = i8x4_dot(ww[2 * q], x, d);
          d = i8x4_dot(ww[2 * q + 1], x + 4, d);
        }
        acc = fmaf(d, h2f(dsc8[k0 / g8]), acc);
      }
      const float v = bf2f(f2bf(warp_sum(acc)));
      if (lane == t) shared_t = v;
    }
    for (int t = 0; t < T && !sh8; ++t) {
      float acc = 0.f;
      for (int v = lane; v < nvs; v += 32) {
        const uint4 wv = *reinterpret_cast<const uint4*>(srow + v * 16);
        const uint4 xv = *reinterpret_cast<const uint4*>(sinter_s + t * Is + v * 8);
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc = fmaf(lo_bf(ww[q]), lo_bf(xx[q]), acc);
          acc = fmaf(hi_bf(ww[q]), hi_bf(xx[q]), acc);
        }
      }
      const float v = bf2f(f2bf(warp_sum(acc)));
      if (lane == t) shared_t = v;
    }
    if (lane < T) {
      const int t = lane;
      const int64_t o = (int64_t)t * H + hw;
      a.routed[o] = routed_t;
      a.sout[o] = f2bf(shared_t);
      const float hh = a.hidden[o] + bf2f(a.attn_out[o]);  // the residual add of residual_rmsnorm_kernel
      const float g = __ldcg(a.gate + t);
      a.hidden[o] = f.next_norm ? fmaf(g, shared_t, hh + routed_t) : hh + fmaf(g, shared_t, routed_t);
    }
  }
  // No copy may still be landing when the CTA exits. On the normal path every copy was waited for by its
  // consumers; after an abort, wait (bounded) for the last chunk issued to every stage and for the entry copies.
  cta_sync();
  if (tid == 0 && vload(&abort_s)) {
    for (int s = 0; s < S; ++s)
      if (issued_s[s] > 0) bar_wait(&full_b[s], (uint32_t)((issued_s[s] - 1) & 1));
    bar_wait(&rbar, 0);
    bar_wait(&sbar, 0);
  }
  if (!f.next_norm || vload(&abort_s)) return;
  // Next layer's RMSNorm: the last CTA to finish (shared_gate_combine_rmsnorm_kernel).
  cta_sync();
  if (tid == 0) {
    __threadfence();
    is_last = atomicInc(&a.ticket[TICKET_COMBINE], gridDim.x - 1) == gridDim.x - 1;
  }
  cta_sync();
  if (!is_last) return;
  __threadfence();
  for (int t = 0; t < T; ++t) {
    const float* hr = a.hidden + (int64_t)t * H;
    float ss = 0.f;
    for (int i = tid; i < H; i += kFThreads) {
      const float v = __ldcg(hr + i);
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)H + a.w.eps);
    for (int i = tid; i < H; i += kFThreads)
      a.normed[(int64_t)t * H + i] = f2bf(__ldcg(hr + i) * inv * bf2f(a.next_rms1[i]));
  }
}

// ------------------------------------------------------------------ host side

static int device_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

static int max_smem_optin() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (n <= 0) n = 227 * 1024;
  }
  return n;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Programmatic dependent launch, as for the three-kernel path: on unless the environment sets MOE_B200_PDL=0.
static bool fused_pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("MOE_B200_PDL");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

struct FusedCfg {
  int stages, stage_bytes, cjobs, kd, rpc;
  size_t smem;
};

static bool fused_plan(const moe_layer_weights& w, int T, FusedCfg* out) {
  if (T < 1 || T > kFusedMaxT || w.TOPK * T > 64) return false;
  const int grid = device_sms();
  if (w.E + 1 > kRouterRows * grid || w.Is > kSgu * grid || w.H > 4096) return false;
  // the bulk copies start at 16-byte aligned weight rows
  if (!aligned16(w.router) || !aligned16(w.shared_gate) || !aligned16(w.shared_gate_up) ||
      !aligned16(w.shared_down) || !aligned16(w.exp_gu_q) || !aligned16(w.exp_dn_q) || !aligned16(w.exp_gu_s) ||
      !aligned16(w.exp_dn_s))
    return false;
  if (w.shared_gate_up_q8) {  // int8 shared expert: rows copied whole, scales as aligned supersets
    if (!aligned16(w.shared_gate_up_q8) || !aligned16(w.shared_down_q8) || w.shared_group % 32 != 0 ||
        w.shared_group <= 0 || w.H % w.shared_group != 0 || w.Is % w.shared_group != 0)
      return false;
  }
  const int rpc = (w.H + grid - 1) / grid;
  if (rpc > kFW) return false;  // one output row per warp
  // gate/up jobs per chunk: two per warp at the smallest batches (their activation loads are shared), else one
  int C = T <= 2 ? 2 * kFW : kFW;
  while (C > 1 && 2 * C * (w.H / 2) > (C > kFW ? 64 : 32) * 1024) C >>= 1;
  int kd = C > kFW ? 16 : 8;
  while (kd > 1 && down_stage_bytes(kd, rpc, w.I, w.G) > gate_stage_bytes(C, w.H, w.G)) --kd;
  // chunk-list bound: the CTA's gate/up jobs split at chunk size and expert boundaries, plus the down chunks
  const int P = T * w.TOPK;
  const int per_cta = P * w.I / grid + 1;
  if (per_cta / C + 2 + (P + kd - 1) / kd > kMaxChunks) return false;
  const int sb = (std::max(gate_stage_bytes(C, w.H, w.G), down_stage_bytes(kd, rpc, w.I, w.G)) + 127) / 128 * 128;
  const int limit = max_smem_optin() - 6 * 1024;  // static shared memory of the kernel
  for (int s = kMaxStages; s >= 2; --s) {
    const FusedSmem L = fused_smem(T, w.H, w.TOPK, w.I, w.Is, rpc, sb, s);
    if ((int)L.total <= limit) {
      out->stages = s;
      out->stage_bytes = sb;
      out->cjobs = C;
      out->kd = kd;
      out->rpc = rpc;
      out->smem = L.total;
      return true;
    }
  }
  return false;
}

bool fused_config(const moe_layer_weights& w, int T, int* stages, size_t* smem, int* rows_per_cta) {
  FusedCfg c;
  if (!fused_plan(w, T, &c)) return false;
  *stages = c.stages;
  *smem = c.smem;
  *rows_per_cta = c.rpc;
  return true;
}

cudaError_t launch_fused_decode(const BlockArgs& a, unsigned long long* gbar, bool next_norm, cudaStream_t s) {
  FusedCfg c;
  if (!fused_plan(a.w, a.T, &c)) return cudaErrorInvalidValue;
  static SmemGrant granted;
  cudaError_t e = grant_smem(reinterpret_cast<const void*>(moe_fused_decode_kernel), c.smem, (size_t)200 * 1024, granted);
  if (e != cudaSuccess) return e;
  FusedArgs f;
  memset(&f, 0, sizeof f);
  f.a = a;
  f.gbar = gbar;
  f.stages = c.stages;
  f.stage_bytes = c.stage_bytes;
  f.cjobs = c.cjobs;
  f.kd = c.kd;
  f.rows_per_cta = c.rpc;
  f.next_norm = next_norm ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_sms());
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = fused_pdl_enabled() ? 2 : 1;
  return launched(cudaLaunchKernelEx(&cfg, moe_fused_decode_kernel, f));
}

}  // namespace moe
