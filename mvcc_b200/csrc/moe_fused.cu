// moe_fused.cu -- fused persistent decode kernel of the MoE block for T <= 8 tokens: one cooperative launch does
// qwen.cu:429-448 end to end.
//
// One CTA per SM, 16 warps. The work is partitioned so that every SM streams about the same number of weight
// bytes, and every byte is requested as soon as its dependency allows:
//   start     cp.async of the routing-independent weights this CTA owns: router rows (router row r -> CTA r % G,
//             the shared gate vector is row E), shared-expert gate/up row pairs (pair j -> CTA j % G) and the
//             shared-expert down rows of the CTA's output rows [h0, h1);
//   phase R   RMSNorm of every token (every CTA, into shared memory), router logits of the CTA's rows -> global;
//             arrive at grid barrier 1; compute the shared-expert gate/up pairs while the barrier settles; wait;
//   phase G   every CTA runs the reference's top-k on all logits itself (no second round trip) and builds the
//             unique-expert table in shared memory; each warp then streams its routed gate/up row pairs and its
//             down-row batches through a private cp.async ring (loads run ahead of compute, across the barrier);
//             `inter` -> global; arrive and wait at grid barrier 2;
//   phase D   stage every pair's `inter` and the shared `sinter`; each warp reduces one output row h over every
//             unique expert (weighted per pair) and the shared expert, and applies the gated residual combine;
//             the last CTA to finish (ticket) optionally applies the next layer's RMSNorm.
// Grid barriers use a monotone 64-bit arrival counter in the workspace (each launch adds exactly 2 x G arrivals,
// so the targets follow from its value at launch start) and bounded spins: after kSpinLimit polls a CTA records
// MOE_ERR_BARRIER in the error word, drains its own copies and returns. The launch is cooperative, so all CTAs are
// co-resident. Reductions and numerics are those of the three-kernel path (moe_decode.cu).
#include <algorithm>
#include <cstring>

#include "moe_device.cuh"
#include "moe_fused.h"

namespace moe {

constexpr int kFW = 16;
constexpr int kFThreads = kFW * 32;
constexpr int kSgu = 4;                   // shared gate/up pairs per CTA (Is <= 4 x grid)
constexpr int kRouterRows = 2;            // router rows per CTA (E + 1 <= 2 x grid)
constexpr long long kSpinLimit = 1 << 21; // barrier polls (x ~100 ns) before giving up

struct FusedArgs {
  BlockArgs a;
  unsigned long long* gbar;  // grid-barrier arrival counter
  int slot_bytes;            // per-warp ring slot
  int stages;                // ring slots per warp
  int rows_per_cta;          // output rows h per CTA
  int next_norm;             // apply the next layer's RMSNorm
};

// Shared-memory carve-up (bytes), identical on host and device.
struct FusedSmem {
  size_t xs, sinter, router, sgu, sdn, acc, ring, total;
};

__host__ __device__ inline size_t f_align(size_t x) { return (x + 127) & ~(size_t)127; }

__host__ __device__ inline FusedSmem fused_smem(int T, int H, int TOPK, int I, int Is, int rows_per_cta,
                                                 int slot_bytes, int stages) {
  FusedSmem L;
  size_t o = 0;
  const size_t xs = (size_t)T * H * 4, inter = (size_t)T * TOPK * inter_stride(I) * 2;
  L.xs = o;     o = f_align(o + (xs > inter ? xs : inter));
  L.sinter = o; o = f_align(o + (size_t)T * Is * 2);
  L.router = o; o = f_align(o + (size_t)kRouterRows * H * 2);
  L.sgu = o;    o = f_align(o + (size_t)kSgu * 2 * H * 2);
  L.sdn = o;    o = f_align(o + (size_t)rows_per_cta * Is * 2);
  L.acc = o;    o = f_align(o + (size_t)kFW * T * 32 * 4);
  L.ring = o;   o = f_align(o + (size_t)kFW * stages * slot_bytes);
  L.total = o;
  return L;
}

__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_wait_stages(int stages) {
  switch (stages) {  // wait until at most stages - 1 groups are pending
    case 1: cp_wait<0>(); break;
    case 2: cp_wait<1>(); break;
    case 3: cp_wait<2>(); break;
    default: cp_wait<3>(); break;
  }
}

// Copies `bytes` (a multiple of 16) from global to shared with the calling warp's lanes.
__device__ __forceinline__ void warp_copy16(uint8_t* dst, const uint8_t* src, int bytes, int lane) {
  for (int o = lane * 16; o < bytes; o += 32 * 16) cp_async16(dst + o, src + o);
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier on a monotone arrival counter. Every launch adds exactly 2 x G arrivals and launches do not overlap,
// so the counter is a multiple of G when a launch starts; a CTA reads it once at start (any value seen before its
// own first arrival lies in [base, base + G)) and barrier k completes at base + k x G. Arrival is a release
// reduction (no round trip); the wait spins, bounded, on an acquire load.
__device__ __forceinline__ void grid_arrive(unsigned long long* gbar) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(gbar) : "memory");
}
__device__ __forceinline__ bool grid_wait(const unsigned long long* gbar, unsigned long long target, uint32_t* err,
                                          int* ok_s) {
  if (threadIdx.x == 0) {
    int ok = 1;
    long long it = 0;
    while (ld_acquire_u64(gbar) < target) {
      if (++it > kSpinLimit) {
        atomicOr(err, (uint32_t)MOE_ERR_BARRIER);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

// The reference's top-k table built in shared memory (same rule and order as build_unique in moe_decode.cu).
__device__ void table_smem(const int32_t* idx_s, int P, int E, int* cnt_s, int* start_s, int* uniq_s, int* uoff_s,
                           int* upairs_s, int* ptok_s, int K, int* nuniq_s) {
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) cnt_s[e] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    const int e = idx_s[p];
    if (e >= 0 && e < E) atomicAdd(&cnt_s[e], 1);
  }
  __syncthreads();
  if (tid < 32) {
    const int lane = tid;
    int nz = 0, np = 0;
    for (int j = 0; j < 8; ++j) {
      const int e = lane * 8 + j;
      if (e < E && cnt_s[e] > 0) { ++nz; np += cnt_s[e]; }
    }
    int nz_ex = nz, np_ex = np;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a1 = __shfl_up_sync(0xffffffffu, nz_ex, o), a2 = __shfl_up_sync(0xffffffffu, np_ex, o);
      if (lane >= o) { nz_ex += a1; np_ex += a2; }
    }
    nz_ex -= nz;
    np_ex -= np;
    for (int j = 0; j < 8; ++j) {
      const int e = lane * 8 + j;
      if (e < E && cnt_s[e] > 0) {
        uniq_s[nz_ex] = e;
        uoff_s[nz_ex] = np_ex;
        start_s[e] = np_ex;
        ++nz_ex;
        np_ex += cnt_s[e];
      }
    }
    if (lane == 31) {
      *nuniq_s = nz_ex;
      uoff_s[nz_ex] = np_ex;
    }
  }
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    const int e = idx_s[p];
    if (e < 0 || e >= E) continue;
    int rank = 0;
    for (int q = 0; q < p; ++q) rank += (idx_s[q] == e);
    upairs_s[start_s[e] + rank] = p;
    ptok_s[start_s[e] + rank] = p / K;
  }
  __syncthreads();
}

// One routed gate/up row pair (gate row i and up row I + i of expert e) from its ring slot, for every pair of
// unique expert uix; same reduction as compute_routed in moe_decode.cu.
__device__ __forceinline__ void fused_gate_job(const BlockArgs& a, const float* xs, const uint8_t* slot, int uix,
                                               int i, const int* uoff_s, const int* upairs_s, const int* ptok_s,
                                               int gshift, const Nib8Magic& M) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, I = a.w.I, nch = H >> 5;
  const int half = H >> 1, sgroups = H / a.w.G;
  const uint16_t* gsc = reinterpret_cast<const uint16_t*>(slot + H);
  const uint16_t* usc = gsc + sgroups;
  for (int p = uoff_s[uix]; p < uoff_s[uix + 1]; ++p) {
    const int pair = upairs_s[p];
    const float* xt = xs + ptok_s[p] * H;
    float g = 0.f, u = 0.f;
    for (int c = lane; c < nch; c += 32) {
      const uint4 gq = *reinterpret_cast<const uint4*>(slot + c * 16);
      const uint4 uq = *reinterpret_cast<const uint4*>(slot + half + c * 16);
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
  }
}

__global__ void __launch_bounds__(kFThreads, 1) moe_fused_decode_kernel(FusedArgs f) {
  extern __shared__ __align__(128) uint8_t smem[];
  const BlockArgs& a = f.a;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, H = a.w.H, E = a.w.E, K = a.w.TOPK, I = a.w.I, Is = a.w.Is, G = a.w.G;
  const int P = T * K, nch = H >> 5, nvs = Is >> 3;
  const int grid = gridDim.x, cta = blockIdx.x;
  const FusedSmem L = fused_smem(T, H, K, I, Is, f.rows_per_cta, f.slot_bytes, f.stages);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  uint16_t* sinter_s = reinterpret_cast<uint16_t*>(smem + L.sinter);
  uint8_t* router_s = smem + L.router;
  uint8_t* sgu_s = smem + L.sgu;
  uint8_t* sdn_s = smem + L.sdn;
  float* acc_s = reinterpret_cast<float*>(smem + L.acc);
  uint8_t* ring = smem + L.ring + (size_t)warp * f.stages * f.slot_bytes;
  __shared__ float red[32];
  __shared__ int32_t idx_s[64];
  __shared__ float wts_s[64];
  __shared__ int cnt_s[256], start_s[256], uniq_s[256], uoff_s[257], upairs_s[64], ptok_s[64];
  __shared__ int nuniq_s, ok_s, is_last;
  __shared__ unsigned long long base_s;
  const int h0 = cta * f.rows_per_cta, h1 = min(H, h0 + f.rows_per_cta);
  if (tid == 0) base_s = (ld_acquire_u64(f.gbar) / grid) * grid;

  // ---- start: routing-independent weights of this CTA (one cp.async group per thread)
  const int nrows = E + 1;
  for (int r = 0; r < kRouterRows; ++r) {
    const int row = cta + r * grid;
    if (row < nrows) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(row < E ? a.w.router + (int64_t)row * H : a.w.shared_gate);
      for (int o = tid * 16; o < H * 2; o += kFThreads * 16) cp_async16(router_s + (size_t)r * H * 2 + o, src + o);
    }
  }
  cp_commit();  // group: router rows
  for (int r = 0; r < kSgu; ++r) {
    const int j = cta + r * grid;
    if (j < Is) {
      const uint8_t* gsrc = reinterpret_cast<const uint8_t*>(a.w.shared_gate_up + (int64_t)j * H);
      const uint8_t* usrc = reinterpret_cast<const uint8_t*>(a.w.shared_gate_up + (int64_t)(Is + j) * H);
      uint8_t* dst = sgu_s + (size_t)r * 2 * H * 2;
      for (int o = tid * 16; o < H * 2; o += kFThreads * 16) {
        cp_async16(dst + o, gsrc + o);
        cp_async16(dst + H * 2 + o, usrc + o);
      }
    }
  }
  if (h0 < h1) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.w.shared_down + (int64_t)h0 * Is);
    const int bytes = (h1 - h0) * Is * 2;
    for (int o = tid * 16; o < bytes; o += kFThreads * 16) cp_async16(sdn_s + o, src + o);
  }
  cp_commit();  // group: shared-expert rows

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
        const uint2 d = dr[i];
        hv[r] = hr[i];
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
        const uint2 wr = reinterpret_cast<const uint2*>(a.w.rms2)[i];
        const uint32_t y0 = f2bf(hv[r].x * inv * lo_bf(wr.x)), y1 = f2bf(hv[r].y * inv * hi_bf(wr.x));
        const uint32_t y2 = f2bf(hv[r].z * inv * lo_bf(wr.y)), y3 = f2bf(hv[r].w * inv * hi_bf(wr.y));
        *reinterpret_cast<float4*>(xs + t * H + xperm(i * 4, nch)) =
            make_float4(bf2f(y0), bf2f(y1), bf2f(y2), bf2f(y3));
        if (cta == 0)
          reinterpret_cast<uint2*>(a.normed + (int64_t)t * H)[i] = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
      }
    }
  }
  cp_wait<1>();  // router rows landed; shared-expert rows may still be in flight
  __syncthreads();

  // Router rows (warps 0..1): gemv_bf16 order per lane over its 32-k chunks, butterfly sum.
  if (warp < kRouterRows) {
    const int row = cta + warp * grid;
    if (row < nrows) {
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
      }
    }
  }
  grid_arrive(f.gbar);
  cp_wait<0>();  // shared-expert rows
  __syncthreads();

  // Shared-expert gate/up pairs of this CTA while the router barrier settles (warps 2..5).
  if (warp >= 2 && warp < 2 + kSgu) {
    const int r = warp - 2, j = cta + r * grid;
    if (j < Is) {
      const uint8_t* grow = sgu_s + (size_t)r * 2 * H * 2;
      const uint8_t* urow = grow + H * 2;
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
      }
    }
  }
  const unsigned long long base = base_s;
  if (!grid_wait(f.gbar, base + grid, a.err, &ok_s)) return;

  // ---- phase G: top-k per token (warp t), unique-expert table, routed gate/up through the per-warp rings
  if (warp < T) topk_warp(a.logits + (int64_t)warp * E, E, K, idx_s + warp * K, wts_s + warp * K);
  __syncthreads();
  table_smem(idx_s, P, E, cnt_s, start_s, uniq_s, uoff_s, upairs_s, ptok_s, K, &nuniq_s);
  const int U = nuniq_s;
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

  // This warp's items: gate/up jobs [g0, g1) of the U x I job space, then the down-row batches of row hw.
  const int J = U * I;
  const int cj0 = (int)((int64_t)cta * J / grid), cj1 = (int)((int64_t)(cta + 1) * J / grid);
  const int g0 = cj0 + (int)((int64_t)warp * (cj1 - cj0) / kFW), g1 = cj0 + (int)((int64_t)(warp + 1) * (cj1 - cj0) / kFW);
  const int ng = g1 - g0;
  const int hw = h0 + warp;
  const int nd = hw < h1 ? (U + 7) / 8 : 0;
  const int n_items = ng + nd;
  const int S = f.stages, SB = f.slot_bytes;
  const int gshift = __ffs(G) - 6, dshift = __ffs(G) - 5;
  const int rowb = H >> 1, sgb = (H / G) * 2;      // gate/up job: row bytes, scale bytes per row
  const int drowb = I >> 1, dsb = (I / G) * 2;     // down: row bytes, scale bytes per row

  auto issue = [&](int it) {
    uint8_t* slot = ring + (size_t)(it % S) * SB;
    if (it < ng) {
      const int j = g0 + it, uix = j / I, i = j - uix * I, e = uniq_s[uix];
      const uint8_t* gq = a.w.exp_gu_q + ((int64_t)e * 2 * I + i) * rowb;
      const uint8_t* gs = reinterpret_cast<const uint8_t*>(a.w.exp_gu_s + ((int64_t)e * 2 * I + i) * (H / G));
      warp_copy16(slot, gq, rowb, lane);
      warp_copy16(slot + rowb, gq + (int64_t)I * rowb, rowb, lane);
      warp_copy16(slot + 2 * rowb, gs, sgb, lane);
      warp_copy16(slot + 2 * rowb + sgb, gs + (int64_t)I * sgb, sgb, lane);
    } else {
      const int b0 = (it - ng) * 8;
      for (int b = 0; b < 8 && b0 + b < U; ++b) {
        const int e = uniq_s[b0 + b];
        warp_copy16(slot + b * drowb, a.w.exp_dn_q + ((int64_t)e * H + hw) * drowb, drowb, lane);
        const uint8_t* sc =
            reinterpret_cast<const uint8_t*>(a.w.exp_dn_s + ((int64_t)e * H + hw) * (I / G));
        uint8_t* sdst = slot + 8 * drowb + b * dsb;
        if (dsb >= 16) warp_copy16(sdst, sc, dsb, lane);
        else if (lane == 0) cp_async8(sdst, sc);
      }
    }
  };

  for (int s = 0; s < S; ++s) {
    if (s < n_items) issue(s);
    cp_commit();
  }
  const Nib8Magic M = nib8_magic();
  for (int it = 0; it < ng; ++it) {
    cp_wait_stages(S);
    __syncwarp();
    const int j = g0 + it, uix = j / I, i = j - uix * I;
    fused_gate_job(a, xs, ring + (size_t)(it % S) * SB, uix, i, uoff_s, upairs_s, ptok_s, gshift, M);
    __syncwarp();
    if (it + S < n_items) issue(it + S);
    cp_commit();
  }
  grid_arrive(f.gbar);
  if (!grid_wait(f.gbar, base + 2 * (unsigned long long)grid, a.err, &ok_s)) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    return;
  }

  // ---- phase D: stage inter (bf16, permuted) and sinter; reduce this warp's output row
  const int nchd = I >> 4, Ld = min(32, nchd), PI = inter_stride(I);
  uint16_t* inter_s = reinterpret_cast<uint16_t*>(smem + L.xs);
  for (int idx = tid; idx < P * I / 8; idx += kFThreads) {
    const int p = (idx * 8) / I, k = idx * 8 - p * I;
    *reinterpret_cast<uint4*>(inter_s + (size_t)p * PI + iperm(k, Ld)) = __ldcg(reinterpret_cast<const uint4*>(a.inter) + idx);
  }
  for (int idx = tid; idx < T * Is / 8; idx += kFThreads)
    reinterpret_cast<uint4*>(sinter_s)[idx] = __ldcg(reinterpret_cast<const uint4*>(a.sinter) + idx);
  __syncthreads();

  float* acc_w = acc_s + (size_t)warp * T * 32;
  for (int t = 0; t < T; ++t) acc_w[t * 32 + lane] = 0.f;
  for (int it = ng; it < n_items; ++it) {
    cp_wait_stages(S);
    __syncwarp();
    const uint8_t* slot = ring + (size_t)(it % S) * SB;
    const int b0 = (it - ng) * 8;
    for (int b = 0; b < 8 && b0 + b < U; ++b) {
      const uint8_t* wr = slot + b * drowb;
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(slot + 8 * drowb + b * dsb);
      for (int p = uoff_s[b0 + b]; p < uoff_s[b0 + b + 1]; ++p) {
        const int pair = upairs_s[p];
        const uint8_t* xr = reinterpret_cast<const uint8_t*>(inter_s + (size_t)pair * PI);
        float part = 0.f;
        for (int c = lane; c < nchd; c += 32) {
          const int j = c >> 5;
          const uint2 wq = *reinterpret_cast<const uint2*>(wr + c * 8);
          u64 x01, x23, x45, x67;
          Nib8Acc A;
          nib8_zero(A);
          inter_pairs<false>(xr + (size_t)((j * 2) * Ld + lane) * 16, x01, x23, x45, x67);
          nib8x2(wq.x, x01, x23, x45, x67, M, A);
          inter_pairs<false>(xr + (size_t)((j * 2 + 1) * Ld + lane) * 16, x01, x23, x45, x67);
          nib8x2(wq.y, x01, x23, x45, x67, M, A);
          part = fmaf(nib8_fold(A), h2f(sc[c >> dshift]), part);
        }
        float* slotacc = acc_w + ptok_s[p] * 32 + lane;
        *slotacc = fmaf(wts_s[pair], part, *slotacc);
      }
    }
    __syncwarp();
    if (it + S < n_items) issue(it + S);
    cp_commit();
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (hw < h1) {
    float routed_t = 0.f, shared_t = 0.f;
    for (int t = 0; t < T; ++t) {
      const float v = warp_sum(acc_w[t * 32 + lane]);
      if (lane == t) routed_t = v;
    }
    const uint8_t* srow = sdn_s + (size_t)(hw - h0) * Is * 2;
    for (int t = 0; t < T; ++t) {
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
  if (!f.next_norm) return;
  // Next layer's RMSNorm: the last CTA to finish (shared_gate_combine_rmsnorm_kernel).
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    is_last = atomicInc(&a.ticket[TICKET_COMBINE], gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
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

// Slot: the larger of one gate/up row pair (+ scales) and one batch of 8 down rows (+ scales), 16-byte multiple.
static int fused_slot_bytes(const moe_layer_weights& w) {
  const int gate = w.H + 2 * (w.H / w.G) * 2;
  const int down = 8 * (w.I / 2) + 8 * (w.I / w.G) * 2;
  return (std::max(gate, down) + 15) / 16 * 16;
}

bool fused_config(const moe_layer_weights& w, int T, int* stages, size_t* smem, int* rows_per_cta) {
  if (T < 1 || T > kFusedMaxT) return false;
  const int grid = device_sms();
  if (w.E + 1 > kRouterRows * grid || w.Is > kSgu * grid || w.H > 4096) return false;
  const int rpc = (w.H + grid - 1) / grid;
  if (rpc > kFW) return false;  // one output row per warp
  const int slot = fused_slot_bytes(w);
  const int limit = max_smem_optin() - 6 * 1024;  // static shared memory of the kernel
  for (int s = 4; s >= 2; --s) {
    const FusedSmem L = fused_smem(T, w.H, w.TOPK, w.I, w.Is, rpc, slot, s);
    if ((int)L.total <= limit) {
      *stages = s;
      *smem = L.total;
      *rows_per_cta = rpc;
      return true;
    }
  }
  return false;
}

cudaError_t launch_fused_decode(const BlockArgs& a, unsigned long long* gbar, bool next_norm, cudaStream_t s) {
  int stages = 0, rpc = 0;
  size_t smem = 0;
  if (!fused_config(a.w, a.T, &stages, &smem, &rpc)) return cudaErrorInvalidValue;
  static size_t granted = 0;
  if (smem > granted) {
    cudaError_t e = cudaFuncSetAttribute(moe_fused_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)std::max(smem, (size_t)200 * 1024));
    if (e != cudaSuccess) return e;
    granted = std::max(smem, (size_t)200 * 1024);
  }
  FusedArgs f;
  memset(&f, 0, sizeof f);
  f.a = a;
  f.gbar = gbar;
  f.slot_bytes = fused_slot_bytes(a.w);
  f.stages = stages;
  f.rows_per_cta = rpc;
  f.next_norm = next_norm ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(device_sms());
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_fused_decode_kernel, f);
}

}  // namespace moe
