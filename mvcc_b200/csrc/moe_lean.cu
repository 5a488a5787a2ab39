// moe_lean.cu -- compact single-launch decode kernel of the MoE block for one or two tokens (qwen.cu:429-448 end
// to end). Opt-in (MOE_B200_LEAN=1): at batch 1 of the Qwen3.5-MoE geometry it measured 24.6 us per step against
// 21.2 us for the ring kernel (moe_fused.cu), which stays the default decode path for every batch up to 8.
//
// Three measurements of the ring kernel at batch 1 (clock64 stamps per CTA) set its design:
//  * Code size. The ring kernel's machine code is ~126 KB, more than the SM's instruction caches hold. Every phase
//    runs once per launch, so each phase starts with instruction fetches from L2 (the `no_instruction` stall of its
//    ncu profile), and its dot-product loops ran 3-10x slower than their instruction count. This kernel keeps one
//    instance of each loop body: one call site per dot product, and outer loops left rolled.
//  * Per-warp arrival. Each warp issues the bulk copies of its own gate/up jobs and waits on its own mbarrier. It
//    starts computing as soon as its own rows land, not when the CTA's whole share has arrived.
//  * No serial step after routing. The unique-expert table is one 32-lane sort, and every warp derives its job
//    range arithmetically.
// The norm weights, router rows and shared-expert rows do not depend on the previous kernel; they are requested
// before griddepcontrol.wait.
//
// One CTA per SM (cooperative launch), 16 warps:
//   entry  warp 0: mbarriers, then bulk copies of this CTA's two router rows (the shared gate vector is row E), its
//          four shared-expert gate/up row pairs and its shared-expert down rows [h0, h1); every thread: the norm
//          weights; then griddepcontrol.wait, hidden and attn_out;
//   R      RMSNorm of every token into shared memory (fp32, permuted); warps 0-1: the router rows -> logits;
//          arrive at grid barrier 1; warps 2-5: the shared-expert pairs -> sinter while the barrier settles; wait;
//   G      warp t: top-k of token t over all logits (the reference's rule); warp 0: the unique-expert table;
//          warp w: bulk copies of its part of the CTA's contiguous share of the U x I routed gate/up jobs, wait,
//          dot products -> inter (global); warp 15 also issues the CTA's down rows (rows [h0, h1) of every unique
//          expert), which land while the gate/up work runs; grid barrier 2;
//   D      stage every pair's inter and sinter; warp w reduces output row h0 + w over the unique experts' pairs
//          (weighted, pair order) and the shared expert, and applies the gated residual combine; the last CTA to
//          finish optionally applies the next layer's RMSNorm.
// Shared memory is reused across phases. The region of the router and shared gate/up rows later takes the down rows.
// The region of the gate/up jobs later takes the staged inter. Bounded waits, grid barriers, error reporting and
// every reduction order are those of the ring kernel.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "moe_lean.h"
#include "moe_sync.cuh"

namespace moe {

namespace {
constexpr int kLW = 16;
constexpr int kLThreads = kLW * 32;
constexpr int kLRouter = 2;  // router rows per CTA (E + 1 <= 2 x grid)
constexpr int kLSgu = 4;     // shared gate/up pairs per CTA (Is <= 4 x grid)
constexpr int kLMaxP = 32;   // pairs (T x TOPK) the one-warp table sorts
}  // namespace

struct LeanArgs {
  BlockArgs a;
  unsigned long long* gbar;  // grid-barrier arrival counter
  int rpc;                   // output rows h per CTA (at most kLW)
  int jmax;                  // gate/up job slots per CTA
  int umax;                  // unique-expert slots for the down rows
  int next_norm;             // apply the next layer's RMSNorm
  uint32_t o_xs, o_a, o_sdn, o_b, o_sin;  // shared-memory offsets (bytes)
};

// Bytes of the down rows' scale slot of one unique expert: the 16-byte aligned superset of rpc scale rows.
__host__ __device__ inline int lean_dscale_slot(int rpc, int I, int G) { return ((rpc * (I / G) * 2 + 15) & ~15) + 16; }

__global__ void __launch_bounds__(kLThreads, 1) moe_lean_decode_kernel(const __grid_constant__ LeanArgs f) {
  extern __shared__ __align__(128) uint8_t smem[];
  const BlockArgs& a = f.a;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, H = a.w.H, E = a.w.E, K = a.w.TOPK, I = a.w.I, Is = a.w.Is, G = a.w.G;
  const int P = T * K, nch = H >> 5, nvs = Is >> 3;
  const int grid = gridDim.x, cta = blockIdx.x, rpc = f.rpc, jmax = f.jmax;
  float* xs = reinterpret_cast<float*>(smem + f.o_xs);
  uint8_t* ra = smem + f.o_a;   // router + shared gate/up rows; then the down rows
  uint8_t* sdn = smem + f.o_sdn;
  uint8_t* rb = smem + f.o_b;   // gate/up job rows and scales; then the staged inter
  uint16_t* sin_s = reinterpret_cast<uint16_t*>(smem + f.o_sin);
  __shared__ __align__(8) uint64_t jbar[kLW];
  __shared__ __align__(8) uint64_t rbar, sbar, dbar;
  __shared__ float red[32];
  __shared__ int32_t idx_s[kLMaxP];
  __shared__ float wts_s[kLMaxP];
  __shared__ int uniq_s[kLMaxP], uoff_s[kLMaxP + 1], upairs_s[kLMaxP], ptok_s[kLMaxP], pu_s[kLMaxP];
  __shared__ int nuniq_s, ok_s, is_last, abort_s, dissued_s;
  __shared__ unsigned jissued_s;
  __shared__ unsigned long long base_s;
  const int h0 = cta * rpc, h1 = min(H, h0 + rpc);
  const int rowb = H >> 1, sgb = (H / G) * 2;   // gate/up: row bytes, scale bytes per row
  const int drowb = I >> 1, dsb = (I / G) * 2;  // down: row bytes, scale bytes per row
  const int nrows = E + 1;
  const uint8_t* gscale = reinterpret_cast<const uint8_t*>(a.w.exp_gu_s);
  const uint8_t* dscale = reinterpret_cast<const uint8_t*>(a.w.exp_dn_s);
  uint8_t* sgu = ra + (size_t)kLRouter * H * 2;  // shared gate rows [kLSgu][H], then up rows [kLSgu][H]
  const size_t sc_off = (size_t)2 * jmax * rowb;  // job scale rows within region B
  const size_t dq_bytes = (size_t)f.umax * rpc * drowb;
  const int dsl = lean_dscale_slot(rpc, I, G);

  // ---- entry: barriers and the routing-independent copies (warp 0), the norm weights (every thread)
  const int r0 = min(nrows, kLRouter * cta), r1 = min(nrows, r0 + kLRouter), re = min(r1, E);
  const int j0 = min(Is, kLSgu * cta), j1 = min(Is, j0 + kLSgu);
  if (warp == 0) {
    if (lane == 0) {
      for (int w = 0; w < kLW; ++w) mbar_init(&jbar[w], 1);
      mbar_init(&rbar, 1);
      mbar_init(&sbar, 1);
      mbar_init(&dbar, 1);
      abort_s = 0;
      dissued_s = 0;
      jissued_s = 0u;
      mbar_fence_init();
      expect_tx(&rbar, (uint32_t)((r1 - r0) * H * 2));
      expect_tx(&sbar, (uint32_t)(2 * (j1 - j0) * H * 2 + (h0 < h1 ? (h1 - h0) * Is * 2 : 0)));
    }
    __syncwarp();
    if (lane == 0 && re > r0) bulk_g2s(ra, a.w.router + (int64_t)r0 * H, (re - r0) * H * 2, &rbar);
    if (lane == 1 && r1 > re) bulk_g2s(ra + (size_t)(re - r0) * H * 2, a.w.shared_gate, H * 2, &rbar);
    if (lane == 2 && j1 > j0) bulk_g2s(sgu, a.w.shared_gate_up + (int64_t)j0 * H, (j1 - j0) * H * 2, &sbar);
    if (lane == 3 && j1 > j0)
      bulk_g2s(sgu + (size_t)kLSgu * H * 2, a.w.shared_gate_up + (int64_t)(Is + j0) * H, (j1 - j0) * H * 2, &sbar);
    if (lane == 4 && h0 < h1) bulk_g2s(sdn, a.w.shared_down + (int64_t)h0 * Is, (h1 - h0) * Is * 2, &sbar);
    __syncwarp();
  }
  uint2 wn[2];  // this thread's norm weights, requested before they are needed
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = tid + r * kLThreads;
    if (i < H / 4) wn[r] = reinterpret_cast<const uint2*>(a.w.rms2)[i];
  }
  cta_sync();
  pdl_wait();
  unsigned long long gb = 0;  // thread 0: the barrier counter at entry, consumed before the first arrival
  if (tid == 0) gb = ld_relaxed_u64(f.gbar);

  // ---- R: RMSNorm of every token into xs (fp32, permuted); CTA 0 writes `normed`
#pragma unroll 1
  for (int t = 0; t < T; ++t) {
    float4 hv[2];
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {  // H <= 4096 = 2 x 512 threads x 4
      const int i = tid + r * kLThreads;
      if (i < H / 4) {
        const uint2 d = reinterpret_cast<const uint2*>(a.attn_out + (int64_t)t * H)[i];
        hv[r] = reinterpret_cast<const float4*>(a.hidden + (int64_t)t * H)[i];
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
      const int i = tid + r * kLThreads;
      if (i < H / 4) {
        const uint32_t y0 = f2bf(hv[r].x * inv * lo_bf(wn[r].x)), y1 = f2bf(hv[r].y * inv * hi_bf(wn[r].x));
        const uint32_t y2 = f2bf(hv[r].z * inv * lo_bf(wn[r].y)), y3 = f2bf(hv[r].w * inv * hi_bf(wn[r].y));
        *reinterpret_cast<float4*>(xs + t * H + xperm(i * 4, nch)) =
            make_float4(bf2f(y0), bf2f(y1), bf2f(y2), bf2f(y3));
        if (cta == 0)
          reinterpret_cast<uint2*>(a.normed + (int64_t)t * H)[i] = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
      }
    }
  }
  cta_sync();

  // Router rows (warps 0..1) and, while grid barrier 1 settles, the shared-expert gate/up pairs (warps 2..5): the
  // same per-lane order over 32-k chunks and butterfly sums as gemv_bf16. One loop body serves both: a router row
  // is a "pair" whose up row is absent.
  const bool router_warp = warp < kLRouter && kLRouter * cta + warp < nrows;
  const bool sgu_warp = warp >= kLRouter && warp < kLRouter + kLSgu && kLSgu * cta + (warp - kLRouter) < Is;
#pragma unroll 1
  for (int phase = 0; phase < 2; ++phase) {
    if (phase == 1) {
      if (tid == 0) base_s = (gb / grid) * grid;
      grid_arrive(f.gbar);
    }
    const bool mine = phase == 0 ? router_warp : sgu_warp;
    if (!mine) continue;
    if (!__all_sync(0xffffffffu, bar_wait(phase == 0 ? &rbar : &sbar, 0))) {
      if (lane == 0) {
        atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
        abort_s = 1;
      }
      continue;
    }
    const int r = phase == 0 ? warp : warp - kLRouter;
    const uint8_t* grow = phase == 0 ? ra + (size_t)r * H * 2 : sgu + (size_t)r * H * 2;
    const uint8_t* urow = phase == 0 ? grow : sgu + (size_t)(kLSgu + r) * H * 2;
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      const float4* xs4 = reinterpret_cast<const float4*>(xs + t * H);
      float g = 0.f, u = 0.f;
#pragma unroll 1
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
      if (lane == 0) {
        if (phase == 0) {
          const int row = kLRouter * cta + r;
          if (row < E) a.logits[(int64_t)t * E + row] = a.w.router_bias ? g + a.w.router_bias[row] : g;
          else a.gate[t] = sigmoid(g);
        } else {
          a.sinter[(int64_t)t * Is + kLSgu * cta + r] = f2bf(silu(bf2f(f2bf(g))) * bf2f(f2bf(u)));
        }
      }
      __syncwarp();
    }
  }
  const unsigned long long base = base_s;
  if (!grid_wait(f.gbar, base + grid, a.err, &ok_s) && tid == 0) abort_s = 1;

  // ---- G: top-k per token (warp t), the unique-expert table (warp 0)
  if (warp < T) topk_warp_redux(a.logits + (int64_t)warp * E, E, K, idx_s + warp * K, wts_s + warp * K);
  cta_sync();
  if (warp == 0) {
    // the P <= 32 pairs sorted by (expert, pair index) with a bitonic network, one key per lane; invalid indices
    // sort last and are dropped (same contents and order as build_unique in moe_decode.cu)
    const int e = lane < P ? idx_s[lane] : -1;
    uint32_t v = (lane < P && e >= 0 && e < E) ? ((uint32_t)e << 5) | (uint32_t)lane : 0xffffffffu;
#pragma unroll 1
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll 1
      for (int j = k >> 1; j > 0; j >>= 1) {
        const uint32_t o = __shfl_xor_sync(0xffffffffu, v, j);
        v = (((lane & j) == 0) == ((lane & k) == 0)) ? min(v, o) : max(v, o);
      }
    }
    const bool valid = v != 0xffffffffu;
    const int ev = (int)(v >> 5);
    int prev = __shfl_up_sync(0xffffffffu, ev, 1);
    if (lane == 0) prev = -1;
    const bool first = valid && ev != prev;
    const uint32_t b = __ballot_sync(0xffffffffu, first);
    const int u = __popc(b & (0xffffffffu >> (31 - lane))) - 1;
    const int nvalid = __popc(__ballot_sync(0xffffffffu, valid));
    if (first) {
      uniq_s[u] = ev;
      uoff_s[u] = lane;
    }
    if (valid) {
      const int p = (int)(v & 31);
      upairs_s[lane] = p;
      ptok_s[lane] = p / K;
      pu_s[lane] = u;
    }
    if (lane == 0) {
      nuniq_s = __popc(b);
      uoff_s[__popc(b)] = nvalid;
    }
  }
  cta_sync();
  const int U = nuniq_s, npairs = uoff_s[U];

  // The CTA's share of the U x I gate/up jobs (row pairs), split over the warps; a warp's jobs lie in at most two
  // consecutive unique experts (its range is shorter than I). Job slot k (relative to the CTA's first job) holds
  // its gate row at rb + k * rowb, its up row at rb + (jmax + k) * rowb and its scale rows at sc_off likewise.
  const int J = U * I;
  const int cj0 = (int)((unsigned)cta * (unsigned)J / (unsigned)grid);  // J x grid < 2^32 (plan)
  const int cj1 = (int)((unsigned)(cta + 1) * (unsigned)J / (unsigned)grid);
  const int n = cj1 - cj0;
  const int k0 = warp * n / kLW, k1 = (warp + 1) * n / kLW;
  const bool live0 = !vload(&abort_s);
  if (live0 && k1 > k0) {
    const int ja = cj0 + k0, ua = ja / I, ia = ja - ua * I;
    const int n1 = min(k1 - k0, I - ia);
    const int seg = (lane >> 2) & 1, part = lane & 3;
    const int nk = seg ? (k1 - k0) - n1 : n1, kk = seg ? k0 + n1 : k0;
    const int64_t g0 = nk > 0 ? (int64_t)uniq_s[ua + seg] * 2 * I + (seg ? 0 : ia) : 0;
    const uint32_t mine = (lane < 8 && nk > 0) ? (uint32_t)(nk * (part < 2 ? rowb : sgb)) : 0u;
    const uint32_t tx = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0) {
      fence_proxy_async_smem();
      expect_tx(&jbar[warp], tx);
      atomicOr(&jissued_s, 1u << warp);
    }
    __syncwarp();
    if (lane < 8 && nk > 0) {
      if (part == 0) bulk_g2s(rb + (size_t)kk * rowb, a.w.exp_gu_q + g0 * rowb, nk * rowb, &jbar[warp]);
      else if (part == 1) bulk_g2s(rb + (size_t)(jmax + kk) * rowb, a.w.exp_gu_q + (g0 + I) * rowb, nk * rowb, &jbar[warp]);
      else if (part == 2) bulk_g2s(rb + sc_off + (size_t)kk * sgb, gscale + g0 * sgb, nk * sgb, &jbar[warp]);
      else bulk_g2s(rb + sc_off + (size_t)(jmax + kk) * sgb, gscale + (g0 + I) * sgb, nk * sgb, &jbar[warp]);
    }
    __syncwarp();
  }
  // the down rows of every unique expert for this CTA's output rows: q rows at ra + u * rpc * drowb, scale rows
  // (aligned superset) at ra + dq_bytes + u * dsl
  if (live0 && warp == kLW - 1 && h0 < h1) {
    const int nr = h1 - h0;
    uint32_t mine = 0;
    for (int u = lane >> 1; u < U; u += 16) {
      const int64_t rr = (int64_t)uniq_s[u] * H + h0;
      mine += (lane & 1) == 0 ? (uint32_t)(nr * drowb) : span_bytes(dscale + rr * dsb, nr * dsb);
    }
    const uint32_t tx = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0) {
      fence_proxy_async_smem();
      expect_tx(&dbar, tx);
      dissued_s = 1;
    }
    __syncwarp();
    for (int u = lane >> 1; u < U; u += 16) {
      const int64_t rr = (int64_t)uniq_s[u] * H + h0;
      if ((lane & 1) == 0) bulk_g2s(ra + (size_t)u * rpc * drowb, a.w.exp_dn_q + rr * drowb, nr * drowb, &dbar);
      else bulk_span(ra + dq_bytes + (size_t)u * dsl, dscale + rr * dsb, nr * dsb, &dbar);
    }
    __syncwarp();
  }
  if (cta == 0 && tid < 32) {
    if (tid < P) {
      a.idx[tid] = idx_s[tid];
      a.wts[tid] = wts_s[tid];
    }
    if (tid < npairs) a.upairs[tid] = upairs_s[tid];
    if (tid < U) a.uniq[tid] = uniq_s[tid];
    if (tid <= U) a.uoff[tid] = uoff_s[tid];
    if (tid == 0) *a.nuniq = U;
  }

  // Routed gate/up jobs of this warp, two at a time when consecutive jobs share an expert (the activation loads
  // are shared; a lone job runs as a pair with itself and stores once). Reductions as compute_routed in
  // moe_decode.cu.
  const Nib8Magic M = nib8_magic();
  const int gshift = __ffs(G) - 6, dshift = __ffs(G) - 5;
  if (live0 && k1 > k0) {
    if (!__all_sync(0xffffffffu, bar_wait(&jbar[warp], 0))) {
      if (lane == 0) {
        atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
        abort_s = 1;
      }
    } else {
#pragma unroll 1
      for (int k = k0; k < k1;) {
        const int j = cj0 + k, u = j / I, i = j - u * I;
        const int kb = (k + 1 < k1 && i + 1 < I) ? k + 1 : k;
        const uint8_t* grow0 = rb + (size_t)k * rowb;
        const uint8_t* urow0 = rb + (size_t)(jmax + k) * rowb;
        const uint8_t* grow1 = rb + (size_t)kb * rowb;
        const uint8_t* urow1 = rb + (size_t)(jmax + kb) * rowb;
        const uint16_t* gsc0 = reinterpret_cast<const uint16_t*>(rb + sc_off + (size_t)k * sgb);
        const uint16_t* usc0 = reinterpret_cast<const uint16_t*>(rb + sc_off + (size_t)(jmax + k) * sgb);
        const uint16_t* gsc1 = reinterpret_cast<const uint16_t*>(rb + sc_off + (size_t)kb * sgb);
        const uint16_t* usc1 = reinterpret_cast<const uint16_t*>(rb + sc_off + (size_t)(jmax + kb) * sgb);
#pragma unroll 1
        for (int p = uoff_s[u]; p < uoff_s[u + 1]; ++p) {
          const int pair = upairs_s[p];
          const float* xt = xs + ptok_s[p] * H;
          float g0 = 0.f, u0 = 0.f, g1 = 0.f, u1 = 0.f;
#pragma unroll 1
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
            a.inter[(int64_t)pair * I + i] = f2bf(silu(g0) * u0);
            if (kb != k) a.inter[(int64_t)pair * I + i + 1] = f2bf(silu(g1) * u1);
          }
          __syncwarp();
        }
        k = kb + 1;
      }
    }
  }
  grid_arrive(f.gbar);
  if (!grid_wait(f.gbar, base + 2 * (unsigned long long)grid, a.err, &ok_s) && tid == 0) abort_s = 1;

  // the next kernel on the stream may start its entry on SMs this grid frees from here on
  pdl_launch_dependents();

  // ---- D: stage inter (bf16, permuted) into region B and sinter; reduce this warp's output row
  const int nchd = I >> 4, Ld = min(32, nchd), PI = inter_stride(I);
  uint16_t* inter_s = reinterpret_cast<uint16_t*>(rb);
  for (int x = tid; x < P * I / 8; x += kLThreads) {
    const int p = (x * 8) / I, k = x * 8 - p * I;
    *reinterpret_cast<uint4*>(inter_s + (size_t)p * PI + iperm(k, Ld)) =
        __ldcg(reinterpret_cast<const uint4*>(a.inter) + x);
  }
  for (int x = tid; x < T * Is / 8; x += kLThreads)
    reinterpret_cast<uint4*>(sin_s)[x] = __ldcg(reinterpret_cast<const uint4*>(a.sinter) + x);
  cta_sync();

  const int hw = h0 + warp;
  bool live = !vload(&abort_s) && hw < h1;
  if (live && !__all_sync(0xffffffffu, bar_wait(&dbar, 0))) {
    if (lane == 0) {
      atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
      abort_s = 1;
    }
    live = false;
  }
  float acc0 = 0.f, acc1 = 0.f;  // tokens 0 and 1 (T <= 2)
  if (live) {
    // four pair partials at a time are independent, then they are accumulated in pair order (the order of the
    // three-kernel path)
#pragma unroll 1
    for (int p0 = 0; p0 < npairs; p0 += 4) {
      float part[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        part[q] = 0.f;
        const int p = p0 + q;
        if (p < npairs) {
          const int b = pu_s[p];
          const int64_t rr = (int64_t)uniq_s[b] * H + h0;
          const uint8_t* wr = ra + ((size_t)b * rpc + warp) * drowb;
          const uint16_t* sc = reinterpret_cast<const uint16_t*>(ra + dq_bytes + (size_t)b * dsl +
                                                                 span_delta(dscale + rr * dsb) + warp * dsb);
          const uint8_t* xr = reinterpret_cast<const uint8_t*>(inter_s + (size_t)upairs_s[p] * PI);
#pragma unroll 1
          for (int cc = lane; cc < nchd; cc += 32) {
            const int jj = cc >> 5;
            const uint2 wq = *reinterpret_cast<const uint2*>(wr + cc * 8);
            u64 x01, x23, x45, x67;
            Nib8Acc A;
            nib8_zero(A);
            inter_pairs<false>(xr + (size_t)((jj * 2) * Ld + lane) * 16, x01, x23, x45, x67);
            nib8x2(wq.x, x01, x23, x45, x67, M, A);
            inter_pairs<false>(xr + (size_t)((jj * 2 + 1) * Ld + lane) * 16, x01, x23, x45, x67);
            nib8x2(wq.y, x01, x23, x45, x67, M, A);
            part[q] = fmaf(nib8_fold(A), h2f(sc[cc >> dshift]), part[q]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int p = p0 + q;
        if (p < npairs) {
          const float wgt = wts_s[upairs_s[p]];
          if (ptok_s[p] == 0) acc0 = fmaf(wgt, part[q], acc0);
          else acc1 = fmaf(wgt, part[q], acc1);
        }
      }
    }
  }
  bool sdn_ok = live;
  if (sdn_ok) {
    sdn_ok = __all_sync(0xffffffffu, bar_wait(&sbar, 0));
    if (!sdn_ok && lane == 0) {  // this warp's output row is not written: the call's results are invalid
      atomicOr(a.err, (uint32_t)MOE_ERR_BARRIER);
      abort_s = 1;
    }
  }
  if (sdn_ok) {
    const float rt0 = warp_sum(acc0), rt1 = warp_sum(acc1);
    const float routed_t = lane == 0 ? rt0 : rt1;
    const uint8_t* srow = sdn + (size_t)(hw - h0) * Is * 2;
    float shared_t = 0.f;
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      float acc = 0.f;
#pragma unroll 1
      for (int v = lane; v < nvs; v += 32) {
        const uint4 wv = *reinterpret_cast<const uint4*>(srow + v * 16);
        const uint4 xv = *reinterpret_cast<const uint4*>(sin_s + t * Is + v * 8);
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
  // consumers; after an abort, wait (bounded) for every copy this CTA issued.
  cta_sync();
  if (tid == 0 && vload(&abort_s)) {
#pragma unroll 1
    for (int w = 0; w < kLW; ++w)
      if (jissued_s & (1u << w)) bar_wait(&jbar[w], 0);
    if (dissued_s) bar_wait(&dbar, 0);
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
#pragma unroll 1
  for (int t = 0; t < T; ++t) {
    const float* hr = a.hidden + (int64_t)t * H;
    float ss = 0.f;
    for (int i = tid; i < H; i += kLThreads) {
      const float v = __ldcg(hr + i);
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)H + a.w.eps);
    for (int i = tid; i < H; i += kLThreads)
      a.normed[(int64_t)t * H + i] = f2bf(__ldcg(hr + i) * inv * bf2f(a.next_rms1[i]));
  }
}

// ------------------------------------------------------------------ host side

namespace {
int lean_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}
int lean_smem_optin() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (n <= 0) n = 227 * 1024;
  }
  return n;
}
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
size_t up128(size_t x) { return (x + 127) & ~(size_t)127; }
// On when the environment sets MOE_B200_LEAN=1 (read once per process); otherwise the ring kernel serves T <= 2.
bool lean_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("MOE_B200_LEAN");
    on = (v && v[0] == '1') ? 1 : 0;
  }
  return on == 1;
}
bool lean_pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("MOE_B200_PDL");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

struct LeanCfg {
  int rpc, jmax, umax;
  uint32_t o_xs, o_a, o_sdn, o_b, o_sin;
  size_t smem;
};

bool lean_plan(const moe_layer_weights& w, int T, LeanCfg* c) {
  if (!lean_enabled() || T < 1 || T > kLeanMaxT) return false;
  const int P = T * w.TOPK, grid = lean_sms();
  if (P > kLMaxP || w.E + 1 > kLRouter * grid || w.Is > kLSgu * grid || w.H > 4096) return false;
  if ((w.H / w.G) % 8 != 0 || w.I % 32 != 0) return false;  // whole 16-byte scale rows and down rows
  if (!al16(w.router) || !al16(w.shared_gate) || !al16(w.shared_gate_up) || !al16(w.shared_down) ||
      !al16(w.exp_gu_q) || !al16(w.exp_dn_q) || !al16(w.exp_gu_s) || !al16(w.exp_dn_s))
    return false;
  const int rpc = (w.H + grid - 1) / grid;
  if (rpc > kLW) return false;  // one output row per warp
  const int umax = std::min(w.E, P);
  const int jmax = (umax * w.I + grid - 1) / grid;
  if ((jmax + kLW - 1) / kLW > w.I) return false;  // a warp's jobs span at most two experts
  if ((long long)umax * w.I * (grid + 1) >= (1ll << 32)) return false;  // job ranges in 32-bit arithmetic
  const size_t rowb = w.H / 2, sgb = (size_t)(w.H / w.G) * 2;
  const size_t reg_a = std::max((size_t)kLRouter * w.H * 2 + (size_t)2 * kLSgu * w.H * 2,
                                (size_t)umax * rpc * (w.I / 2) + (size_t)umax * lean_dscale_slot(rpc, w.I, w.G));
  const size_t reg_b = std::max((size_t)2 * jmax * rowb + (size_t)2 * jmax * sgb,
                                (size_t)P * inter_stride(w.I) * 2);
  size_t o = 0;
  c->o_xs = (uint32_t)o;  o = up128(o + (size_t)T * w.H * 4);
  c->o_a = (uint32_t)o;   o = up128(o + reg_a);
  c->o_sdn = (uint32_t)o; o = up128(o + (size_t)rpc * w.Is * 2);
  c->o_b = (uint32_t)o;   o = up128(o + reg_b);
  c->o_sin = (uint32_t)o; o = up128(o + (size_t)T * w.Is * 2);
  if ((int)o > lean_smem_optin() - 4 * 1024) return false;  // static shared memory of the kernel
  c->rpc = rpc;
  c->jmax = jmax;
  c->umax = umax;
  c->smem = o;
  return true;
}
}  // namespace

bool lean_config(const moe_layer_weights& w, int T) {
  LeanCfg c;
  return lean_plan(w, T, &c);
}

cudaError_t launch_lean_decode(const BlockArgs& a, unsigned long long* gbar, bool next_norm, cudaStream_t s) {
  LeanCfg c;
  if (!lean_plan(a.w, a.T, &c)) return cudaErrorInvalidValue;
  static SmemGrant granted;
  cudaError_t e = grant_smem(reinterpret_cast<const void*>(moe_lean_decode_kernel), c.smem, (size_t)160 * 1024, granted);
  if (e != cudaSuccess) return e;
  LeanArgs f;
  memset(&f, 0, sizeof f);
  f.a = a;
  f.gbar = gbar;
  f.rpc = c.rpc;
  f.jmax = c.jmax;
  f.umax = c.umax;
  f.next_norm = next_norm ? 1 : 0;
  f.o_xs = c.o_xs;
  f.o_a = c.o_a;
  f.o_sdn = c.o_sdn;
  f.o_b = c.o_b;
  f.o_sin = c.o_sin;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lean_sms());
  cfg.blockDim = dim3(kLThreads);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lean_pdl_enabled() ? 2 : 1;
  return launched(cudaLaunchKernelEx(&cfg, moe_lean_decode_kernel, f));
}

}  // namespace moe
