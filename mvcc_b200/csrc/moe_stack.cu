// moe_stack.cu -- the attention layer and the LM head of a decode step (include/moe_stack.h): the reference's
// attention branch of forward() (qwen.cu:413-425) and its LM head (qwen.cu:451-456), rebuilt for B200.
//
// Every piece streams weights or cache rows from HBM once, so each kernel is sized for memory-level parallelism:
//   dense_gemv_kernel   y = x . W^T for T <= 4 tokens (qkv, gate, o, LM head): each warp walks its rows in 4 KB
//                       chunks (16-byte streaming loads, one row per warp at a time), two chunks in flight per
//                       warp, two CTAs per SM; x staged in shared memory in a bank-conflict-free order. The first
//                       chunk is requested before griddepcontrol.wait, so under programmatic dependent launch it
//                       streams while the previous kernel finishes. The LM-head variant keeps each warp's best
//                       (logit, index) and the last CTA to finish (a ticket) reduces the CTAs' results: argmax
//                       fused into the GEMV, one launch.
//   attn_split_kernel   split-K decode attention (kernels.cuh:665-761) with the per-head RMSNorm + rotate-half RoPE
//                       of attn_qk_norm_rope_kernel (kernels.cuh:608-663) fused in: CTA (token, kv head, split)
//                       copies its chunk of K and V rows into shared memory with two bulk copies; meanwhile warp g
//                       normalises and rotates query head g; the step's new keys that fall in the chunk are
//                       normalised, rotated and placed into the staged chunk (the token's own key and value row
//                       also into the caches); then warp g scores the chunk: 32 keys' partial dot products per
//                       lane, one 31-shuffle reduce-scatter that leaves key j's score in lane j, online softmax,
//                       acc += p v. Partials (acc, max, sum) per split; about two CTAs per SM.
//   attn_combine_kernel merges the splits in one pass (online-softmax merging, eight splits' loads in flight per
//                       warp) and applies the optional sigmoid gate (kernels.cuh:765-769).
#include <algorithm>
#include <cstring>

#include "../../include/moe_stack.h"
#include "moe_common.cuh"
#include "moe_device.cuh"
#include "moe_sync.cuh"

namespace moe {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvU = 8;          // 16-byte loads per lane per chunk (a 4 KB chunk of one row)
constexpr int kStackMaxT = 4;
constexpr int kAttnMaxChunk = 64;  // keys per split at most (shared memory: 2 x 64 x 512 B)
constexpr int kArgmaxMaxCtas = 1024;
// Floats per split-K partial: acc [D], max, sum, padded to a multiple of 4 so that every partial starts on a 16-byte
// boundary (its acc is stored as float4).
__host__ __device__ constexpr int part_stride(int D) { return D + 4; }

enum { EPI_BF16 = 0, EPI_ARGMAX = 1 };

struct GemvArgs {
  const uint16_t* x;   // bf16 [T][K], or (x == null):
  const float* xf;     //   fp32 [T][K] rows normalised in the prologue: bf16(xf * rsqrt(mean(xf^2) + eps) * xw)
  const uint16_t* xw;  //   bf16 [K]
  float eps;
  const uint16_t* w0;  // bf16 [n0][K]
  const uint16_t* w1;  // bf16 [N - n0][K] (rows n0 .. N - 1), may be null when n0 == N
  int n0, N, K, T;
  uint16_t* y0;        // bf16 [T][n0]
  uint16_t* y1;        // bf16 [T][N - n0]
  // argmax (T == 1)
  float* logits;       // fp32 [N] or null
  float* pv;           // per-CTA best value
  int32_t* pi;         // per-CTA best index
  uint32_t* ticket;
  int32_t* next;
};

// Position of the 4-float half h of 16-byte unit i (k = 8 i .. 8 i + 7) in the staged x row: lanes reading
// consecutive units hit consecutive 16-byte words.
__device__ __forceinline__ int xs_pos(int i, int h, int nu) { return (h * nu + i) * 4; }

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// MT: the most tokens this instantiation handles (1, or kStackMaxT): the single-token build carries a quarter of the
// inner-loop code, which matters for short launches that start on a cold instruction cache.
template <int EPI, int MT>
__global__ void __launch_bounds__(kGemvWarps * 32, 2) dense_gemv_kernel(const __grid_constant__ GemvArgs g) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float bv_s[kGemvWarps];
  __shared__ int bi_s[kGemvWarps];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = g.K, N = g.N, T = g.T, nu = K >> 3;
  constexpr int kChunk = 32 * kGemvU;  // 16-byte units per chunk (4 KB of a row)
  const int cpr = (nu + kChunk - 1) / kChunk;
  // warp wg owns rows wg, wg + nw, ...; its chunks run row by row, cpr chunks per row
  const int wg = blockIdx.x * kGemvWarps + warp, nw = gridDim.x * kGemvWarps;
  const int nrows = wg < N ? (N - 1 - wg) / nw + 1 : 0;
  const int nch = nrows * cpr;
  auto row_ptr = [&](int r) -> const uint4* {
    const uint16_t* base = r < g.n0 ? g.w0 + (int64_t)r * K : g.w1 + (int64_t)(r - g.n0) * K;
    return reinterpret_cast<const uint4*>(base);
  };
  auto load = [&](uint4 (&w)[kGemvU], int c) {
    const int q = c / cpr, part = c - q * cpr;
    const uint4* p = row_ptr(wg + q * nw);
#pragma unroll
    for (int u = 0; u < kGemvU; ++u) {
      const int i = part * kChunk + u * 32 + lane;
      w[u] = i < nu ? ldg_stream(p + i) : make_uint4(0, 0, 0, 0);
    }
  };
  // two chunks in flight per warp; weights do not depend on the previous kernel: the first two are requested before
  // waiting for it
  uint4 wa[kGemvU], wb[kGemvU];
  if (nch > 0) load(wa, 0);
  if (nch > 1) load(wb, 1);
  pdl_wait();
  pdl_launch_dependents();
  // x -> shared memory (fp32, permuted)
  if (g.x) {
    for (int e = threadIdx.x; e < T * nu; e += blockDim.x) {
      const int t = e / nu, i = e - t * nu;
      const uint4 v = reinterpret_cast<const uint4*>(g.x + (int64_t)t * K)[i];
      float* dst = xs + t * K;
      *reinterpret_cast<float4*>(dst + xs_pos(i, 0, nu)) = make_float4(lo_bf(v.x), hi_bf(v.x), lo_bf(v.y), hi_bf(v.y));
      *reinterpret_cast<float4*>(dst + xs_pos(i, 1, nu)) = make_float4(lo_bf(v.z), hi_bf(v.z), lo_bf(v.w), hi_bf(v.w));
    }
  } else {
    // every CTA normalises the rows itself (rmsnorm_kernel, kernels.cuh:83-93): x = bf16(xf * inv * xw)
    for (int t = 0; t < T; ++t) {
      const float4* row = reinterpret_cast<const float4*>(g.xf + (int64_t)t * K);
      float ss = 0.f;
      for (int i = threadIdx.x; i < K / 4; i += blockDim.x) {
        const float4 v = __ldcg(row + i);
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      }
      ss = warp_sum(ss);
      if (lane == 0) bv_s[warp] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) tot += bv_s[w];
      const float inv = rsqrtf(tot / (float)K + g.eps);
      __syncthreads();  // bv_s is reused by the next row
      float* dst = xs + t * K;
      for (int i = threadIdx.x; i < nu; i += blockDim.x) {
        const float4 a = __ldcg(row + 2 * i), b = __ldcg(row + 2 * i + 1);
        const uint4 wv = reinterpret_cast<const uint4*>(g.xw)[i];
        *reinterpret_cast<float4*>(dst + xs_pos(i, 0, nu)) =
            make_float4(bf2f(f2bf(a.x * inv * lo_bf(wv.x))), bf2f(f2bf(a.y * inv * hi_bf(wv.x))),
                        bf2f(f2bf(a.z * inv * lo_bf(wv.y))), bf2f(f2bf(a.w * inv * hi_bf(wv.y))));
        *reinterpret_cast<float4*>(dst + xs_pos(i, 1, nu)) =
            make_float4(bf2f(f2bf(b.x * inv * lo_bf(wv.z))), bf2f(f2bf(b.y * inv * hi_bf(wv.z))),
                        bf2f(f2bf(b.z * inv * lo_bf(wv.w))), bf2f(f2bf(b.w * inv * hi_bf(wv.w))));
      }
    }
  }
  __syncthreads();
  float best_v = -1e30f;
  int best_i = 0;
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) acc[t] = 0.f;
  auto compute = [&](const uint4 (&w)[kGemvU], int c) {
    const int q = c / cpr, part = c - q * cpr;
#pragma unroll
    for (int u = 0; u < kGemvU; ++u) {
      const int i = part * kChunk + u * 32 + lane;
      if (i >= nu) break;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (t >= T) break;
        const float4 x0 = *reinterpret_cast<const float4*>(xs + t * K + xs_pos(i, 0, nu));
        const float4 x1 = *reinterpret_cast<const float4*>(xs + t * K + xs_pos(i, 1, nu));
        float a = acc[t];
        a = fmaf(lo_bf(w[u].x), x0.x, a);
        a = fmaf(hi_bf(w[u].x), x0.y, a);
        a = fmaf(lo_bf(w[u].y), x0.z, a);
        a = fmaf(hi_bf(w[u].y), x0.w, a);
        a = fmaf(lo_bf(w[u].z), x1.x, a);
        a = fmaf(hi_bf(w[u].z), x1.y, a);
        a = fmaf(lo_bf(w[u].w), x1.z, a);
        a = fmaf(hi_bf(w[u].w), x1.w, a);
        acc[t] = a;
      }
    }
    if (part != cpr - 1) return;
    // the row is complete: reduce across the warp (every lane gets the sums), store or keep the best
    const int r = wg + q * nw;
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = warp_sum(acc[t]);
    if (EPI == EPI_BF16) {
      if (lane < T) {
        float v = acc[0];
#pragma unroll
        for (int t = 1; t < MT; ++t)
          if (lane == t) v = acc[t];
        if (r < g.n0) g.y0[(int64_t)lane * g.n0 + r] = f2bf(v);
        else g.y1[(int64_t)lane * (N - g.n0) + (r - g.n0)] = f2bf(v);
      }
    } else {
      const float v = acc[0];
      if (lane == 0 && g.logits) g.logits[r] = v;
      if (better(v, r, best_v, best_i)) {
        best_v = v;
        best_i = r;
      }
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = 0.f;
  };
  for (int c = 0; c < nch; c += 2) {
    compute(wa, c);
    if (c + 2 < nch) load(wa, c + 2);
    if (c + 1 < nch) {
      compute(wb, c + 1);
      if (c + 3 < nch) load(wb, c + 3);
    }
  }
  if (EPI != EPI_ARGMAX) return;
  // argmax: warp -> CTA -> (last CTA) grid, ties to the lowest index at every level
  if (lane == 0) {
    bv_s[warp] = best_v;
    bi_s[warp] = best_i;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = bv_s[0];
    int i = bi_s[0];
    for (int w = 1; w < kGemvWarps; ++w)
      if (better(bv_s[w], bi_s[w], v, i)) {
        v = bv_s[w];
        i = bi_s[w];
      }
    g.pv[blockIdx.x] = v;
    g.pi[blockIdx.x] = i;
    __threadfence();
    is_last = atomicInc(g.ticket, gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  float v = -1e30f;
  int idx = 0;
  for (int c = threadIdx.x; c < (int)gridDim.x; c += blockDim.x) {
    const float cv = __ldcg(g.pv + c);
    const int ci = __ldcg(g.pi + c);
    if (better(cv, ci, v, idx)) {
      v = cv;
      idx = ci;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (better(ov, oi, v, idx)) {
      v = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    bv_s[warp] = v;
    bi_s[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kGemvWarps; ++w)
      if (better(bv_s[w], bi_s[w], v, idx)) {
        v = bv_s[w];
        idx = bi_s[w];
      }
    *g.next = idx;
  }
}

// Split-K decode attention, GQA, with the per-head norm + RoPE of its inputs fused in. CTA (job = t * Hkv + kv head,
// split sp); warp g < G handles query head kvh * G + g over keys [k0, k1) of the split. D == 256: lane owns dims
// 8 lane .. 8 lane + 7.
struct AttnArgs {
  const uint16_t* qkv;     // bf16 [T][(Hq + 2 Hkv) D]: q heads, k heads, v heads of the new tokens
  const uint16_t* q_norm;  // bf16 [D]
  const uint16_t* k_norm;  // bf16 [D]
  uint16_t* kc;            // bf16 [Hkv][ctx][D]
  uint16_t* vc;
  float* part;  // [(t * Hq + h) * nsplit + sp][part_stride(D)]: acc, max, sum
  uint32_t* err;
  int T, Hq, Hkv, ctx, pos0, nsplit, rope_dim;
  float scale, theta, eps;
};

// RMSNorm of one head row (lane holds dims 8 lane .. + 7 in v), times the norm weights, then rotate-half RoPE over
// the first rope_dim dims at position pos (attn_qk_norm_rope_kernel, kernels.cuh:608-663): dim d < rope_dim / 2
// pairs with d + rope_dim / 2, which another lane holds.
__device__ __forceinline__ void head_norm_rope(float (&v)[8], const uint16_t* w, int rope_dim, float theta, int pos,
                                               float eps, int lane) {
  constexpr int D = 256;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
  const uint4 wv = *reinterpret_cast<const uint4*>(w + lane * 8);
  const float wf[8] = {lo_bf(wv.x), hi_bf(wv.x), lo_bf(wv.y), hi_bf(wv.y),
                       lo_bf(wv.z), hi_bf(wv.z), lo_bf(wv.w), hi_bf(wv.w)};
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * wf[i];
  const int half = rope_dim >> 1, hl = half >> 3;  // lanes per half (half is a multiple of 32)
  const bool rot = lane < 2 * hl, first = lane < hl;
  const int src = rot ? (first ? lane + hl : lane - hl) : lane;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float other = __shfl_sync(0xffffffffu, v[i], src);
    if (rot) {
      const int d = (first ? lane : lane - hl) * 8 + i;  // the dim below half of this pair
      // the reference's fast intrinsics (kernels.cuh:650-653): its rounding, and no slow-path code in this kernel
      const float inv_freq = __powf(theta, -(float)(2 * d) / (float)rope_dim);
      float sn, cs;
      __sincosf((float)pos * inv_freq, &sn, &cs);
      v[i] = first ? v[i] * cs - other * sn : v[i] * cs + other * sn;
    }
  }
}

__global__ void __launch_bounds__(256) attn_split_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int D = 256;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t kvbar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int job = blockIdx.x, sp = blockIdx.y;
  const int t = job / a.Hkv, kvh = job - t * a.Hkv;
  const int G = a.Hq / a.Hkv, heads = a.Hq + 2 * a.Hkv;
  const int nkeys = a.pos0 + t + 1;
  const int chunk = (nkeys + a.nsplit - 1) / a.nsplit;
  const int k0 = min(nkeys, sp * chunk), k1 = min(nkeys, k0 + chunk), n = k1 - k0;
  uint8_t* ks = smem;
  uint8_t* vs = smem + (size_t)chunk * D * 2;
  // The cached rows do not depend on the previous kernel (the qkv GEMV): the caches were last written by earlier
  // steps' launches, which completed before that kernel started. So the chunk is requested before
  // griddepcontrol.wait and streams in while the GEMV finishes; rows of this step's new keys are overwritten below.
  if (threadIdx.x == 0) {
    mbar_init(&kvbar, 1);
    mbar_fence_init();
    expect_tx(&kvbar, (uint32_t)(2 * n * D * 2));
    if (n > 0) {
      bulk_g2s(ks, a.kc + ((int64_t)kvh * a.ctx + k0) * D, n * D * 2, &kvbar);
      bulk_g2s(vs, a.vc + ((int64_t)kvh * a.ctx + k0) * D, n * D * 2, &kvbar);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  // while the chunk lands: warp g normalises and rotates its query head (bf16, as stored by the reference)
  float qf[8];
  if (warp < G) {
    const int h = kvh * G + warp;
    const uint4 qv = reinterpret_cast<const uint4*>(a.qkv + ((int64_t)t * heads + h) * D)[lane];
    float v[8] = {lo_bf(qv.x), hi_bf(qv.x), lo_bf(qv.y), hi_bf(qv.y), lo_bf(qv.z), hi_bf(qv.z), lo_bf(qv.w), hi_bf(qv.w)};
    head_norm_rope(v, a.q_norm, a.rope_dim, a.theta, a.pos0 + t, a.eps, lane);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] = bf2f(f2bf(v[i])) * a.scale;
  }
  const bool ok = bar_wait(&kvbar, 0);
  if (!ok && threadIdx.x == 0) atomicOr(a.err, (uint32_t)MOE_ERR_TIMEOUT);
  // keys of this step's tokens (positions pos0 .. pos0 + t) inside the chunk: the cache does not hold them yet, so
  // they are normalised and rotated here (k) or copied (v) into the staged chunk; token t's own key also goes to the
  // caches (this CTA is the only one whose token ends at that position)
  const int p0 = max(k0, a.pos0);
  for (int p = p0 + warp; p < k1; p += blockDim.x >> 5) {
    const int tn = p - a.pos0;
    const uint16_t* row = a.qkv + (int64_t)tn * heads * D;
    const uint4 kr = reinterpret_cast<const uint4*>(row + (int64_t)(a.Hq + kvh) * D)[lane];
    const uint4 vr = reinterpret_cast<const uint4*>(row + (int64_t)(a.Hq + a.Hkv + kvh) * D)[lane];
    float v[8] = {lo_bf(kr.x), hi_bf(kr.x), lo_bf(kr.y), hi_bf(kr.y), lo_bf(kr.z), hi_bf(kr.z), lo_bf(kr.w), hi_bf(kr.w)};
    head_norm_rope(v, a.k_norm, a.rope_dim, a.theta, p, a.eps, lane);
    const uint4 ko = make_uint4((uint32_t)f2bf(v[0]) | ((uint32_t)f2bf(v[1]) << 16),
                                (uint32_t)f2bf(v[2]) | ((uint32_t)f2bf(v[3]) << 16),
                                (uint32_t)f2bf(v[4]) | ((uint32_t)f2bf(v[5]) << 16),
                                (uint32_t)f2bf(v[6]) | ((uint32_t)f2bf(v[7]) << 16));
    if (ok) {  // after a wait that gave up the copies may still land here: leave the stage to them
      *reinterpret_cast<uint4*>(ks + (size_t)(p - k0) * D * 2 + lane * 16) = ko;
      *reinterpret_cast<uint4*>(vs + (size_t)(p - k0) * D * 2 + lane * 16) = vr;
    }
    if (tn == t) {
      reinterpret_cast<uint4*>(a.kc + ((int64_t)kvh * a.ctx + p) * D)[lane] = ko;
      reinterpret_cast<uint4*>(a.vc + ((int64_t)kvh * a.ctx + p) * D)[lane] = vr;
    }
  }
  __syncthreads();
  // no copy may still be landing when the CTA exits: after a wait that gave up, thread 0 waits once more (bounded)
  if (!ok && threadIdx.x == 0) bar_wait(&kvbar, 0);
  if (warp >= G) return;
  const int h = kvh * G + warp;
  float m = -1e30f, l = 0.f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  if (ok) {
    for (int g0 = 0; g0 < n; g0 += 32) {
      const int ng = min(32, n - g0);
      // partial dot products of up to 32 keys, then a reduce-scatter: lane j ends with key g0 + j's score
      float s[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        s[j] = 0.f;
        if (j < ng) {
          const uint4 kv = *reinterpret_cast<const uint4*>(ks + (size_t)(g0 + j) * D * 2 + lane * 16);
          float d = qf[0] * lo_bf(kv.x);
          d = fmaf(qf[1], hi_bf(kv.x), d);
          d = fmaf(qf[2], lo_bf(kv.y), d);
          d = fmaf(qf[3], hi_bf(kv.y), d);
          d = fmaf(qf[4], lo_bf(kv.z), d);
          d = fmaf(qf[5], hi_bf(kv.z), d);
          d = fmaf(qf[6], lo_bf(kv.w), d);
          d = fmaf(qf[7], hi_bf(kv.w), d);
          s[j] = d;
        }
      }
#pragma unroll
      for (int w = 16; w >= 1; w >>= 1) {
        const bool up = (lane & w) != 0;
#pragma unroll
        for (int i = 0; i < w; ++i) {
          const float send = up ? s[i] : s[i + w];
          const float keep = up ? s[i + w] : s[i];
          s[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
        }
      }
      const float sc = lane < ng ? s[0] : -1e30f;
      float gm = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
      const float m_new = fmaxf(m, gm);
      const float corr = __expf(m - m_new);
      const float p = lane < ng ? __expf(sc - m_new) : 0.f;
      l = l * corr + warp_sum(p);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= corr;
      for (int j = 0; j < ng; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const uint4 vv = *reinterpret_cast<const uint4*>(vs + (size_t)(g0 + j) * D * 2 + lane * 16);
        acc[0] = fmaf(pj, lo_bf(vv.x), acc[0]);
        acc[1] = fmaf(pj, hi_bf(vv.x), acc[1]);
        acc[2] = fmaf(pj, lo_bf(vv.y), acc[2]);
        acc[3] = fmaf(pj, hi_bf(vv.y), acc[3]);
        acc[4] = fmaf(pj, lo_bf(vv.z), acc[4]);
        acc[5] = fmaf(pj, hi_bf(vv.z), acc[5]);
        acc[6] = fmaf(pj, lo_bf(vv.w), acc[6]);
        acc[7] = fmaf(pj, hi_bf(vv.w), acc[7]);
      }
      m = m_new;
    }
  }
  float* dst = a.part + (((int64_t)t * a.Hq + h) * a.nsplit + sp) * part_stride(D);
  *reinterpret_cast<float4*>(dst + lane * 8) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  *reinterpret_cast<float4*>(dst + lane * 8 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  if (lane == 0) {
    dst[D] = m;
    dst[D + 1] = l;
  }
}

// Merge of the nsplit partials of each (token, query head): CTA (job, part) handles dims [32 part, +32); warp w merges
// splits w, w + 8, ... eight at a time (their loads issued together) into a running (max, sum, acc) as online softmax
// does, and warp 0 merges the eight warps' results in warp order; o = bf16(acc / sum), then optionally
// o = bf16(o * sigmoid(gate)).
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ part, const uint16_t* __restrict__ z,
                                                           uint16_t* __restrict__ o, int nsplit) {
  constexpr int D = 256, kW = 8, kB = 8;
  __shared__ float acc_s[kW][32], l_s[kW], m_s[kW];
  pdl_wait();
  pdl_launch_dependents();
  const int job = blockIdx.x >> 3, prt = blockIdx.x & 7;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, d = prt * 32 + lane;
  constexpr int PS = part_stride(D);
  const float* src = part + (int64_t)job * nsplit * PS;
  float m = -1e30f, l = 0.f, acc = 0.f;
  for (int s0 = warp; s0 < nsplit; s0 += kW * kB) {
    float pm[kB], pl[kB], pv[kB];
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int s = s0 + k * kW;
      const float* p = src + (int64_t)min(s, nsplit - 1) * PS;
      pm[k] = __ldcg(p + D);
      pl[k] = s < nsplit ? __ldcg(p + D + 1) : 0.f;
      pv[k] = __ldcg(p + d);
    }
    float mn = m;
#pragma unroll
    for (int k = 0; k < kB; ++k)
      if (pl[k] > 0.f) mn = fmaxf(mn, pm[k]);
    const float c0 = __expf(m - mn);
    l *= c0;
    acc *= c0;
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const float c = pl[k] > 0.f ? __expf(pm[k] - mn) : 0.f;
      l = fmaf(pl[k], c, l);
      acc = fmaf(pv[k], c, acc);
    }
    m = mn;
  }
  acc_s[warp][lane] = acc;
  if (lane == 0) {
    l_s[warp] = l;
    m_s[warp] = m;
  }
  __syncthreads();
  if (warp != 0) return;
  float gm = -1e30f;
#pragma unroll
  for (int w = 0; w < kW; ++w)
    if (l_s[w] > 0.f) gm = fmaxf(gm, m_s[w]);
  float tot = 0.f, lsum = 0.f;
#pragma unroll
  for (int w = 0; w < kW; ++w) {
    const float c = l_s[w] > 0.f ? __expf(m_s[w] - gm) : 0.f;
    tot = fmaf(acc_s[w][lane], c, tot);
    lsum = fmaf(l_s[w], c, lsum);
  }
  uint16_t ov = f2bf(tot / lsum);
  if (z) ov = f2bf(bf2f(ov) * sigmoid(bf2f(z[(int64_t)job * D + d])));
  o[(int64_t)job * D + d] = ov;
}

// One CTA per row: y = bf16(x * rsqrt(mean(x^2) + eps) * w).
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, const uint16_t* __restrict__ w,
                                                           uint16_t* __restrict__ y, int H, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const float* row = x + (int64_t)blockIdx.x * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(row[i], row[i], ss);
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) y[(int64_t)blockIdx.x * H + i] = f2bf(row[i] * inv * bf2f(w[i]));
}

// ------------------------------------------------------------------ host side

int stack_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launched(cudaLaunchKernelExC(&cfg, fn, args));
}

template <int EPI, int MT>
cudaError_t launch_gemv_t(const GemvArgs& g, int max_ctas, cudaStream_t s) {
  const size_t smem = (size_t)g.T * g.K * 4;
  static SmemGrant granted;
  // past 48 KB of dynamic plus static shared memory (the kernel's few reduction slots) a launch needs the opt-in
  if (smem + 1024 > 48 * 1024) {
    cudaError_t e = grant_smem(reinterpret_cast<const void*>(dense_gemv_kernel<EPI, MT>), smem, 0, granted);
    if (e != cudaSuccess) return e;
  }
  const int ctas = std::max(1, std::min(max_ctas, (g.N + kGemvWarps - 1) / kGemvWarps));  // a row per warp at least
  GemvArgs a = g;
  void* args[] = {&a};
  return launch_pdl(reinterpret_cast<const void*>(dense_gemv_kernel<EPI, MT>), dim3(ctas), dim3(kGemvWarps * 32), smem,
                    s, args);
}

template <int EPI>
cudaError_t launch_gemv(const GemvArgs& g, int max_ctas, cudaStream_t s) {
  return g.T == 1 ? launch_gemv_t<EPI, 1>(g, max_ctas, s) : launch_gemv_t<EPI, kStackMaxT>(g, max_ctas, s);
}

struct AttnWs {
  size_t qkv, z, o, part, err, total;
  int nsplit_max;
};

AttnWs attn_ws(const moe_attn_weights* w, int max_T, int ctx) {
  AttnWs L;
  size_t off = 0;
  const int nq = w->Hq * w->D, nqkv = (w->Hq + 2 * w->Hkv) * w->D;
  L.nsplit_max = (ctx + 15) / 16;
  L.err = off;  off = ws_align(off + 4);  // first, so that its offset does not depend on T or ctx
  L.qkv = off;  off = ws_align(off + (size_t)max_T * nqkv * 2);
  L.z = off;    off = ws_align(off + (w->gate ? (size_t)max_T * nq * 2 : 0));
  L.o = off;    off = ws_align(off + (size_t)max_T * nq * 2);
  L.part = off; off = ws_align(off + (size_t)max_T * w->Hq * L.nsplit_max * part_stride(w->D) * 4);
  L.total = off;
  return L;
}

bool attn_ok(const moe_attn_weights* w) {
  if (!w || !w->qkv || !w->o || !w->q_norm || !w->k_norm) return false;
  if (w->D != 256 || w->H <= 0 || w->H % 256 != 0 || w->H > 8192 || w->Hkv <= 0 || w->Hq <= 0) return false;
  if (w->Hq % w->Hkv != 0 || 8 % (w->Hq / w->Hkv) != 0) return false;
  if (w->rope_dim <= 0 || w->rope_dim > w->D || w->rope_dim % 64 != 0) return false;
  if (w->Hq * w->D > 8192) return false;  // the o GEMV stages Hq D inputs per token in shared memory
  return true;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" {

size_t moe_attn_workspace_bytes(const moe_attn_weights* w, int max_T, int ctx) {
  if (!attn_ok(w) || max_T < 1 || max_T > kStackMaxT || ctx < 1) return 0;
  return attn_ws(w, max_T, ctx).total;
}

int moe_attn_workspace_error(void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  if (!workspace || workspace_bytes < 4 || !al16(workspace)) return -(int)cudaErrorInvalidValue;
  uint32_t* errp = static_cast<uint32_t*>(workspace);  // the error word leads the layout (attn_ws)
  uint32_t v = 0;
  const cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(&v, errp, sizeof v, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(errp, 0, sizeof v, s);
  if (e != cudaSuccess) return -(int)e;
  return (int)v;
}

}  // extern "C"

// The attention branch; its input is normed (bf16) or, when normed is null, hidden (fp32) normalised with rms1
// inside the first GEMV.
static int attn_forward(const moe_attn_weights* w, uint16_t* kc, uint16_t* vc, int ctx, int pos0, const uint16_t* normed,
                        const float* hidden, const uint16_t* rms1, uint16_t* attn_out, int T, void* workspace,
                        size_t workspace_bytes, moe_stream_t stream) {
  if (!attn_ok(w) || !kc || !vc || !(normed || (hidden && rms1)) || !attn_out || !workspace || T < 1 ||
      T > kStackMaxT || pos0 < 0 || ctx < 1 || pos0 + T > ctx)
    return (int)cudaErrorInvalidValue;
  if (!normed && (!al16(hidden) || !al16(rms1))) return (int)cudaErrorInvalidValue;
  const AttnWs L = attn_ws(w, T, ctx);
  if (workspace_bytes < L.total) return (int)cudaErrorInvalidValue;
  if (!al16(kc) || !al16(vc) || !al16(normed) || !al16(workspace) || !al16(w->qkv) || !al16(w->o) ||
      (w->gate && !al16(w->gate)))
    return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* qkv = reinterpret_cast<uint16_t*>(ws + L.qkv);
  uint16_t* z = w->gate ? reinterpret_cast<uint16_t*>(ws + L.z) : nullptr;
  uint16_t* o = reinterpret_cast<uint16_t*>(ws + L.o);
  float* part = reinterpret_cast<float*>(ws + L.part);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws + L.err);
  const int nq = w->Hq * w->D, nqkv = (w->Hq + 2 * w->Hkv) * w->D;
  const int gemv_ctas = stack_sms() * 2;  // two CTAs per SM (the GEMV's launch bounds)
  // 1. qkv (and the gate) = normed . W^T, one launch
  GemvArgs g;
  memset(&g, 0, sizeof g);
  g.x = normed;
  g.xf = hidden;
  g.xw = rms1;
  g.eps = w->eps;
  g.w0 = w->qkv;
  g.w1 = w->gate;
  g.n0 = nqkv;
  g.N = nqkv + (w->gate ? nq : 0);
  g.K = w->H;
  g.T = T;
  g.y0 = qkv;
  g.y1 = z;
  cudaError_t e = launch_gemv<EPI_BF16>(g, gemv_ctas, s);
  if (e != cudaSuccess) return (int)e;
  // 2. per-head norm + RoPE, cache append and split-K attention in one launch: about two CTAs per SM, 16 .. 64
  // keys per split
  {
    const int nkeys = pos0 + T, jobs = T * w->Hkv;
    const int want = (2 * stack_sms() + jobs - 1) / jobs;
    int nsplit = std::max((nkeys + kAttnMaxChunk - 1) / kAttnMaxChunk, std::min(want, (nkeys + 15) / 16));
    nsplit = std::max(1, std::min(nsplit, L.nsplit_max));
    const int chunk = (nkeys + nsplit - 1) / nsplit;  // the longest token's chunk
    const size_t smem = (size_t)2 * chunk * w->D * 2;
    static SmemGrant granted;
    e = grant_smem(reinterpret_cast<const void*>(attn_split_kernel), (size_t)2 * kAttnMaxChunk * 256 * 2, 0, granted);
    if (e != cudaSuccess) return (int)e;
    AttnArgs a;
    a.qkv = qkv;
    a.q_norm = w->q_norm;
    a.k_norm = w->k_norm;
    a.kc = kc;
    a.vc = vc;
    a.part = part;
    a.err = err;
    a.T = T;
    a.Hq = w->Hq;
    a.Hkv = w->Hkv;
    a.ctx = ctx;
    a.pos0 = pos0;
    a.nsplit = nsplit;
    a.rope_dim = w->rope_dim;
    a.scale = 1.f / sqrtf((float)w->D);
    a.theta = w->theta;
    a.eps = w->eps;
    void* args[] = {&a};
    e = launch_pdl(reinterpret_cast<const void*>(attn_split_kernel), dim3(jobs, nsplit), dim3(256), smem, s, args);
    if (e != cudaSuccess) return (int)e;
    const float* pp = part;
    const uint16_t* zz = z;
    int ns = nsplit;
    void* cargs[] = {&pp, &zz, &o, &ns};
    e = launch_pdl(reinterpret_cast<const void*>(attn_combine_kernel), dim3(T * w->Hq * 8), dim3(256), 0, s, cargs);
    if (e != cudaSuccess) return (int)e;
  }
  // 3. attn_out = o . Wo^T
  memset(&g, 0, sizeof g);
  g.x = o;
  g.w0 = w->o;
  g.n0 = w->H;
  g.N = w->H;
  g.K = nq;
  g.T = T;
  g.y0 = attn_out;
  return (int)launch_gemv<EPI_BF16>(g, gemv_ctas, s);
}

extern "C" {

int moe_attn_forward(const moe_attn_weights* w, uint16_t* kc, uint16_t* vc, int ctx, int pos0, const uint16_t* normed,
                     uint16_t* attn_out, int T, void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  if (!normed) return (int)cudaErrorInvalidValue;
  return attn_forward(w, kc, vc, ctx, pos0, normed, nullptr, nullptr, attn_out, T, workspace, workspace_bytes, stream);
}

int moe_attn_forward_rms(const moe_attn_weights* w, const uint16_t* rms1, const float* hidden, uint16_t* kc,
                         uint16_t* vc, int ctx, int pos0, uint16_t* attn_out, int T, void* workspace,
                         size_t workspace_bytes, moe_stream_t stream) {
  if (!rms1 || !hidden) return (int)cudaErrorInvalidValue;
  return attn_forward(w, kc, vc, ctx, pos0, nullptr, hidden, rms1, attn_out, T, workspace, workspace_bytes, stream);
}

int moe_rmsnorm(const float* x, const uint16_t* w, uint16_t* y, int T, int H, float eps, moe_stream_t stream) {
  if (!x || !w || !y || T < 1 || H < 1) return (int)cudaErrorInvalidValue;
  void* args[] = {&x, &w, &y, &H, &eps};
  return (int)launch_pdl(reinterpret_cast<const void*>(rmsnorm_rows_kernel), dim3(T), dim3(256), 0,
                         (cudaStream_t)stream, args);
}

size_t moe_lm_head_workspace_bytes(int V, int H) {
  if (V < 1 || H < 8 || H % 8 != 0 || H > 8192) return 0;
  return 256 + (size_t)kArgmaxMaxCtas * 8;
}

int moe_lm_head_argmax(const uint16_t* normed, const uint16_t* lm_head, int V, int H, float* logits, int32_t* next,
                       void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  if (!normed || !lm_head || !next || !workspace || V < 1 || H < 8 || H % 8 != 0 || H > 8192 ||
      workspace_bytes < moe_lm_head_workspace_bytes(V, H) || !al16(normed) || !al16(lm_head))
    return (int)cudaErrorInvalidValue;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  GemvArgs g;
  memset(&g, 0, sizeof g);
  g.x = normed;
  g.w0 = lm_head;
  g.n0 = V;
  g.N = V;
  g.K = H;
  g.T = 1;
  g.logits = logits;
  g.ticket = reinterpret_cast<uint32_t*>(ws);
  g.pv = reinterpret_cast<float*>(ws + 256);
  g.pi = reinterpret_cast<int32_t*>(ws + 256 + (size_t)kArgmaxMaxCtas * 4);
  g.next = next;
  return (int)launch_gemv<EPI_ARGMAX>(g, std::min(kArgmaxMaxCtas, stack_sms() * 2), (cudaStream_t)stream);
}

}  // extern "C"
