// moe_stack.cu -- the attention layer and the LM head of a decode step (include/moe_stack.h): the reference's
// attention branch of forward() (qwen.cu:413-425) and its LM head (qwen.cu:451-456), rebuilt for B200.
//
// Every piece streams weights or cache rows from HBM once, so each kernel is sized for memory-level parallelism:
//   dense_gemv_kernel   y = x . W^T for T <= 4 tokens (qkv, gate, o, LM head): one warp per pair of rows, 16-byte
//                       loads, 2 x 4 KB in flight per warp, x staged in shared memory in a bank-conflict-free
//                       order. The first rows' weights are requested before griddepcontrol.wait, so under
//                       programmatic dependent launch they stream while the previous kernel finishes. The LM-head
//                       variant keeps each warp's best (logit, index) and the last CTA to finish (a ticket)
//                       reduces the CTAs' results: argmax fused into the GEMV, one launch.
//   qk_norm_rope_kernel per (token, head) warp: RMSNorm of the q and k heads, rotate-half RoPE, the new k and v rows
//                       into the caches (attn_qk_norm_rope_kernel, kernels.cuh:608-663).
//   attn_split_kernel   split-K decode attention (kernels.cuh:665-761): CTA (token, kv head, split) copies its chunk
//                       of K and V rows into shared memory with two bulk copies, and warp g scores the chunk for
//                       query head g: 32 keys' partial dot products per lane, one 31-shuffle reduce-scatter that
//                       leaves key j's score in lane j, online softmax, acc += p v. Partials (acc, max, sum) per
//                       split.
//   attn_combine_kernel merges the splits (and applies the optional sigmoid gate, kernels.cuh:765-769).
#include <algorithm>
#include <cstring>

#include "../../include/moe_stack.h"
#include "moe_common.cuh"
#include "moe_device.cuh"
#include "moe_sync.cuh"

namespace moe {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvRows = 2;       // rows per warp per iteration
constexpr int kGemvU = 4;          // 16-byte loads per lane per row per iteration
constexpr int kStackMaxT = 4;
constexpr int kAttnMaxChunk = 64;  // keys per split (shared memory: 2 x 64 x 512 B)
constexpr int kArgmaxMaxCtas = 1024;
// Floats per split-K partial: acc [D], max, sum, padded to a multiple of 4 so that every partial starts on a 16-byte
// boundary (its acc is stored as float4).
__host__ __device__ constexpr int part_stride(int D) { return D + 4; }

enum { EPI_BF16 = 0, EPI_ARGMAX = 1 };

struct GemvArgs {
  const uint16_t* x;   // bf16 [T][K]
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

template <int EPI>
__global__ void __launch_bounds__(kGemvWarps * 32) dense_gemv_kernel(const __grid_constant__ GemvArgs g) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float bv_s[kGemvWarps];
  __shared__ int bi_s[kGemvWarps];
  __shared__ int is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = g.K, N = g.N, T = g.T, nu = K >> 3;
  const int stride = gridDim.x * kGemvWarps * kGemvRows;
  int r0 = (blockIdx.x * kGemvWarps + warp) * kGemvRows;
  // the first rows' weights do not depend on the previous kernel: request them before waiting for it
  uint4 wv[kGemvRows][kGemvU];
  auto row_ptr = [&](int r) -> const uint4* {
    const uint16_t* base = r < g.n0 ? g.w0 + (int64_t)r * K : g.w1 + (int64_t)(r - g.n0) * K;
    return reinterpret_cast<const uint4*>(base);
  };
  auto load = [&](int r, int it) {
#pragma unroll
    for (int q = 0; q < kGemvRows; ++q) {
      const int rr = r + q;
      const uint4* p = rr < N ? row_ptr(rr) : nullptr;
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) {
        const int i = it * (32 * kGemvU) + u * 32 + lane;
        wv[q][u] = (p && i < nu) ? ldg_stream(p + i) : make_uint4(0, 0, 0, 0);
      }
    }
  };
  if (r0 < N) load(r0, 0);
  pdl_wait();
  pdl_launch_dependents();
  // x -> shared memory (fp32, permuted)
  for (int e = threadIdx.x; e < T * nu; e += blockDim.x) {
    const int t = e / nu, i = e - t * nu;
    const uint4 v = reinterpret_cast<const uint4*>(g.x + (int64_t)t * K)[i];
    float* dst = xs + t * K;
    *reinterpret_cast<float4*>(dst + xs_pos(i, 0, nu)) = make_float4(lo_bf(v.x), hi_bf(v.x), lo_bf(v.y), hi_bf(v.y));
    *reinterpret_cast<float4*>(dst + xs_pos(i, 1, nu)) = make_float4(lo_bf(v.z), hi_bf(v.z), lo_bf(v.w), hi_bf(v.w));
  }
  __syncthreads();
  float best_v = -1e30f;
  int best_i = 0;
  const int iters = (nu + 32 * kGemvU - 1) / (32 * kGemvU);
  for (; r0 < N; r0 += stride) {
    float acc[kGemvRows][kStackMaxT];
#pragma unroll
    for (int q = 0; q < kGemvRows; ++q)
#pragma unroll
      for (int t = 0; t < kStackMaxT; ++t) acc[q][t] = 0.f;
    for (int it = 0; it < iters; ++it) {
      if (it > 0) load(r0, it);
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) {
        const int i = it * (32 * kGemvU) + u * 32 + lane;
        if (i >= nu) break;
#pragma unroll
        for (int t = 0; t < kStackMaxT; ++t) {
          if (t >= T) break;
          const float4 x0 = *reinterpret_cast<const float4*>(xs + t * K + xs_pos(i, 0, nu));
          const float4 x1 = *reinterpret_cast<const float4*>(xs + t * K + xs_pos(i, 1, nu));
#pragma unroll
          for (int q = 0; q < kGemvRows; ++q) {
            const uint4 w = wv[q][u];
            float a = acc[q][t];
            a = fmaf(lo_bf(w.x), x0.x, a);
            a = fmaf(hi_bf(w.x), x0.y, a);
            a = fmaf(lo_bf(w.y), x0.z, a);
            a = fmaf(hi_bf(w.y), x0.w, a);
            a = fmaf(lo_bf(w.z), x1.x, a);
            a = fmaf(hi_bf(w.z), x1.y, a);
            a = fmaf(lo_bf(w.w), x1.z, a);
            a = fmaf(hi_bf(w.w), x1.w, a);
            acc[q][t] = a;
          }
        }
      }
    }
    // the next rows' first weights before this pair's reductions
    const int r_next = r0 + stride;
#pragma unroll
    for (int q = 0; q < kGemvRows; ++q)
#pragma unroll
      for (int t = 0; t < kStackMaxT; ++t) acc[q][t] = warp_sum(acc[q][t]);
    if (r_next < N) load(r_next, 0);
#pragma unroll
    for (int q = 0; q < kGemvRows; ++q) {
      const int r = r0 + q;
      if (r >= N) break;
      if (EPI == EPI_BF16) {
        if (lane < T) {
          float v = acc[q][0];
#pragma unroll
          for (int t = 1; t < kStackMaxT; ++t)
            if (lane == t) v = acc[q][t];
          if (r < g.n0) g.y0[(int64_t)lane * g.n0 + r] = f2bf(v);
          else g.y1[(int64_t)lane * (N - g.n0) + (r - g.n0)] = f2bf(v);
        }
      } else {
        const float v = acc[q][0];
        if (lane == 0 && g.logits) g.logits[r] = v;
        if (better(v, r, best_v, best_i)) {
          best_v = v;
          best_i = r;
        }
      }
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

// Per (token, head) warp: RMSNorm + rotate-half RoPE of q and k heads; k and v rows into the caches at pos0 + t.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const uint16_t* __restrict__ qkv,
                                                           const uint16_t* __restrict__ q_norm,
                                                           const uint16_t* __restrict__ k_norm, uint16_t* __restrict__ q,
                                                           uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int T,
                                                           int Hq, int Hkv, int D, int rope_dim, float theta, int pos0,
                                                           int ctx, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int job = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int heads = Hq + 2 * Hkv;
  if (job >= T * heads) return;
  const int t = job / heads, hh = job - t * heads;
  const uint16_t* src = qkv + ((int64_t)t * heads + hh) * D;
  const int pos = pos0 + t;
  if (hh >= Hq + Hkv) {  // v rows are copied unchanged
    uint16_t* dst = vc + ((int64_t)(hh - Hq - Hkv) * ctx + pos) * D;
    for (int d = lane; d < D; d += 32) dst[d] = src[d];
    return;
  }
  const bool is_q = hh < Hq;
  const uint16_t* w = is_q ? q_norm : k_norm;
  uint16_t* dst = is_q ? q + ((int64_t)t * Hq + hh) * D : kc + ((int64_t)(hh - Hq) * ctx + pos) * D;
  float v[8];  // D == 256: lane holds d = lane + 32 i
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = bf2f(src[lane + 32 * i]);
    ss = fmaf(v[i], v[i], ss);
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = v[i] * inv * bf2f(w[lane + 32 * i]);
  // pairs (d, d + rope_dim / 2) for d < rope_dim / 2; rope_dim / 2 is a multiple of 32, so both lie in this lane
  const int half = rope_dim >> 1, hs = half >> 5;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < half) {
      const float inv_freq = powf(theta, -(float)(2 * d) / (float)rope_dim);
      float s, c;
      sincosf((float)pos * inv_freq, &s, &c);
      float b = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j == i + hs) b = v[j];
      const float a = v[i];
      v[i] = a * c - b * s;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j == i + hs) v[j] = b * c + a * s;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[lane + 32 * i] = f2bf(v[i]);
}

// Split-K decode attention, GQA: CTA (job = t * Hkv + kv head, split sp), warp g < G handles query head
// kvh * G + g over keys [k0, k1) of the split. D == 256: lane owns dims 8 lane .. 8 lane + 7.
struct AttnArgs {
  const uint16_t* q;
  const uint16_t* kc;
  const uint16_t* vc;
  float* part;  // [(t * Hq + h) * nsplit + sp][part_stride(D)]: acc, max, sum
  uint32_t* err;
  int T, Hq, Hkv, ctx, pos0, nsplit;
  float scale;
};

__global__ void __launch_bounds__(256) attn_split_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int D = 256;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t kvbar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int job = blockIdx.x, sp = blockIdx.y;
  const int t = job / a.Hkv, kvh = job - t * a.Hkv;
  const int G = a.Hq / a.Hkv;
  const int nkeys = a.pos0 + t + 1;
  const int chunk = (nkeys + a.nsplit - 1) / a.nsplit;
  const int k0 = min(nkeys, sp * chunk), k1 = min(nkeys, k0 + chunk), n = k1 - k0;
  uint8_t* ks = smem;
  uint8_t* vs = smem + kAttnMaxChunk * D * 2;
  if (threadIdx.x == 0) {
    mbar_init(&kvbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    expect_tx(&kvbar, (uint32_t)(2 * n * D * 2));
    if (n > 0) {
      bulk_g2s(ks, a.kc + ((int64_t)kvh * a.ctx + k0) * D, n * D * 2, &kvbar);
      bulk_g2s(vs, a.vc + ((int64_t)kvh * a.ctx + k0) * D, n * D * 2, &kvbar);
    }
  }
  const bool ok = bar_wait(&kvbar, 0);
  if (!ok && threadIdx.x == 0) atomicOr(a.err, (uint32_t)MOE_ERR_TIMEOUT);
  if (warp >= G) return;
  const int h = kvh * G + warp;
  float qf[8];
  {
    const uint4 qv = reinterpret_cast<const uint4*>(a.q + ((int64_t)t * a.Hq + h) * D)[lane];
    qf[0] = lo_bf(qv.x); qf[1] = hi_bf(qv.x); qf[2] = lo_bf(qv.y); qf[3] = hi_bf(qv.y);
    qf[4] = lo_bf(qv.z); qf[5] = hi_bf(qv.z); qf[6] = lo_bf(qv.w); qf[7] = hi_bf(qv.w);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] *= a.scale;
  }
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

// Merge of the nsplit partials of each (token, query head): CTA (job, quarter) handles dims [64 quarter, +64) with
// 4 groups of 64 threads over the splits, merged in shared memory; o = bf16(acc / sum), then optionally
// o = bf16(o * sigmoid(gate)).
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ part, const uint16_t* __restrict__ z,
                                                           uint16_t* __restrict__ o, int nsplit) {
  constexpr int D = 256;
  __shared__ float acc_s[4][64], l_s[4];
  pdl_wait();
  pdl_launch_dependents();
  const int job = blockIdx.x >> 2, quarter = blockIdx.x & 3;
  const int grp = threadIdx.x >> 6, d = quarter * 64 + (threadIdx.x & 63);
  constexpr int PS = part_stride(D);
  const float* src = part + (int64_t)job * nsplit * PS;
  // global max over all splits (every thread computes it; the reads are broadcasts)
  float gm = -1e30f;
  for (int s = 0; s < nsplit; ++s) gm = fmaxf(gm, __ldcg(src + s * PS + D));
  float acc = 0.f, gl = 0.f;
  for (int s = grp; s < nsplit; s += 4) {
    const float* p = src + s * PS;
    const float pl = __ldcg(p + D + 1);
    const float c = pl > 0.f ? __expf(__ldcg(p + D) - gm) : 0.f;
    gl += pl * c;
    acc = fmaf(__ldcg(p + d), c, acc);
  }
  acc_s[grp][threadIdx.x & 63] = acc;
  if ((threadIdx.x & 63) == 0) l_s[grp] = gl;
  __syncthreads();
  if (grp != 0) return;
  const float tot = acc_s[0][threadIdx.x] + acc_s[1][threadIdx.x] + acc_s[2][threadIdx.x] + acc_s[3][threadIdx.x];
  const float lsum = l_s[0] + l_s[1] + l_s[2] + l_s[3];
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

template <int EPI>
cudaError_t launch_gemv(const GemvArgs& g, int max_ctas, cudaStream_t s) {
  const size_t smem = (size_t)g.T * g.K * 4;
  static size_t granted = 0;
  if (smem > 48 * 1024 && smem > granted) {
    cudaError_t e = cudaFuncSetAttribute(dense_gemv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    granted = smem;
  }
  const int per_cta = kGemvWarps * kGemvRows;
  const int ctas = std::max(1, std::min(max_ctas, (g.N + per_cta - 1) / per_cta));
  GemvArgs a = g;
  void* args[] = {&a};
  return launch_pdl(reinterpret_cast<const void*>(dense_gemv_kernel<EPI>), dim3(ctas), dim3(kGemvWarps * 32), smem,
                    s, args);
}

struct AttnWs {
  size_t qkv, z, q, o, part, err, total;
  int nsplit_max;
};

AttnWs attn_ws(const moe_attn_weights* w, int max_T, int ctx) {
  AttnWs L;
  size_t off = 0;
  const int nq = w->Hq * w->D, nqkv = (w->Hq + 2 * w->Hkv) * w->D;
  L.nsplit_max = (ctx + 15) / 16;
  L.qkv = off;  off = ws_align(off + (size_t)max_T * nqkv * 2);
  L.z = off;    off = ws_align(off + (w->gate ? (size_t)max_T * nq * 2 : 0));
  L.q = off;    off = ws_align(off + (size_t)max_T * nq * 2);
  L.o = off;    off = ws_align(off + (size_t)max_T * nq * 2);
  L.part = off; off = ws_align(off + (size_t)max_T * w->Hq * L.nsplit_max * part_stride(w->D) * 4);
  L.err = off;  off = ws_align(off + 4);
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

int moe_attn_forward(const moe_attn_weights* w, uint16_t* kc, uint16_t* vc, int ctx, int pos0, const uint16_t* normed,
                     uint16_t* attn_out, int T, void* workspace, size_t workspace_bytes, moe_stream_t stream) {
  if (!attn_ok(w) || !kc || !vc || !normed || !attn_out || !workspace || T < 1 || T > kStackMaxT || pos0 < 0 ||
      ctx < 1 || pos0 + T > ctx)
    return (int)cudaErrorInvalidValue;
  const AttnWs L = attn_ws(w, T, ctx);
  if (workspace_bytes < L.total) return (int)cudaErrorInvalidValue;
  if (!al16(kc) || !al16(vc) || !al16(normed) || !al16(workspace) || !al16(w->qkv) || !al16(w->o) ||
      (w->gate && !al16(w->gate)))
    return (int)cudaErrorInvalidValue;
  const cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* qkv = reinterpret_cast<uint16_t*>(ws + L.qkv);
  uint16_t* z = w->gate ? reinterpret_cast<uint16_t*>(ws + L.z) : nullptr;
  uint16_t* q = reinterpret_cast<uint16_t*>(ws + L.q);
  uint16_t* o = reinterpret_cast<uint16_t*>(ws + L.o);
  float* part = reinterpret_cast<float*>(ws + L.part);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws + L.err);
  const int nq = w->Hq * w->D, nqkv = (w->Hq + 2 * w->Hkv) * w->D;
  const int gemv_ctas = stack_sms() * 3;
  // 1. qkv (and the gate) = normed . W^T, one launch
  GemvArgs g;
  memset(&g, 0, sizeof g);
  g.x = normed;
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
  // 2. per-head norm + RoPE, cache append
  {
    const uint16_t* a0 = qkv;
    const uint16_t* a1 = w->q_norm;
    const uint16_t* a2 = w->k_norm;
    int Hq = w->Hq, Hkv = w->Hkv, D = w->D, rd = w->rope_dim, p0 = pos0, cx = ctx, TT = T;
    float th = w->theta, eps = w->eps;
    void* args[] = {&a0, &a1, &a2, &q, &kc, &vc, &TT, &Hq, &Hkv, &D, &rd, &th, &p0, &cx, &eps};
    const int jobs = T * (w->Hq + 2 * w->Hkv);
    e = launch_pdl(reinterpret_cast<const void*>(qk_norm_rope_kernel), dim3((jobs + 7) / 8), dim3(256), 0, s, args);
    if (e != cudaSuccess) return (int)e;
  }
  // 3. split-K attention: about one wave of CTAs, 16 .. 64 keys per split
  {
    const int nkeys = pos0 + T, jobs = T * w->Hkv;
    const int want = (stack_sms() + jobs - 1) / jobs;
    int nsplit = std::max((nkeys + kAttnMaxChunk - 1) / kAttnMaxChunk, std::min(want, (nkeys + 15) / 16));
    nsplit = std::max(1, std::min(nsplit, L.nsplit_max));
    const size_t smem = (size_t)2 * kAttnMaxChunk * w->D * 2;
    static bool granted = false;
    if (!granted) {
      e = cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
      granted = true;
    }
    AttnArgs a;
    a.q = q;
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
    a.scale = 1.f / sqrtf((float)w->D);
    void* args[] = {&a};
    e = launch_pdl(reinterpret_cast<const void*>(attn_split_kernel), dim3(jobs, nsplit), dim3(256), smem, s, args);
    if (e != cudaSuccess) return (int)e;
    const float* pp = part;
    const uint16_t* zz = z;
    int ns = nsplit;
    void* cargs[] = {&pp, &zz, &o, &ns};
    e = launch_pdl(reinterpret_cast<const void*>(attn_combine_kernel), dim3(T * w->Hq * 4), dim3(256), 0, s, cargs);
    if (e != cudaSuccess) return (int)e;
  }
  // 4. attn_out = o . Wo^T
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
  return (int)launch_gemv<EPI_ARGMAX>(g, std::min(kArgmaxMaxCtas, stack_sms() * 4), (cudaStream_t)stream);
}

}  // extern "C"
