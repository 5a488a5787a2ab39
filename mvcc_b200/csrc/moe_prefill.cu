// moe_prefill.cu -- the MoE block for T >= 8 tokens: the reference's sort + tile path of moe() (qwen.cu:345-363,
// kernels.cuh:904-1069) together with the router and shared expert through dense() (qwen.cu:298-319), all GEMMs on
// the tcgen05 tile GEMM of moe_gemm.cu.
//
// Launch sequence of prefill_block (one stream):
//   memset      per-expert pair bitmaps
//   norm        residual RMSNorm (residual_rmsnorm_kernel, kernels.cuh:98-114) and the shared-expert gate logit
//   router      GEMM normed . router^T -> fp32 logits
//   topk        the reference's top-k rule per token (router_topk_kernel, kernels.cuh:774-809); marks bit p of
//               expert e's bitmap for every pair p = t * TOPK + slot
//   scan        per expert: popcounts and word prefixes of its bitmap; the last CTA turns the counts into the
//               expert offsets and the grouped-GEMM tile lists (kTileRows = 128 pairs per tile, and double tiles
//               of 256 pairs)
//   scatter     pair p of expert e goes to offsets[e] + (pairs of e before p): a stable counting sort by pair
//               index, bit-exact and deterministic (moe_sort_kernel, kernels.cuh:906-923, orders ties arbitrarily)
//   gate_up     grouped INT4 GEMM, A rows gathered per sorted pair, epilogue bf16(silu(g) * u) -> inter (sorted)
//   down        grouped INT4 GEMM over inter, epilogue acc * w[pair] -> slot partials (per pair, unsorted)
//   shared      two bf16 GEMMs: gate/up with epilogue bf16(silu(bf16 g) * bf16 u), down -> bf16 sout
//   combine     per token: routed = slot partials summed in slot order (moe_slot_reduce_kernel,
//               kernels.cuh:1059-1069), hidden += routed + sigmoid gate * sout (shared_gate_combine[_rmsnorm],
//               kernels.cuh:1081-1121), optional next-layer RMSNorm.
// Numerics are the reference's tile numerics: fp32 accumulation of bf16 activations times bf16-dequantized INT4
// weights, bf16 inter, fp32 per-slot partials reduced in slot order.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "moe_device.cuh"
#include "moe_gemm.h"
#include "moe_prefill.h"

namespace moe {

constexpr int kPT = 256;  // threads of the small prefill kernels

// ---- residual RMSNorm + shared-gate logit, one CTA per token
__global__ void __launch_bounds__(kPT) prefill_norm_kernel(const BlockArgs a) {
  __shared__ float red[32];
  const int t = blockIdx.x, tid = threadIdx.x, H = a.w.H;
  const float4* hr = reinterpret_cast<const float4*>(a.hidden + (int64_t)t * H);
  const uint2* dr = reinterpret_cast<const uint2*>(a.attn_out + (int64_t)t * H);
  float4 hv[4];
  float ss = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {  // H <= 4096 = 4 x 256 threads x 4
    const int i = tid + r * kPT;
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
  float gd = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tid + r * kPT;
    if (i < H / 4) {
      const uint2 wr = reinterpret_cast<const uint2*>(a.w.rms2)[i];
      const uint2 gw = reinterpret_cast<const uint2*>(a.w.shared_gate)[i];
      const uint32_t y0 = f2bf(hv[r].x * inv * lo_bf(wr.x)), y1 = f2bf(hv[r].y * inv * hi_bf(wr.x));
      const uint32_t y2 = f2bf(hv[r].z * inv * lo_bf(wr.y)), y3 = f2bf(hv[r].w * inv * hi_bf(wr.y));
      reinterpret_cast<uint2*>(a.normed + (int64_t)t * H)[i] = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
      gd = fmaf(bf2f(y0), lo_bf(gw.x), gd);
      gd = fmaf(bf2f(y1), hi_bf(gw.x), gd);
      gd = fmaf(bf2f(y2), lo_bf(gw.y), gd);
      gd = fmaf(bf2f(y3), hi_bf(gw.y), gd);
    }
  }
  gd = block_sum(gd, red);
  if (tid == 0) a.gate[t] = sigmoid(gd);
}

// ---- top-k per token (one warp each) + pair bitmaps
__global__ void __launch_bounds__(kPT) prefill_topk_kernel(const BlockArgs a, int mark) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (kPT / 32) + warp;
  if (t >= a.T) return;
  const int E = a.w.E, K = a.w.TOPK;
  topk_warp(a.logits + (int64_t)t * E, E, K, a.idx + (int64_t)t * K, a.wts + (int64_t)t * K);
  if (mark && lane < K) {
    const int p = t * K + lane;
    const int e = clampi(a.idx[p], 0, E - 1);  // this lane's own write
    atomicOr(a.bits + (int64_t)e * a.nwp + (p >> 5), 1u << (p & 31));
  }
}

// ---- pair bitmaps from caller routing (moe_routed_experts); invalid indices are flagged and dropped
__global__ void __launch_bounds__(kPT) prefill_mark_kernel(const BlockArgs a) {
  const int P = a.T * a.w.TOPK;
  const int p = blockIdx.x * kPT + threadIdx.x;
  if (p >= P) return;
  const int e = a.idx[p];
  if (e < 0 || e >= a.w.E) {
    atomicOr(a.err, (uint32_t)MOE_ERR_EXPERT_INDEX);
    return;
  }
  atomicOr(a.bits + (int64_t)e * a.nwp + (p >> 5), 1u << (p & 31));
}

// ---- per-expert counts and word prefixes (CTA e); the last CTA builds offsets and the tile list
__global__ void __launch_bounds__(kPT) prefill_scan_kernel(const BlockArgs a) {
  __shared__ int sm[32];
  __shared__ int is_last;
  const int e = blockIdx.x, tid = threadIdx.x, E = a.w.E, nwp = a.nwp;
  const uint32_t* bits = a.bits + (int64_t)e * nwp;
  uint32_t* wpre = a.wpre + (int64_t)e * nwp;
  const int per = (nwp + kPT - 1) / kPT, w0 = min(nwp, tid * per), w1 = min(nwp, w0 + per);
  int c = 0;
  for (int w = w0; w < w1; ++w) c += __popc(__ldcg(bits + w));
  int total;
  int run = block_excl_scan(c, sm, &total);
  for (int w = w0; w < w1; ++w) {
    wpre[w] = run;
    run += __popc(__ldcg(bits + w));
  }
  if (tid == 0) a.counts[e] = total;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    is_last = atomicInc(&a.ticket[TICKET_SCAN], gridDim.x - 1) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // offsets and tiles over E <= 256 experts: one expert per thread
  const int cnt = tid < E ? __ldcg(a.counts + tid) : 0;
  int npairs;
  const int off = block_excl_scan(cnt, sm, &npairs);
  if (tid < E) a.offsets[tid] = off;
  if (tid == 0) a.offsets[E] = npairs;
  // the tile list (kTileRows rows) and the double-tile list (2 kTileRows rows) over the same sorted pairs
#pragma unroll 1
  for (int li = 0; li < 2; ++li) {
    const int rows = kTileRows << li, cap = li ? a.max_tiles2 : a.max_tiles;
    GemmTile* tiles = static_cast<GemmTile*>(li ? a.tiles2 : a.tiles);
    const int nt = (cnt + rows - 1) / rows;
    int ntiles;
    const int tbase = block_excl_scan(nt, sm, &ntiles);
    if (tid < E) {
      for (int j = 0; j < nt && tbase + j < cap; ++j) {
        GemmTile g;
        g.e = tid;
        g.m0 = off + rows * j;
        g.mcount = min(rows, cnt - rows * j);
        g.pad = 0;
        tiles[tbase + j] = g;
      }
    }
    if (tid == 0) *(li ? a.ntiles2 : a.ntiles) = min(ntiles, cap);
  }
}

// ---- stable scatter: sorted[offsets[e] + rank of p among e's pairs] = p
__global__ void __launch_bounds__(kPT) prefill_scatter_kernel(const BlockArgs a) {
  const int P = a.T * a.w.TOPK;
  const int p = blockIdx.x * kPT + threadIdx.x;
  if (p >= P) return;
  const int e = a.idx[p];
  if (e < 0 || e >= a.w.E) return;
  const int64_t w = (int64_t)e * a.nwp + (p >> 5);
  const uint32_t below = a.bits[w] & ((1u << (p & 31)) - 1u);
  const int pos = a.offsets[e] + (int)a.wpre[w] + __popc(below);
  if (pos >= 0 && pos < P) a.sorted[pos] = p;
}

// ---- inter rows back from expert-sorted order to pair order (16 bytes per thread)
__global__ void __launch_bounds__(kPT) prefill_unsort_kernel(const BlockArgs a, uint16_t* out) {
  const int P = a.T * a.w.TOPK, cpr = a.w.I / 8;
  const int64_t i = (int64_t)blockIdx.x * kPT + threadIdx.x;
  if (i >= (int64_t)P * cpr) return;
  const int pos = (int)(i / cpr), c = (int)(i - (int64_t)pos * cpr);
  if (pos >= a.offsets[a.w.E]) return;  // positions past the placed pairs (invalid indices dropped)
  const int p = a.sorted[pos];
  if (p < 0 || p >= P) return;
  reinterpret_cast<uint4*>(out + (int64_t)p * a.w.I)[c] = reinterpret_cast<const uint4*>(a.inter + (int64_t)pos * a.w.I)[c];
}

// ---- slot-order reduction and gated residual combine, one CTA per token.
// mode: 1 = write routed (fp32, or bf16 into a.routed16 when set), 2 = combine into hidden (+ next-layer RMSNorm when
// a.next_rms1 is set). The routed sum is over the token's slots with a valid expert, in slot order, or, on the
// expert-parallel source side (a.ep_pos set), over the bf16 partial rows the ranks returned, in rank order.
__global__ void __launch_bounds__(kPT) prefill_combine_kernel(const BlockArgs a, int mode) {
  __shared__ float red[32];
  const int t = blockIdx.x, tid = threadIdx.x, H = a.w.H, K = a.w.TOPK;
  const bool ep = a.ep_pos != nullptr;
  int ok[8];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    ok[k] = ep ? (k < a.ep_world ? a.ep_pos[(int64_t)t * a.ep_world + k] : -1)
               : (k < K && (unsigned)a.idx[(int64_t)t * K + k] < (unsigned)a.w.E);
  const float g = (mode & 2) ? a.gate[t] : 0.f;
  const bool nn = (mode & 2) && a.next_rms1;
  float4 hv[4];
  float ss = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tid + r * kPT;
    if (i >= H / 4) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (ep ? ok[k] < 0 : !ok[k]) continue;
      float4 v;
      if (ep) {
        const uint2 u = __ldcs(reinterpret_cast<const uint2*>(a.ep_ret + (int64_t)ok[k] * H) + i);
        v = make_float4(lo_bf(u.x), hi_bf(u.x), lo_bf(u.y), hi_bf(u.y));
      } else {
        v = __ldcs(reinterpret_cast<const float4*>(a.slot + ((int64_t)t * K + k) * H) + i);
      }
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    if ((mode & 1) && a.routed16)
      reinterpret_cast<uint2*>(a.routed16 + (int64_t)t * H)[i] =
          make_uint2((uint32_t)f2bf(acc.x) | ((uint32_t)f2bf(acc.y) << 16),
                     (uint32_t)f2bf(acc.z) | ((uint32_t)f2bf(acc.w) << 16));
    else if (mode & 1)
      reinterpret_cast<float4*>(a.routed + (int64_t)t * H)[i] = acc;
    if (mode & 2) {
      const float4 h = reinterpret_cast<const float4*>(a.hidden + (int64_t)t * H)[i];
      const uint2 d = reinterpret_cast<const uint2*>(a.attn_out + (int64_t)t * H)[i];
      const uint2 so = reinterpret_cast<const uint2*>(a.sout + (int64_t)t * H)[i];
      const float hh[4] = {h.x + lo_bf(d.x), h.y + hi_bf(d.x), h.z + lo_bf(d.y), h.w + hi_bf(d.y)};
      const float sv[4] = {lo_bf(so.x), hi_bf(so.x), lo_bf(so.y), hi_bf(so.y)};
      const float rv[4] = {acc.x, acc.y, acc.z, acc.w};
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = nn ? fmaf(g, sv[j], hh[j] + rv[j]) : hh[j] + fmaf(g, sv[j], rv[j]);
      hv[r] = make_float4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<float4*>(a.hidden + (int64_t)t * H)[i] = hv[r];
      ss += o[0] * o[0];
      ss += o[1] * o[1];
      ss += o[2] * o[2];
      ss += o[3] * o[3];
    }
  }
  if (!nn) return;
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)H + a.w.eps);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = tid + r * kPT;
    if (i >= H / 4) continue;
    const uint2 wr = reinterpret_cast<const uint2*>(a.next_rms1)[i];
    const uint32_t y0 = f2bf(hv[r].x * inv * lo_bf(wr.x)), y1 = f2bf(hv[r].y * inv * hi_bf(wr.x));
    const uint32_t y2 = f2bf(hv[r].z * inv * lo_bf(wr.y)), y3 = f2bf(hv[r].w * inv * hi_bf(wr.y));
    reinterpret_cast<uint2*>(a.normed + (int64_t)t * H)[i] = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
  }
}

// ------------------------------------------------------------------ host side

bool prefill_supported(const moe_layer_weights& w) { return w.E % 16 == 0; }

// 256 B rows per tile: the most MMA work per pipeline step for the issuing thread's fixed barrier cost (at double
// tiles, 128 rows would leave TMEM room for a second accumulator buffer, but measured slower: 428 against 336 us for
// config 4's gate/up GEMM).
static cudaError_t launch_wide(const GemmParams& p, int epi, bool int4, int tile_rows, int max_tiles, cudaStream_t s) {
  return launch_gemm(p, epi, 256, tile_rows, int4, max_tiles, false, s);
}

// Rows per tile of the routed gate/up and down GEMMs: double tiles (2 kTileRows: two 128-row sub-tiles per
// dequantised B stage) for gate/up, kTileRows for down (its 8 k-steps per item are short beside its epilogue, which
// with single tiles overlaps the next item: 13 us less per config-4 step than double tiles), unless the environment
// sets MOE_B200_GEMM_TILE_ROWS to 128 or 256 (both GEMMs) or to "G,D" with G, D in {128, 256} (read once per
// process).
static void expert_tile_rows(int* gu, int* dn) {
  static int v[2] = {0, 0};
  if (!v[0]) {
    int r[2] = {2 * kTileRows, kTileRows};
    if (const char* e = getenv("MOE_B200_GEMM_TILE_ROWS")) {
      int x = 0, y = 0;
      const int n = sscanf(e, "%d,%d", &x, &y);
      if (n >= 1 && (x == kTileRows || x == 2 * kTileRows)) r[0] = r[1] = x;
      if (n == 2 && (y == kTileRows || y == 2 * kTileRows)) r[1] = y;
    }
    v[1] = r[1];
    v[0] = r[0];
  }
  *gu = v[0];
  *dn = v[1];
}

static GemmParams base_params(const BlockArgs& a) {
  GemmParams p;
  memset(&p, 0, sizeof p);
  p.G = a.w.G;
  p.E = 1;
  p.err = a.err;
  return p;
}

static cudaError_t run_router(const BlockArgs& a, cudaStream_t s) {
  GemmParams p = base_params(a);
  p.A = a.normed;
  p.lda = a.w.H;
  p.a_nrows = a.T;
  p.Bh = a.w.router;
  p.b_rows_per_e = 0;
  p.N = (a.w.E + 127) / 128 * 128;
  p.n_valid = a.w.E;
  p.K = a.w.H;
  p.M = a.T;
  p.out = a.logits;
  p.col_bias = a.w.router_bias;
  p.ldo = a.w.E;
  p.out_nrows = a.T;
  return launch_gemm(p, EPI_F32, 128, 128, false, (a.T + 127) / 128, false, s);
}

// Bitmaps from the top-k (SORT_TOPK), from caller routing (SORT_MARK), or already marked by the caller's kernel
// (SORT_MARKED); then the per-expert scan and the stable scatter.
enum { SORT_MARK = 0, SORT_TOPK = 1, SORT_MARKED = 2 };
static cudaError_t run_sort(const BlockArgs& a, int from, cudaStream_t s) {
  const int P = a.T * a.w.TOPK;
  cudaError_t e = cudaSuccess;
  if (from == SORT_TOPK) {
    prefill_topk_kernel<<<(a.T + kPT / 32 - 1) / (kPT / 32), kPT, 0, s>>>(a, 1);
    if ((e = launched(cudaGetLastError())) != cudaSuccess) return e;
  } else if (from == SORT_MARK) {
    prefill_mark_kernel<<<(P + kPT - 1) / kPT, kPT, 0, s>>>(a);
    if ((e = launched(cudaGetLastError())) != cudaSuccess) return e;
  }
  prefill_scan_kernel<<<a.w.E, kPT, 0, s>>>(a);
  if ((e = launched(cudaGetLastError())) != cudaSuccess) return e;
  prefill_scatter_kernel<<<(P + kPT - 1) / kPT, kPT, 0, s>>>(a);
  return launched(cudaGetLastError());
}

static cudaError_t run_experts(const BlockArgs& a, cudaStream_t s, void* mark = nullptr) {
  const int P = a.T * a.w.TOPK;
  int rows_gu, rows_dn;
  expert_tile_rows(&rows_gu, &rows_dn);
  const bool dgu = rows_gu > kTileRows, ddn = rows_dn > kTileRows;
  // gate/up: A = normed rows of the sorted pairs' tokens (gathered: a sorted copy loaded as TMA tiles measured
  // 10 us faster in the GEMM but cost 30 us to write), B = expert gate rows i and up rows I + i
  GemmParams g = base_params(a);
  g.A = a.normed;
  g.lda = a.xstride ? a.xstride : a.w.H;
  g.a_rows = a.sorted;
  g.a_div = a.w.TOPK;
  g.list_len = P;
  g.a_nrows = a.T;
  g.Bq = a.w.exp_gu_q;
  g.Bs = a.w.exp_gu_s;
  g.b_rows_per_e = 2 * (int64_t)a.w.I;
  g.paired = 1;
  g.pair_off = a.w.I;
  g.N = 2 * a.w.I;
  g.n_valid = g.N;
  g.K = a.w.H;
  g.E = a.w.E;
  g.tiles = static_cast<const GemmTile*>(dgu ? a.tiles2 : a.tiles);
  g.ntiles = dgu ? a.ntiles2 : a.ntiles;
  g.out = a.inter;
  g.ldo = a.w.I;
  g.out_nrows = P;
  cudaError_t e = launch_wide(g, EPI_SILU_TILE, true, rows_gu, dgu ? a.max_tiles2 : a.max_tiles, s);
  if (e == cudaSuccess) e = record_event(mark, s);
  if (e != cudaSuccess) return e;
  // down: A = inter rows in sorted order, B = expert down rows; epilogue weights by w[pair] into slot[pair]
  GemmParams d = base_params(a);
  d.A = a.inter;
  d.lda = a.w.I;
  d.a_nrows = P;
  d.Bq = a.w.exp_dn_q;
  d.Bs = a.w.exp_dn_s;
  d.b_rows_per_e = a.w.H;
  d.N = a.w.H;
  d.n_valid = d.N;
  d.K = a.w.I;
  d.E = a.w.E;
  d.tiles = static_cast<const GemmTile*>(ddn ? a.tiles2 : a.tiles);
  d.ntiles = ddn ? a.ntiles2 : a.ntiles;
  d.out = a.slot;
  d.ldo = a.w.H;
  d.out_rows = a.sorted;
  d.list_len = P;
  d.row_scale = a.wts;
  d.out_nrows = P;
  return launch_wide(d, EPI_SLOT, true, rows_dn, ddn ? a.max_tiles2 : a.max_tiles, s);
}

cudaError_t prefill_shared(const BlockArgs& a, cudaStream_t s) {
  GemmParams g = base_params(a);
  g.A = a.normed;
  g.lda = a.w.H;
  g.a_nrows = a.T;
  g.Bh = a.w.shared_gate_up;
  g.paired = 1;
  g.pair_off = a.w.Is;
  g.N = 2 * a.w.Is;
  g.n_valid = g.N;
  g.K = a.w.H;
  g.M = a.T;
  g.out = a.sinter;
  g.ldo = a.w.Is;
  g.out_nrows = a.T;
  cudaError_t e = launch_wide(g, EPI_SILU_ROUND, false, kTileRows, (a.T + 127) / 128, s);
  if (e != cudaSuccess) return e;
  GemmParams d = base_params(a);
  d.A = a.sinter;
  d.lda = a.w.Is;
  d.a_nrows = a.T;
  d.Bh = a.w.shared_down;
  d.N = a.w.H;
  d.n_valid = d.N;
  d.K = a.w.Is;
  d.M = a.T;
  d.out = a.sout;
  d.ldo = a.w.H;
  d.out_nrows = a.T;
  return launch_wide(d, EPI_BF16, false, kTileRows, (a.T + 127) / 128, s);
}

static cudaError_t clear_bits(const BlockArgs& a, cudaStream_t s) {
  return cudaMemsetAsync(a.bits, 0, sizeof(uint32_t) * (size_t)a.w.E * a.nwp, s);
}

cudaError_t prefill_router(const BlockArgs& a, cudaStream_t s) {
  cudaError_t e = run_router(a, s);
  if (e != cudaSuccess) return e;
  prefill_topk_kernel<<<(a.T + kPT / 32 - 1) / (kPT / 32), kPT, 0, s>>>(a, 0);
  return launched(cudaGetLastError());
}

cudaError_t prefill_routed(const BlockArgs& a, uint16_t* inter_out, cudaStream_t s) {
  cudaError_t e = clear_bits(a, s);
  if (e == cudaSuccess) e = run_sort(a, SORT_MARK, s);
  if (e == cudaSuccess) e = run_experts(a, s);
  if (e != cudaSuccess) return e;
  prefill_combine_kernel<<<a.T, kPT, 0, s>>>(a, 1);
  if ((e = launched(cudaGetLastError())) != cudaSuccess || !inter_out) return e;
  const int64_t n = (int64_t)a.T * a.w.TOPK * (a.w.I / 8);
  prefill_unsort_kernel<<<(unsigned)((n + kPT - 1) / kPT), kPT, 0, s>>>(a, inter_out);
  return launched(cudaGetLastError());
}

cudaError_t prefill_block(const BlockArgs& a, cudaStream_t s, void* const* marks) {
  cudaError_t e = clear_bits(a, s);
  if (e != cudaSuccess) return e;
  prefill_norm_kernel<<<a.T, kPT, 0, s>>>(a);
  if ((e = launched(cudaGetLastError())) != cudaSuccess) return e;
  if ((e = run_router(a, s)) != cudaSuccess) return e;
  if ((e = run_sort(a, SORT_TOPK, s)) != cudaSuccess) return e;
  if (marks && (e = record_event(marks[1], s)) != cudaSuccess) return e;
  if ((e = run_experts(a, s, marks ? marks[2] : nullptr)) != cudaSuccess) return e;
  if ((e = prefill_shared(a, s)) != cudaSuccess) return e;
  prefill_combine_kernel<<<a.T, kPT, 0, s>>>(a, 1 | 2);
  if ((e = launched(cudaGetLastError())) != cudaSuccess) return e;
  return marks ? record_event(marks[3], s) : cudaSuccess;
}

cudaError_t prefill_norm(const BlockArgs& a, cudaStream_t s) {
  prefill_norm_kernel<<<a.T, kPT, 0, s>>>(a);
  return launched(cudaGetLastError());
}

cudaError_t prefill_bits_clear(const BlockArgs& a, cudaStream_t s) { return clear_bits(a, s); }

cudaError_t prefill_routed_marked(const BlockArgs& a, cudaStream_t s) {
  cudaError_t e = run_sort(a, SORT_MARKED, s);
  if (e == cudaSuccess) e = run_experts(a, s);
  if (e != cudaSuccess) return e;
  prefill_combine_kernel<<<a.T, kPT, 0, s>>>(a, 1);
  return launched(cudaGetLastError());
}

cudaError_t prefill_routed_marked_gemms(const BlockArgs& a, cudaStream_t s) {
  cudaError_t e = run_sort(a, SORT_MARKED, s);
  return e == cudaSuccess ? run_experts(a, s) : e;
}

cudaError_t prefill_combine(const BlockArgs& a, cudaStream_t s) {
  prefill_combine_kernel<<<a.T, kPT, 0, s>>>(a, 2);
  return launched(cudaGetLastError());
}

}  // namespace moe
