// moe_decode.cu -- decode-path kernels of the MoE block for T <= 16 tokens per call.
//
// Three launches per block (the reference issues eight, qwen.cu:429-448), chained with programmatic dependent
// launch: each kernel first fetches the weights that do not depend on its predecessor (router rows, shared-expert
// rows), then waits (griddepcontrol.wait) for the predecessor's results.
//   route_kernel     residual + RMSNorm, router GEMV, shared-expert gate logit; the last CTA to finish (ticket)
//                    runs top-k and builds the unique-expert table, so every routed expert's weights are streamed
//                    once per call however many tokens picked it.
//   gate_up_kernel   per SM, 9 warps take routed int4 gate/up row pairs (+ SiLU) of the unique experts and 3 warps
//                    take bf16 shared-expert gate/up row pairs, so each SM mixes ALU-heavy and byte-heavy rows.
//   down_kernel      per output row h: routed int4 down rows of the unique experts (weighted per pair), shared down,
//                    sigmoid-gated residual combine; the last CTA optionally applies the next layer's RMSNorm.
// Grids are one wave (<= one CTA per SM) so that a waiting dependent never blocks a running predecessor.
//
// Lane/k mapping: a lane owns 32-k chunks c = lane + 32j of a row (16 bytes of nibbles, 64 bytes of bf16), as the
// reference's int4 GEMV does (kernels.cuh:850-857). Activations sit in shared memory in a permuted order in which,
// for a fixed word q of the chunk, consecutive lanes read consecutive 16-byte vectors (no bank conflicts).
#include <algorithm>
#include <cstdlib>

#include "moe_device.cuh"

namespace moe {

constexpr int kDecodeMaxT = 16;
constexpr int kGuWarps = 12, kGuRoutedWarps = 9;  // gate_up_kernel: 384 threads, 9 routed + 3 shared warps
constexpr int kDnWarps = 16;                       // down_kernel: 512 threads

// ------------------------------------------------------------------ routing table

// From idx [P] (P = T * TOPK pairs): nuniq, uniq[u] ascending, uoff[u..u+1] = the range of upairs holding expert
// uniq[u]'s pairs in ascending pair order. Block-wide, deterministic. Pairs whose expert id lies outside [0, E)
// are dropped and flagged in the error word.
__device__ void build_unique(const int32_t* idx_s, int P, int E, BlockArgs& a, int* cnt_s, int* start_s) {
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) cnt_s[e] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    const int e = idx_s[p];
    if (e >= 0 && e < E) atomicAdd(&cnt_s[e], 1);
    else atomicOr(a.err, (uint32_t)MOE_ERR_EXPERT_INDEX);
  }
  __syncthreads();
  if (tid < 32) {
    const int lane = tid;
    constexpr int PER = 8;  // E <= 256
    int nz = 0, np = 0;
    for (int j = 0; j < PER; ++j) {
      const int e = lane * PER + j;
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
    for (int j = 0; j < PER; ++j) {
      const int e = lane * PER + j;
      if (e < E && cnt_s[e] > 0) {
        a.uniq[nz_ex] = e;
        a.uoff[nz_ex] = np_ex;
        start_s[e] = np_ex;
        ++nz_ex;
        np_ex += cnt_s[e];
      }
    }
    if (lane == 31) {
      *a.nuniq = nz_ex;
      a.uoff[nz_ex] = np_ex;
    }
  }
  __syncthreads();
  for (int p = tid; p < P; p += blockDim.x) {
    const int e = idx_s[p];
    if (e < 0 || e >= E) continue;
    int rank = 0;
    for (int q = 0; q < p; ++q) rank += (idx_s[q] == e);
    a.upairs[start_s[e] + rank] = p;
  }
}

// ------------------------------------------------------------------ K1: norm + router + top-k

// NB8 = 16-byte chunks per lane of one router row (H / 256). flags: 1 = norm from hidden + attn_out (else read
// `normed`), 2 = shared-expert gate: the gate vector is handled as router row E, its logit goes through sigmoid
// into `gate` (shared_gate_combine_kernel, kernels.cuh:1087-1090).
template <int NB8>
__global__ void __launch_bounds__(256) route_kernel(BlockArgs a, int flags) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);  // [T][H] bf16
  __shared__ float red[32];
  __shared__ int32_t idx_s[kDecodeMaxT * 8];
  __shared__ int cnt_s[256], start_s[256];
  __shared__ int is_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.w.H, E = a.w.E, T = a.T, K = a.w.TOPK;
  const int nvec = H >> 3;
  const int rows = E + ((flags & 2) ? 1 : 0);

  // Router row of this warp into registers first: it does not depend on the previous kernel.
  const int e = blockIdx.x * 8 + warp;
  uint4 wv[NB8];
  if (e < rows) {
    const uint16_t* wrow = e < E ? a.w.router + (int64_t)e * H : a.w.shared_gate;
#pragma unroll
    for (int m = 0; m < NB8; ++m) {
      const int v = lane + 32 * m;
      if (v < nvec) wv[m] = ldg_stream(wrow + v * 8);
    }
  }
  pdl_launch_dependents();
  pdl_wait();

  if (flags & 1) {
    for (int t = 0; t < T; ++t) {
      const float4* hr = reinterpret_cast<const float4*>(a.hidden + (int64_t)t * H);
      const uint2* dr = reinterpret_cast<const uint2*>(a.attn_out + (int64_t)t * H);
      float4 hv[4];
      uint2 dv[4];
      float ss = 0.f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {  // H <= 4096 = 4 x 256 threads x 4
        const int i = tid + r * blockDim.x;
        if (i < H / 4) {
          hv[r] = hr[i];
          dv[r] = dr[i];
        }
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = tid + r * blockDim.x;
        if (i < H / 4) {
          hv[r].x += lo_bf(dv[r].x);
          hv[r].y += hi_bf(dv[r].x);
          hv[r].z += lo_bf(dv[r].y);
          hv[r].w += hi_bf(dv[r].y);
          ss += hv[r].x * hv[r].x;
          ss += hv[r].y * hv[r].y;
          ss += hv[r].z * hv[r].z;
          ss += hv[r].w * hv[r].w;
        }
      }
      ss = block_sum(ss, red);
      const float inv = rsqrtf(ss / (float)H + a.w.eps);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = tid + r * blockDim.x;
        if (i < H / 4) {
          const uint2 wr = reinterpret_cast<const uint2*>(a.w.rms2)[i];
          const uint32_t y0 = f2bf(hv[r].x * inv * lo_bf(wr.x)), y1 = f2bf(hv[r].y * inv * hi_bf(wr.x));
          const uint32_t y2 = f2bf(hv[r].z * inv * lo_bf(wr.y)), y3 = f2bf(hv[r].w * inv * hi_bf(wr.y));
          const uint2 y = make_uint2(y0 | (y1 << 16), y2 | (y3 << 16));
          reinterpret_cast<uint2*>(xs + t * H)[i] = y;
          if (blockIdx.x == 0) reinterpret_cast<uint2*>(a.normed + (int64_t)t * H)[i] = y;
        }
      }
    }
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(a.normed);
    uint4* dst = reinterpret_cast<uint4*>(xs);
    for (int i = tid; i < T * H / 8; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();

  // Router GEMV: uint4 chunks at lane + 32m, fmaf in k order, butterfly sum (gemv_bf16_kernel, kernels.cuh:124-155).
  if (e < rows) {
    for (int t = 0; t < T; ++t) {
      float acc = 0.f;
#pragma unroll
      for (int m = 0; m < NB8; ++m) {
        const int v = lane + 32 * m;
        if (v < nvec) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + t * H + v * 8);
          const uint32_t ww[4] = {wv[m].x, wv[m].y, wv[m].z, wv[m].w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc = fmaf(lo_bf(ww[j]), lo_bf(xx[j]), acc);
            acc = fmaf(hi_bf(ww[j]), hi_bf(xx[j]), acc);
          }
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) {
        if (e < E) a.logits[(int64_t)t * E + e] = a.w.router_bias ? acc + a.w.router_bias[e] : acc;
        else a.gate[t] = sigmoid(acc);
      }
    }
  }

  // Last CTA: top-k over the complete logits, then the unique-expert table.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    // atomicInc wraps to 0 after gridDim.x - 1 arrivals, so a counter that starts the launch at zero ends it at
    // zero. It must start at zero (moe_workspace_init, or the clear in the allocation-free router): a stale value
    // would shift which CTA sees gridDim.x - 1, and that CTA would not be the last to arrive.
    const unsigned tk = atomicInc(&a.ticket[TICKET_ROUTE], gridDim.x - 1);
    is_last = (tk == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int t = warp; t < T; t += 8) topk_warp(a.logits + (int64_t)t * E, E, K, a.idx + t * K, a.wts + t * K);
  __syncthreads();
  for (int p = tid; p < T * K; p += blockDim.x) idx_s[p] = __ldcg(a.idx + p);
  __syncthreads();
  build_unique(idx_s, T * K, E, a, cnt_s, start_s);
}

// Unique-expert table from caller-provided idx (moe_routed_experts). One CTA.
__global__ void __launch_bounds__(256) route_table_kernel(BlockArgs a) {
  __shared__ int32_t idx_s[kDecodeMaxT * 8];
  __shared__ int cnt_s[256], start_s[256];
  pdl_launch_dependents();
  pdl_wait();
  const int P = a.T * a.w.TOPK;
  for (int p = threadIdx.x; p < P; p += blockDim.x) idx_s[p] = a.idx[p];
  __syncthreads();
  build_unique(idx_s, P, a.w.E, a, cnt_s, start_s);
}

// ------------------------------------------------------------------ K2: gate/up

template <int NCL>
struct RoutedRow {
  uint4 g[NCL], u[NCL];
  float gs[NCL], us[NCL];
};

template <int NCL>
__device__ __forceinline__ void load_routed(const BlockArgs& a, int e, int i, int gshift, RoutedRow<NCL>& r) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, I = a.w.I, G = a.w.G;
  const int64_t rowbytes = H >> 1, groups = H / G;
  const uint8_t* gw = a.w.exp_gu_q + ((int64_t)e * 2 * I + i) * rowbytes;
  const uint8_t* uw = gw + (int64_t)I * rowbytes;
  const uint16_t* gsr = a.w.exp_gu_s + ((int64_t)e * 2 * I + i) * groups;
  const uint16_t* usr = gsr + (int64_t)I * groups;
  const int nch = H >> 5;
#pragma unroll
  for (int j = 0; j < NCL; ++j) {
    const int c = lane + 32 * j;
    if (c < nch) {
      r.g[j] = ldg_stream(gw + c * 16);
      r.u[j] = ldg_stream(uw + c * 16);
      r.gs[j] = h2f(__ldg(gsr + (c >> gshift)));
      r.us[j] = h2f(__ldg(usr + (c >> gshift)));
    }
  }
}

// inter[pair][i] = bf16(silu(g) * u) for every pair of unique expert uix: per lane, per 32-k chunk, the packed
// position-scaled nibble dot times the chunk's group scale, then a butterfly sum (the reduction structure of
// moe_gate_up_int4_kernel, kernels.cuh:827-860).
template <int NCL>
__device__ __forceinline__ void compute_routed(const BlockArgs& a, const float* xs, const int* uoff_s,
                                               const int* upairs_s, const int* ptok_s, int uix, int i,
                                               const RoutedRow<NCL>& r, const Nib8Magic& M) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, I = a.w.I;
  const int nch = H >> 5;
  for (int p = uoff_s[uix]; p < uoff_s[uix + 1]; ++p) {
    const int pair = upairs_s[p];
    const float* xt = xs + ptok_s[p] * H;
    float g = 0.f, u = 0.f;
#pragma unroll
    for (int j = 0; j < NCL; ++j) {
      const int c = lane + 32 * j;
      if (c < nch) {
        Nib8Acc ag, au;
        nib8_zero(ag);
        nib8_zero(au);
        const uint32_t gw[4] = {r.g[j].x, r.g[j].y, r.g[j].z, r.g[j].w};
        const uint32_t uw[4] = {r.u[j].x, r.u[j].y, r.u[j].z, r.u[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          u64 x01, x23, x45, x67;
          lds_pairs(xt + ((q * 2) * nch + c) * 4, x01, x23);
          lds_pairs(xt + ((q * 2 + 1) * nch + c) * 4, x45, x67);
          nib8x2(gw[q], x01, x23, x45, x67, M, ag);
          nib8x2(uw[q], x01, x23, x45, x67, M, au);
        }
        g = fmaf(nib8_fold(ag), r.gs[j], g);
        u = fmaf(nib8_fold(au), r.us[j], u);
      }
    }
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) a.inter[(int64_t)pair * I + i] = f2bf(silu(g) * u);
  }
}

// sinter[t][j] for every token from the staged bf16 gate row j and up row Is + j (gemv_bf16_kernel per token,
// then silu_mul_kernel on the bf16-rounded outputs, qwen.cu:436-437).
template <int NCL>
__device__ __forceinline__ void compute_shared_row(const BlockArgs& a, const float* xs, int j, const uint4* stage) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, Is = a.w.Is, nch = H >> 5;
  for (int t = 0; t < a.T; ++t) {
    const float4* xs4 = reinterpret_cast<const float4*>(xs + t * H);
    float g = 0.f, u = 0.f;
#pragma unroll
    for (int m = 0; m < NCL; ++m) {
      const int c = lane + 32 * m;
      if (c < nch) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float x[8];
          x_word(xs4, nch, c, q, x);
          g = dot_bf16_word(stage[((0 * NCL + m) * 4 + q) * 32 + lane], x, g);
          u = dot_bf16_word(stage[((1 * NCL + m) * 4 + q) * 32 + lane], x, u);
        }
      }
    }
    g = warp_sum(g);
    u = warp_sum(u);
    // sgu is bf16 (qwen.cu:436, OutT = bf16), then silu_mul_kernel (kernels.cuh:1071-1079).
    if (lane == 0) a.sinter[(int64_t)t * Is + j] = f2bf(silu(bf2f(f2bf(g))) * bf2f(f2bf(u)));
  }
}

// Shared-expert row pair staged in shared memory: [g|u][NCL][q][lane] uint4 (conflict-free lane reads).
template <int NCL>
__device__ __forceinline__ void stage_shared_row(const BlockArgs& a, int j, uint4* stage) {
  const int lane = threadIdx.x & 31;
  const int H = a.w.H, nch = H >> 5;
  const uint16_t* grow = a.w.shared_gate_up + (int64_t)j * H;
  const uint16_t* urow = a.w.shared_gate_up + (int64_t)(a.w.Is + j) * H;
#pragma unroll
  for (int m = 0; m < NCL; ++m) {
    const int c = lane + 32 * m;
    if (c < nch) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        cp_async16(stage + ((0 * NCL + m) * 4 + q) * 32 + lane, grow + c * 32 + q * 8);
        cp_async16(stage + ((1 * NCL + m) * 4 + q) * 32 + lane, urow + c * 32 + q * 8);
      }
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int NCL>
constexpr int shared_stage_uint4() { return 2 * NCL * 4 * 32; }  // per warp

// flags: 1 = routed experts, 2 = shared expert. 384 threads; with both, warps [0, 9) routed, [9, 12) shared.
// Dynamic shared memory: T x H fp32 activations (permuted), then one staged shared-expert row pair per warp.
template <int NCL>
__global__ void __launch_bounds__(384) gate_up_kernel(BlockArgs a, int flags) {
  extern __shared__ __align__(16) float xs[];  // [T][H] fp32, permuted (xperm)
  __shared__ int uniq_s[256], uoff_s[257], upairs_s[kDecodeMaxT * 8], ptok_s[kDecodeMaxT * 8];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int H = a.w.H, T = a.T, nch = H >> 5;
  const int gshift = __ffs(a.w.G) - 6;  // 32-k chunk -> group: c >> gshift (G = 32, 64, 128)
  const bool routed = flags & 1, shared = flags & 2;
  // Warps [0, n_rw) take routed rows, the last kGuWarps - kGuRoutedWarps warps shared-expert rows (the routed
  // warps idle when only the shared expert runs, so shared memory holds at most three staged row pairs).
  const int n_rw = routed && !shared ? kGuWarps : kGuRoutedWarps;
  const bool is_shared_warp = shared && warp >= n_rw;

  // Shared-expert warps start copying their first row pair into shared memory before waiting on the routing
  // kernel (cp.async: no registers held across the wait).
  const int n_sw = (kGuWarps - n_rw) * gridDim.x;
  const int sw = blockIdx.x * (kGuWarps - n_rw) + (warp - n_rw);
  uint4* stage = reinterpret_cast<uint4*>(xs + (size_t)T * H) + (size_t)(warp - n_rw) * shared_stage_uint4<NCL>();
  if (is_shared_warp && sw < a.w.Is) stage_shared_row<NCL>(a, sw, stage);
  pdl_launch_dependents();
  pdl_wait();

  // Routed warps: job range, and the first job's rows in flight before the shared-memory prologue.
  const int I = a.w.I;
  int U = 0, j0 = 0, j1 = 0;
  RoutedRow<NCL> ra, rb;
  if (routed && !is_shared_warp) {
    U = table_nuniq(a);
    const int J = U * I;
    const int nw = gridDim.x * n_rw, rw = blockIdx.x * n_rw + warp;
    j0 = (int)(((int64_t)rw * J) / nw);
    j1 = (int)(((int64_t)(rw + 1) * J) / nw);
    if (j0 < j1) load_routed<NCL>(a, clampi(a.uniq[j0 / I], 0, a.w.E - 1), j0 % I, gshift, ra);
  }

  for (int i = tid; i < T * H / 4; i += blockDim.x) {  // 4 consecutive k stay consecutive under xperm
    const int t = (i * 4) / H, k = i * 4 - t * H;
    const uint2 v = reinterpret_cast<const uint2*>(a.normed)[i];
    *reinterpret_cast<float4*>(xs + t * H + xperm(k, nch)) = make_float4(lo_bf(v.x), hi_bf(v.x), lo_bf(v.y),
                                                                         hi_bf(v.y));
  }
  if (routed) {
    const int Ut = table_nuniq(a), P = T * a.w.TOPK;
    for (int i = tid; i < Ut; i += blockDim.x) uniq_s[i] = clampi(a.uniq[i], 0, a.w.E - 1);
    for (int i = tid; i <= Ut; i += blockDim.x) uoff_s[i] = clampi(a.uoff[i], 0, P);
    for (int i = tid; i < P; i += blockDim.x) {
      const int pr = clampi(a.upairs[i], 0, P - 1);
      upairs_s[i] = pr;
      ptok_s[i] = pr / a.w.TOPK;
    }
  }
  __syncthreads();

  if (is_shared_warp) {
    for (int j = sw; j < a.w.Is; j += n_sw) {
      if (j != sw) {
        __syncwarp();  // the previous row pair is consumed before the stage is overwritten
        stage_shared_row<NCL>(a, j, stage);
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncwarp();
      compute_shared_row<NCL>(a, xs, j, stage);
    }
    return;
  }
  if (!routed || j0 >= j1) return;
  // Walk the jobs (unique expert, row) incrementally, two row pairs in flight.
  const Nib8Magic M = nib8_magic();
  int ua = j0 / I, ia = j0 % I;
  for (int j = j0; j < j1; j += 2) {
    int ub = ua, ib = ia + 1;
    if (ib == I) { ib = 0; ++ub; }
    if (j + 1 < j1) load_routed<NCL>(a, uniq_s[ub], ib, gshift, rb);
    compute_routed<NCL>(a, xs, uoff_s, upairs_s, ptok_s, ua, ia, ra, M);
    if (j + 1 < j1) {
      ua = ub;
      ia = ib + 1;
      if (ia == I) { ia = 0; ++ua; }
      if (j + 2 < j1) load_routed<NCL>(a, uniq_s[ua], ia, gshift, ra);
      compute_routed<NCL>(a, xs, uoff_s, upairs_s, ptok_s, ub, ib, rb, M);
    }
  }
}

// ------------------------------------------------------------------ K3: down + combine

// mode bits: 1 = routed, 2 = shared, 4 = combine into hidden (with 1|2), 8 = next-layer RMSNorm.
// NCD = 16-k chunks per lane of a down row (I / 512 rounded up), NBS = uint4 per lane of a shared down row
// (Is / 256 rounded up), XF32 = stage the routed intermediates as fp32 (else bf16, converted on use).
template <int NCD, int NBS, bool XF32>
__global__ void __launch_bounds__(512) down_kernel(BlockArgs a, int mode) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int T = a.T, H = a.w.H, I = a.w.I, Is = a.w.Is, K = a.w.TOPK;
  const int P = T * K;
  const int nchd = I >> 4, L = min(32, nchd), PI = inter_stride(I);
  const int gshift = __ffs(a.w.G) - 5;  // 16-k chunk -> group: c >> gshift
  constexpr int XB = XF32 ? 4 : 2;     // bytes per staged inter value
  uint8_t* inter_s = smem;                                                    // [P][PI] permuted (iperm)
  uint16_t* sinter_s = reinterpret_cast<uint16_t*>(smem + (size_t)P * PI * XB);  // [T][Is]
  float* acc_s = reinterpret_cast<float*>(sinter_s + (size_t)T * Is);       // [warps][T][32]
  __shared__ float wts_s[kDecodeMaxT * 8];
  __shared__ int uniq_s[256], uoff_s[257], upairs_s[kDecodeMaxT * 8], ptok_s[kDecodeMaxT * 8];
  __shared__ float red[32];
  __shared__ int is_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool routed = mode & 1, shared = mode & 2;
  const int rows_per_cta = (H + gridDim.x - 1) / gridDim.x;
  const int h0 = blockIdx.x * rows_per_cta, h1 = min(H, h0 + rows_per_cta);
  const int nvs = Is >> 3;

  // The first row's shared-expert down weights do not depend on the gate/up kernel.
  uint4 sw[NBS];
  int h = h0 + warp;
  if (shared && h < h1) {
    const uint16_t* srow = a.w.shared_down + (int64_t)h * Is;
#pragma unroll
    for (int m = 0; m < NBS; ++m) {
      const int v = lane + 32 * m;
      if (v < nvs) sw[m] = ldg_stream(srow + v * 8);
    }
  }
  pdl_launch_dependents();
  pdl_wait();

  const int64_t rowbytes = I >> 1, groups = I / a.w.G;
  // Rows of up to 8 unique experts (down row h of each) and their scales, in flight together.
  uint2 wq[8][NCD];
  float sc[8][NCD];
  auto load_batch = [&](int hh, int ub, int U_) {
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (ub + b < U_) {
        const int e = routed ? clampi(__ldg(a.uniq + ub + b), 0, a.w.E - 1) : 0;
        const uint8_t* wr = a.w.exp_dn_q + ((int64_t)e * H + hh) * rowbytes;
        const uint16_t* sr = a.w.exp_dn_s + ((int64_t)e * H + hh) * groups;
#pragma unroll
        for (int j = 0; j < NCD; ++j) {
          const int c = lane + 32 * j;
          if (c < nchd) {
            wq[b][j] = ldg_stream8(wr + c * 8);
            sc[b][j] = h2f(__ldg(sr + (c >> gshift)));
          }
        }
      }
    }
  };
  int U = 0;
  if (routed) {
    U = table_nuniq(a);
    if (h < h1) load_batch(h, 0, U);  // the first batch of the first row, before the prologue
    for (int i = tid; i < P * I / 8; i += blockDim.x) {  // 8 consecutive k stay consecutive under iperm
      const int p = (i * 8) / I, k = i * 8 - p * I;
      const uint4 v = reinterpret_cast<const uint4*>(a.inter)[i];
      uint8_t* dst = inter_s + ((size_t)p * PI + iperm(k, L)) * XB;
      if (XF32) {
        float4* d4 = reinterpret_cast<float4*>(dst);
        d4[0] = make_float4(lo_bf(v.x), hi_bf(v.x), lo_bf(v.y), hi_bf(v.y));
        d4[1] = make_float4(lo_bf(v.z), hi_bf(v.z), lo_bf(v.w), hi_bf(v.w));
      } else {
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
    for (int p = tid; p < P; p += blockDim.x) {
      wts_s[p] = a.wts[p];
      const int pr = clampi(a.upairs[p], 0, P - 1);
      upairs_s[p] = pr;
      ptok_s[p] = pr / K;
    }
    for (int i = tid; i < U; i += blockDim.x) uniq_s[i] = clampi(a.uniq[i], 0, a.w.E - 1);
    for (int i = tid; i <= U; i += blockDim.x) uoff_s[i] = clampi(a.uoff[i], 0, P);
  }
  if (shared) {
    const uint4* src = reinterpret_cast<const uint4*>(a.sinter);
    uint4* dst = reinterpret_cast<uint4*>(sinter_s);
    for (int i = tid; i < T * Is / 8; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();

  const Nib8Magic M = nib8_magic();
  float* acc_w = acc_s + (size_t)warp * T * 32;
  bool preloaded = routed;
  for (; h < h1; h += kDnWarps) {
    // Routed: per unique expert (batches of 8 rows in flight), per pair, lane partial times the routing weight
    // accumulated per token in shared memory; one butterfly sum per token at the end.
    float routed_t = 0.f;
    if (routed) {
      for (int t = 0; t < T; ++t) acc_w[t * 32 + lane] = 0.f;
      for (int ub = 0; ub < U; ub += 8) {
        if (!(preloaded && ub == 0)) load_batch(h, ub, U);
        preloaded = false;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          if (ub + b < U) {
            for (int p = uoff_s[ub + b]; p < uoff_s[ub + b + 1]; ++p) {
              const int pair = upairs_s[p];
              const uint8_t* xr = inter_s + (size_t)pair * PI * XB;
              float part = 0.f;
#pragma unroll
              for (int j = 0; j < NCD; ++j) {
                const int c = lane + 32 * j;
                if (c < nchd) {
                  u64 x01, x23, x45, x67;
                  Nib8Acc A;
                  nib8_zero(A);
                  inter_pairs<XF32>(xr + (size_t)((j * 2) * L + lane) * 8 * XB, x01, x23, x45, x67);
                  nib8x2(wq[b][j].x, x01, x23, x45, x67, M, A);
                  inter_pairs<XF32>(xr + (size_t)((j * 2 + 1) * L + lane) * 8 * XB, x01, x23, x45, x67);
                  nib8x2(wq[b][j].y, x01, x23, x45, x67, M, A);
                  part = fmaf(nib8_fold(A), sc[b][j], part);
                }
              }
              float* slot = acc_w + ptok_s[p] * 32 + lane;
              *slot = fmaf(wts_s[pair], part, *slot);
            }
          }
        }
      }
      for (int t = 0; t < T; ++t) {
        const float v = warp_sum(acc_w[t * 32 + lane]);
        if (lane == t) routed_t = v;
      }
    }
    // Shared expert down row h (gemv over sinter, kernels.cuh:124-155), bf16 output.
    float shared_t = 0.f;
    if (shared) {
      if (h != h0 + warp) {
        const uint16_t* srow = a.w.shared_down + (int64_t)h * Is;
#pragma unroll
        for (int m = 0; m < NBS; ++m) {
          const int v = lane + 32 * m;
          if (v < nvs) sw[m] = ldg_stream(srow + v * 8);
        }
      }
      for (int t = 0; t < T; ++t) {
        float acc = 0.f;
#pragma unroll
        for (int m = 0; m < NBS; ++m) {
          const int v = lane + 32 * m;
          if (v < nvs) {
            const uint4 xv = *reinterpret_cast<const uint4*>(sinter_s + t * Is + v * 8);
            const uint32_t ww[4] = {sw[m].x, sw[m].y, sw[m].z, sw[m].w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              acc = fmaf(lo_bf(ww[q]), lo_bf(xx[q]), acc);
              acc = fmaf(hi_bf(ww[q]), hi_bf(xx[q]), acc);
            }
          }
        }
        const float v = bf2f(f2bf(warp_sum(acc)));
        if (lane == t) shared_t = v;
      }
    }
    if (lane < T) {
      const int t = lane;
      const int64_t o = (int64_t)t * H + h;
      if (routed) a.routed[o] = routed_t;
      if (shared) a.sout[o] = f2bf(shared_t);
      if (mode & 4) {
        const float hh = a.hidden[o] + bf2f(a.attn_out[o]);  // the residual add of residual_rmsnorm_kernel
        const float g = a.gate[t];
        a.hidden[o] = (mode & 8) ? fmaf(g, shared_t, hh + routed_t) : hh + fmaf(g, shared_t, routed_t);
      }
    }
  }
  if (!(mode & 8)) return;
  // Next layer's RMSNorm over the finished rows: the last CTA to arrive (shared_gate_combine_rmsnorm_kernel).
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned tk = atomicInc(&a.ticket[TICKET_COMBINE], gridDim.x - 1);
    is_last = (tk == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int t = 0; t < T; ++t) {
    const float* hr = a.hidden + (int64_t)t * H;
    float ss = 0.f;
    for (int i = tid; i < H; i += blockDim.x) {
      const float v = __ldcg(hr + i);
      ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(ss / (float)H + a.w.eps);
    for (int i = tid; i < H; i += blockDim.x)
      a.normed[(int64_t)t * H + i] = f2bf(__ldcg(hr + i) * inv * bf2f(a.next_rms1[i]));
  }
}

// ------------------------------------------------------------------ launchers

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Raises a kernel's dynamic shared-memory limit on its first launch on a device, to at least 200 KB (grant_smem).
// Raised even for small requests: the default 48 KB limit covers static plus dynamic shared memory, so a dynamic
// request just under 48 KB can still exceed it. `granted` is a static of the caller, one per kernel instantiation.
template <typename F>
static cudaError_t set_smem(F* kern, size_t bytes, SmemGrant& granted) {
  return grant_smem(reinterpret_cast<const void*>(kern), bytes, (size_t)200 * 1024, granted);
}

// Programmatic dependent launch is on unless the environment sets MOE_B200_PDL=0 (read once per process).
static bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = getenv("MOE_B200_PDL");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Launch with programmatic stream serialization: the kernel may start while its predecessor on the stream is
// still running; it synchronises with griddepcontrol.wait before reading the predecessor's outputs.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), int grid, int block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return launched(cudaLaunchKernelEx(&cfg, kern, args...));
}

template <int NB8>
static cudaError_t route_dispatch(const BlockArgs& a, int flags, cudaStream_t s) {
  static SmemGrant granted;
  const size_t smem = (size_t)a.T * a.w.H * sizeof(uint16_t);
  cudaError_t err = set_smem(route_kernel<NB8>, smem, granted);
  if (err != cudaSuccess) return err;
  const int rows = a.w.E + ((flags & 2) ? 1 : 0);
  return launch_pdl(route_kernel<NB8>, (rows + 7) / 8, 256, smem, s, a, flags);
}

cudaError_t launch_route(const BlockArgs& a, bool from_hidden, bool with_gate, cudaStream_t s) {
  const int flags = (from_hidden ? 1 : 0) | (with_gate ? 2 : 0);
  if (a.w.H <= 1024) return route_dispatch<4>(a, flags, s);
  if (a.w.H <= 2048) return route_dispatch<8>(a, flags, s);
  return route_dispatch<16>(a, flags, s);
}

cudaError_t launch_route_table(const BlockArgs& a, cudaStream_t s) {
  return launch_pdl(route_table_kernel, 1, 256, 0, s, a);
}

template <int NCL>
static cudaError_t gate_up_dispatch(const BlockArgs& a, int flags, cudaStream_t s) {
  static SmemGrant granted;
  const size_t smem = gate_up_smem_bytes(a.T, a.w.H);
  cudaError_t err = set_smem(gate_up_kernel<NCL>, smem, granted);
  if (err != cudaSuccess) return err;
  return launch_pdl(gate_up_kernel<NCL>, sm_count(), kGuWarps * 32, smem, s, a, flags);
}

cudaError_t launch_gate_up(const BlockArgs& a, bool routed, bool shared, cudaStream_t s) {
  const int flags = (routed ? 1 : 0) | (shared ? 2 : 0);
  if (a.w.H <= 1024) return gate_up_dispatch<1>(a, flags, s);
  if (a.w.H <= 2048) return gate_up_dispatch<2>(a, flags, s);
  return gate_up_dispatch<4>(a, flags, s);
}

// Activations plus one staged shared-expert row pair per shared warp.
size_t gate_up_smem_bytes(int T, int H) {
  const int ncl = H <= 1024 ? 1 : (H <= 2048 ? 2 : 4);
  return (size_t)T * H * sizeof(float) + (size_t)(kGuWarps - kGuRoutedWarps) * 2 * ncl * 4 * 32 * 16;
}

size_t down_smem_bytes(int T, int TOPK, int I, int Is, bool xf32) {
  return (size_t)T * TOPK * inter_stride(I) * (xf32 ? 4 : 2) + (size_t)T * Is * 2 + (size_t)kDnWarps * T * 32 * 4;
}

template <int NCD, int NBS, bool XF32>
static cudaError_t down_dispatch(const BlockArgs& a, int mode, cudaStream_t s) {
  static SmemGrant granted;
  const size_t smem = down_smem_bytes(a.T, a.w.TOPK, a.w.I, a.w.Is, XF32);
  cudaError_t err = set_smem(down_kernel<NCD, NBS, XF32>, smem, granted);
  if (err != cudaSuccess) return err;
  return launch_pdl(down_kernel<NCD, NBS, XF32>, std::min(sm_count(), a.w.H), kDnWarps * 32, smem, s, a, mode);
}

template <int NCD, int NBS>
static cudaError_t down_dispatch_x(const BlockArgs& a, int mode, cudaStream_t s) {
  if (down_smem_bytes(a.T, a.w.TOPK, a.w.I, a.w.Is, true) <= 200 * 1024)
    return down_dispatch<NCD, NBS, true>(a, mode, s);
  return down_dispatch<NCD, NBS, false>(a, mode, s);
}

cudaError_t launch_down_combine(const BlockArgs& a, int mode, cudaStream_t s) {
  const int ncd = (a.w.I / 16 + 31) / 32, nbs = (a.w.Is / 8 + 31) / 32;
  if (ncd <= 1 && nbs <= 2) return down_dispatch_x<1, 2>(a, mode, s);
  if (ncd <= 2 && nbs <= 4) return down_dispatch_x<2, 4>(a, mode, s);
  return down_dispatch_x<4, 8>(a, mode, s);
}

}  // namespace moe
