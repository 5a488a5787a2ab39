// moe_device.cuh -- device helpers shared by the decode kernels (moe_decode.cu) and the fused decode kernel
// (moe_fused.cu): programmatic-dependent-launch waits, block reductions, the permuted activation layouts, the
// reference's top-k rule, bf16 row dots and cp.async.
#pragma once
#include "moe_common.cuh"
#include "moe_decode.h"

namespace moe {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  __syncwarp();  // bar.sync does not reconverge the warp split by the lane-0 store
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// Exclusive block-wide prefix sum of one int per thread (blockDim.x a multiple of 32, at most 1024); *total
// receives the block's sum. sm: 32 ints of shared memory.
__device__ __forceinline__ int block_excl_scan(int v, int* sm, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) sm[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? sm[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) sm[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int before = warp ? sm[warp - 1] : 0;
  *total = sm[nw - 1];
  return before + x - v;
}

// Position of k in the permuted fp32 activation row: k = 32c + 8q + 4h + e -> ((2q + h) * NCH + c) * 4 + e.
__device__ __forceinline__ int xperm(int k, int nch) {
  const int c = k >> 5, r = k & 31;
  return (((r >> 3) * 2 + ((r >> 2) & 1)) * nch + c) * 4 + (r & 3);
}

// The routing table lives in caller-owned workspace; every read of it that feeds an address is clamped to its
// valid range, so a stale or corrupted workspace can give wrong results but never an out-of-bounds access.
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ int table_nuniq(const BlockArgs& a) {
  return clampi(*a.nuniq, 0, min(a.w.E, a.T * a.w.TOPK));
}

// Warp top-k of one token's logits, the reference's rule (router_topk_kernel, kernels.cuh:774-809): K rounds of
// argmax by (value desc, index asc); weights = exp(v - max) / sum over the picks. Fully unrolled over the 8
// possible rounds so that picks stay in registers.
static __device__ void topk_warp(const float* row, int E, int K, int32_t* idx_out, float* wts_out) {
  const int lane = threadIdx.x & 31;
  float vals[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int e = lane + i * 32;
    vals[i] = e < E ? __ldcg(row + e) : -1e30f;
  }
  float pv[8];
  int pi[8];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    float bv = -1e30f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = lane + i * 32;
      if (vals[i] > bv || (vals[i] == bv && e < bi)) { bv = vals[i]; bi = e; }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    pv[kk] = bv;
    pi[kk] = bi;
    if (kk < K) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + i * 32 == bi) vals[i] = -1e30f;
    }
  }
  float mx = pv[0];
#pragma unroll
  for (int kk = 1; kk < 8; ++kk)
    if (kk < K) mx = fmaxf(mx, pv[kk]);
  float den = 0.f;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    pv[kk] = __expf(pv[kk] - mx);
    if (kk < K) den += pv[kk];
  }
  // lanes 0..K-1 write pick `lane` (a register select, no local memory)
  float myw = 0.f;
  int myi = 0;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    if (lane == kk) { myw = pv[kk]; myi = pi[kk]; }
  if (lane < K) {
    idx_out[lane] = myi;
    wts_out[lane] = myw / den;
  }
}

// x[k] for the 8 k of word q of chunk c from the permuted row xs4 (float4 view).
__device__ __forceinline__ void x_word(const float4* xs4, int nch, int c, int q, float* x) {
  const float4 x0 = xs4[(q * 2) * nch + c], x1 = xs4[(q * 2 + 1) * nch + c];
  x[0] = x0.x; x[1] = x0.y; x[2] = x0.z; x[3] = x0.w;
  x[4] = x1.x; x[5] = x1.y; x[6] = x1.z; x[7] = x1.w;
}

__device__ __forceinline__ float dot_bf16_word(const uint4& w, const float* x, float acc) {
  acc = fmaf(lo_bf(w.x), x[0], acc);
  acc = fmaf(hi_bf(w.x), x[1], acc);
  acc = fmaf(lo_bf(w.y), x[2], acc);
  acc = fmaf(hi_bf(w.y), x[3], acc);
  acc = fmaf(lo_bf(w.z), x[4], acc);
  acc = fmaf(hi_bf(w.z), x[5], acc);
  acc = fmaf(lo_bf(w.w), x[6], acc);
  acc = fmaf(hi_bf(w.w), x[7], acc);
  return acc;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}

// Permuted position of k in one bf16 inter row of stride inter_stride(I): lane chunk c = k / 16 = lane + 32j
// (L = min(32, I / 16) active lanes), halves of 8: ((j * 2 + half) * L + lane) * 8 + e, so that a warp's 16-byte
// reads of one half are consecutive.
__device__ __forceinline__ int iperm(int k, int L) {
  const int c = k >> 4, r = k & 15;
  return (((c >> 5) * 2 + (r >> 3)) * L + (c & 31)) * 8 + (r & 7);
}

// Packed float pairs of the 8 staged inter values at `src` (XF32: fp32 staging, else bf16 staging).
template <bool XF32>
__device__ __forceinline__ void inter_pairs(const void* src, u64& x01, u64& x23, u64& x45, u64& x67) {
  if (XF32) {
    lds_pairs(src, x01, x23);
    lds_pairs(static_cast<const float*>(src) + 4, x45, x67);
  } else {
    const uint4 v = *static_cast<const uint4*>(src);
    x01 = ((u64)(v.x & 0xffff0000u) << 32) | (u64)(v.x << 16);
    x23 = ((u64)(v.y & 0xffff0000u) << 32) | (u64)(v.y << 16);
    x45 = ((u64)(v.z & 0xffff0000u) << 32) | (u64)(v.z << 16);
    x67 = ((u64)(v.w & 0xffff0000u) << 32) | (u64)(v.w << 16);
  }
}

}  // namespace moe
