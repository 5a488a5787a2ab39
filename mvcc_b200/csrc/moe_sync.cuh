// moe_sync.cuh -- synchronisation and routing helpers shared by the single-launch decode kernels (moe_fused.cu,
// moe_lean.cu): bulk asynchronous copies counted on shared-memory mbarriers, bounded waits, the grid barrier on a
// monotone arrival counter, and the reference's top-k rule in one warp.
#pragma once
#include <stdint.h>

#include "moe_device.cuh"
#include "moe_tc.cuh"

namespace moe {

using tc::fence_proxy_async_smem;
using tc::mbar_fence_init;
using tc::mbar_init;
using tc::smem_u32;

constexpr long long kSpinLimit = 1 << 21;          // grid-barrier polls (x ~100 ns) before giving up
constexpr unsigned long long kWaitNs = 1000000000; // stage-barrier wait limit (1 s of global time)
constexpr int kMinPolls = 1 << 18;                 // stage-barrier polls before a wait may give up at all
constexpr int kMaxPolls = 1 << 26;                 // stage-barrier polls after which a wait gives up whatever the timer

// ------------------------------------------------------------------ bulk copies and barriers

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(mbar))
               : "memory");
}
__device__ __forceinline__ void expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(mbar)),
      "r"(bytes)
      : "memory");
}
// Bytes of the 16-byte aligned superset of [src, src + bytes), and the offset of src within it.
__device__ __forceinline__ uint32_t span_bytes(const void* src, int bytes) {
  const uintptr_t s = reinterpret_cast<uintptr_t>(src);
  return (uint32_t)(((s + bytes + 15) & ~(uintptr_t)15) - (s & ~(uintptr_t)15));
}
__device__ __forceinline__ int span_delta(const void* src) { return (int)(reinterpret_cast<uintptr_t>(src) & 15); }
__device__ __forceinline__ void bulk_span(void* dst, const void* src, int bytes, uint64_t* mbar) {
  const uintptr_t s = reinterpret_cast<uintptr_t>(src);
  bulk_g2s(dst, reinterpret_cast<const void*>(s & ~(uintptr_t)15), span_bytes(src, bytes), mbar);
}

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for phase `parity` of the mbarrier; false once kWaitNs of global time and kMinPolls polls have both passed,
// or after kMaxPolls polls. %globaltimer is not guaranteed monotone (the driver may re-align it with the host clock),
// so the elapsed time is taken signed, a step backwards restarts the interval, a step forwards alone cannot end a
// wait, and the poll cap ends it even if the timer stood still.
__device__ __forceinline__ bool bar_wait(uint64_t* mbar, uint32_t parity) {
  const uint32_t addr = smem_u32(mbar);
  unsigned long long t0 = 0;
  for (int i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63) == 0) {
      const unsigned long long t = gtime();
      const long long dt = (long long)(t - t0);
      if (i == 0 || dt < 0) t0 = t;
      else if ((i >= kMinPolls && dt > (long long)kWaitNs) || i >= kMaxPolls) return false;
    }
  }
}
__device__ __forceinline__ int vload(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// CTA barrier that also reconverges the calling warp: after a section run by one lane (or part of a warp), the warp
// can leave bar.sync still split into groups that then issue every later instruction separately; __syncwarp joins
// them again.
__device__ __forceinline__ void cta_sync() {
  __syncthreads();
  __syncwarp();
}

// Relaxed read of the barrier counter at entry: any value from before this CTA's first arrival gives the base, and an
// acquire load would hold back the bulk copies issued after it.
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
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
  cta_sync();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(gbar) : "memory");
  __syncwarp();
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
      __nanosleep(20);
    }
    *ok_s = ok;
  }
  cta_sync();
  return *ok_s != 0;
}

// ------------------------------------------------------------------ routing in one warp

// Order-preserving 32-bit key of a float (larger float -> larger key); 0 is below every float's key.
__device__ __forceinline__ uint32_t fkey(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// The reference's top-k rule (router_topk_kernel, kernels.cuh:774-809) over one token's logits: K rounds of argmax
// by (value desc, index asc), weights exp(v - max) / sum over the picks. Each lane first sorts its 8 logits by (value
// desc, index asc); a round is then two warp reductions over the lanes' heads (redux.sync: max of the value key, min
// of the index among the lanes holding it) and a shift in the winning lane. Lane kk keeps pick kk. The rounds stay a
// loop: this code runs once per launch, and a compact body costs fewer instruction fetches than an unrolled one.
__device__ __forceinline__ void cas_desc(uint32_t& ka, int& ia, uint32_t& kb, int& ib) {
  // (ka, ia) before (kb, ib) when ka > kb, or ka == kb and ia < ib
  const bool swap = kb > ka || (kb == ka && ib < ia);
  const uint32_t k0 = swap ? kb : ka, k1 = swap ? ka : kb;
  const int i0 = swap ? ib : ia, i1 = swap ? ia : ib;
  ka = k0; kb = k1; ia = i0; ib = i1;
}
__device__ __forceinline__ void topk_warp_redux(const float* row, int E, int K, int32_t* idx_out, float* wts_out) {
  const int lane = threadIdx.x & 31;
  uint32_t k0, k1, k2, k3, k4, k5, k6, k7;
  int i0 = lane, i1 = lane + 32, i2 = lane + 64, i3 = lane + 96, i4 = lane + 128, i5 = lane + 160, i6 = lane + 192,
      i7 = lane + 224;
  k0 = fkey(i0 < E ? __ldcg(row + i0) : -1e30f);
  k1 = fkey(i1 < E ? __ldcg(row + i1) : -1e30f);
  k2 = fkey(i2 < E ? __ldcg(row + i2) : -1e30f);
  k3 = fkey(i3 < E ? __ldcg(row + i3) : -1e30f);
  k4 = fkey(i4 < E ? __ldcg(row + i4) : -1e30f);
  k5 = fkey(i5 < E ? __ldcg(row + i5) : -1e30f);
  k6 = fkey(i6 < E ? __ldcg(row + i6) : -1e30f);
  k7 = fkey(i7 < E ? __ldcg(row + i7) : -1e30f);
  // Batcher's odd-even merge sort of 8 (19 compare-exchanges)
  cas_desc(k0, i0, k1, i1); cas_desc(k2, i2, k3, i3); cas_desc(k4, i4, k5, i5); cas_desc(k6, i6, k7, i7);
  cas_desc(k0, i0, k2, i2); cas_desc(k1, i1, k3, i3); cas_desc(k4, i4, k6, i6); cas_desc(k5, i5, k7, i7);
  cas_desc(k1, i1, k2, i2); cas_desc(k5, i5, k6, i6);
  cas_desc(k0, i0, k4, i4); cas_desc(k1, i1, k5, i5); cas_desc(k2, i2, k6, i6); cas_desc(k3, i3, k7, i7);
  cas_desc(k2, i2, k4, i4); cas_desc(k3, i3, k5, i5);
  cas_desc(k1, i1, k2, i2); cas_desc(k3, i3, k4, i4); cas_desc(k5, i5, k6, i6);
  uint32_t mykey = 0;
  int myidx = 0;
#pragma unroll 1
  for (int kk = 0; kk < K; ++kk) {
    const uint32_t mk = __reduce_max_sync(0xffffffffu, k0);
    const int wi = (int)__reduce_min_sync(0xffffffffu, k0 == mk ? (uint32_t)i0 : 0x7fffffffu);
    if (lane == kk) {
      mykey = mk;
      myidx = wi;
    }
    if (i0 == wi) {  // the winner pops its head
      k0 = k1; i0 = i1; k1 = k2; i1 = i2; k2 = k3; i2 = i3; k3 = k4; i3 = i4;
      k4 = k5; i4 = i5; k5 = k6; i5 = i6; k6 = k7; i6 = i7; k7 = 0; i7 = 0x7fffffff;
    }
    __syncwarp();
  }
  // picks come in descending order, so the first is the maximum
  const float mx = fkey_inv(__shfl_sync(0xffffffffu, mykey, 0));
  const float ev = lane < K ? __expf(fkey_inv(mykey) - mx) : 0.f;
  float den = 0.f;
#pragma unroll 1
  for (int kk = 0; kk < K; ++kk) den += __shfl_sync(0xffffffffu, ev, kk);
  if (lane < K) {
    idx_out[lane] = myidx;
    wts_out[lane] = ev / den;
  }
  __syncwarp();
}

}  // namespace moe
