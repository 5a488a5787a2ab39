// moe_gemm.cu -- persistent, warp-specialized tcgen05 tile GEMM for the prefill path: the dense router and
// shared-expert GEMMs (dense(), qwen.cu:298-319) and the grouped INT4 expert GEMMs (moe_gate_up_tile_kernel,
// moe_down_tile_kernel, kernels.cuh:942-1057).
//
// One CTA per SM walks work items (tile of up to MS x 128 A rows) x (n-tile of BN B rows), K in steps of 64. Stage
// s of the ring holds one step's A rows (MS sub-tiles of 128) and bf16 B rows; full[s] completes when both are in,
// empty[s] when the MMAs that read them are done -- one wait and one commit per step for the issuing thread, whose
// shared-memory round trips (a few hundred cycles per barrier operation) must stay under a step's MMA time (512
// cycles per sub-tile at N = 256). MS = 2 (double tiles of the routed expert GEMMs) runs two 128-row sub-tiles
// against each dequantised B stage: half the dequantisation and barrier work per MMA.
// 4 + 4 MS + NDW warps (NDW = 8 dequantisation warps by default, 16 optionally):
//   warps 0-1   A producers: contiguous A rows come in as one 2D TMA tile (box 64 x 128, 128-byte swizzle) per
//               step; gathered rows (one per (token, slot) pair of the sorted pair list) come in by cp.async,
//               eight lanes per row so that each row is one 128-byte line request, into the same swizzled K-major
//               layout (cp.async.mbarrier.arrive.noinc on full[s]);
//   warp 2      B producer, one lane: TMA tiles of the step's bf16 B rows into stage s, or of INT4 rows (rk
//               k-steps of each row per box) into the raw ring (fullR) and, once per item, of the item's fp16 group
//               scales (double-buffered, or single where shared memory is short); completion by transaction count
//               (mbarrier expect_tx). Every load targets this CTA's own shared memory only;
//   warp 3      allocates TMEM (NB accumulator buffers of MS x BN fp32 columns: NB = 2 where they fit in 512
//               columns, else 1) and, from one lane, issues the tcgen05.mma of each step (M=128, N=BN, K=16 x 4
//               per sub-tile that holds rows), committing to empty[s] and, after an item's last step, to
//               acc_full[buffer];
//   warps 4..   4 MS epilogue warps: wait acc_full, tcgen05.ld the accumulator rows of their TMEM lane quarter
//               (warp % 4) of their sub-tile, apply the epilogue, store, release the buffer (acc_empty) --
//               overlapping the next item's main loop when NB = 2;
//   last NDW    INT4 only: each thread owns (row, K half) jobs of the tile (two at BN = 256 with 8 warps, one
//               with 16) and converts their 32 nibbles per step from the raw ring into the swizzled bf16 B of
//               stage s as dequant32_bf16 does
//               (kernels.cuh:925-940: bf16((q - 8) * scale), one rounding), fences the writes to the async proxy and
//               arrives on full[s]. Raw bytes and scales come by TMA: loading them through the load/store unit
//               costs about as many cycles as the conversion itself.
// Every wait is bounded: kWaitNs after its first miss a waiting thread records MOE_ERR_TIMEOUT in the error word,
// raises the CTA's abort flag (other waits poll it) and leaves its loop; the CTA then drains its copies, frees TMEM
// and exits.
//
// Exact dequantization with one FMA per pair of weights: a nibble q at bit position 4p of a word, OR-ed into
// 0x4B000000, is the float f = 2^23 + q * 2^(4p). For p in {2, 3, 4} the product M_p * s of the offset
// M_p = 2^23 + 8 * 2^(4p) with an fp16 scale s fits in 24 bits, so fma(f, s * 2^(-4p), -M_p * s * 2^(-4p))
// yields (q - 8) * s exactly (15 significant bits); every nibble of a word reaches one of those positions in the
// word itself, the word shifted left by 8 or shifted right by 12. One cvt.rn.bf16x2.f32 then rounds two values to
// bf16: the reference's single rounding.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "moe_common.cuh"
#include "moe_gemm.h"
#include "moe_tc.cuh"

namespace moe {

using namespace tc;

constexpr int kBK = 64, kTileM = 128;
// Warps 0-3 and the 4 MS epilogue warps have fixed roles; NDW dequantisation warps follow (8 by default, 16 with
// MOE_B200_GEMM_DEQ_WARPS=16 for the routed INT4 GEMMs: twice the warps to hide the conversion's latency, one job per
// thread at BN = 256).
__host__ __device__ constexpr int deq_warp0(int ms) { return 4 + 4 * ms; }
__host__ __device__ constexpr int gemm_threads(int ndw, int ms) { return (deq_warp0(ms) + ndw) * 32; }
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s: far beyond any item's main loop
constexpr uint32_t kMinPolls = 1u << 18;               // polls before a wait may give up at all
constexpr uint32_t kMaxPolls = 1u << 26;               // polls after which a wait gives up whatever the timer says

struct GemmCfg {
  int bn, sa;            // BN, A + B ring depth
  int ms, nb, nsc;       // 128-row sub-tiles per item, TMEM accumulator buffers, scale buffers
  int sr, rk;            // INT4: raw ring depth, k-steps per raw stage (a row's 32 * rk bytes per box)
  int ksc, sstride;      // INT4: scales per B row, their bytes per row in shared memory
  int a_tma, s_tma;      // A by TMA tiles (contiguous rows); scales by TMA (rows of at least 16 bytes)
  size_t a, b, raw, sc, bar, total;
};

__host__ __device__ inline GemmCfg gemm_cfg(int bn, bool int4, int sa, int sr, int rk, int K, int G, int ms,
                                            int nsc) {
  GemmCfg c;
  c.bn = bn;
  c.sa = sa;
  c.ms = ms;
  c.nb = 2 * ms * bn <= 512 ? 2 : 1;
  c.nsc = int4 ? nsc : 0;
  const int nk = K / kBK;
  while (rk > 1 && nk % rk) rk >>= 1;
  c.rk = rk;
  c.sr = int4 ? sr : 0;
  c.ksc = int4 ? K / G : 0;
  c.sstride = c.ksc * 2;
  c.a_tma = 0;
  c.s_tma = int4 && c.sstride >= 16;
  size_t o = 0;
  c.a = o;   o += (size_t)sa * ms * kTileM * 128;  // 16 KiB per sub-tile and stage (1024-byte aligned)
  c.b = o;   o += (size_t)sa * bn * 128;
  c.raw = o; o += (size_t)c.sr * bn * 32 * rk;
  c.sc = o;  o += int4 ? (size_t)c.nsc * bn * c.sstride : 0;
  c.bar = (o + 127) / 128 * 128;
  o = c.bar + 8 * (size_t)(2 * sa + 2 * c.sr + 8) + 16;
  c.total = o + 1024;  // the dynamic base is aligned up to 1024 bytes at run time
  return c;
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* mbar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(mbar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile(
      "{\n\t"
      ".reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t"
      "}" ::"r"(smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// 2D TMA tile load into this CTA's shared memory, completion counted in bytes on mbar (this CTA only).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(mbar))
      : "memory");
}
// 4D variant: a paired gate/up operand, viewed as [expert][half][row][k], comes in as one box of both halves.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(mbar))
      : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile(
      "{\n\t"
      ".reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t"
      "}" ::"r"(smem_u32(mbar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity; bounded in time (kWaitNs from the first miss, and at least kMinPolls
// polls: %globaltimer may step when the driver re-aligns it, so a step backwards restarts the interval and a step
// forwards alone cannot end a wait) and in polls (kMaxPolls, should the timer stand still), and gives up early when
// another role of the CTA has aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* mbar, uint32_t parity, volatile int* abort_flag, uint32_t* err) {
  const uint32_t a = smem_u32(mbar);
  unsigned long long t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 63) == 63) {
      if (*abort_flag) return false;
      const unsigned long long now = global_ns();
      const long long dt = (long long)(now - t0);
      if (t0 == 0 || dt < 0) {
        t0 = now;
      } else if ((i >= kMinPolls && dt > (long long)kWaitNs) || i >= kMaxPolls) {
        *abort_flag = 1;
        if (err) atomicOr(err, (uint32_t)MOE_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// Per-scale constants of dequant8_bf16: (scale * 2^(-4p), -M_p * scale * 2^(-4p)) packed for the position pairs
// (p2, p3), (p4, p2), (p3, p4).
struct DqConst {
  u64 s23, c23, s42, c42, s34, c34;
};
__device__ __forceinline__ u64 pack2f(float lo, float hi) {
  return ((u64)__float_as_uint(hi) << 32) | (u64)__float_as_uint(lo);
}
__device__ __forceinline__ DqConst dq_const(float s) {
  const float s2 = s * (1.f / 256.f), s3 = s * (1.f / 4096.f), s4 = s * (1.f / 65536.f);
  const float c2 = -32776.f * s, c3 = -2056.f * s, c4 = -136.f * s;  // -(2^15 + 8) s, -(2^11 + 8) s, -(2^7 + 8) s
  DqConst d;
  d.s23 = pack2f(s2, s3);
  d.c23 = pack2f(c2, c3);
  d.s42 = pack2f(s4, s2);
  d.c42 = pack2f(c4, c2);
  d.s34 = pack2f(s3, s4);
  d.c34 = pack2f(c3, c4);
  return d;
}

// 8 nibbles of u (k = 8w .. 8w + 7, nibble i at bits 4i) -> 8 bf16 (one 16-byte chunk), exact products, RNE.
//   nibbles 0, 1: u << 8 at p = 2, 3;  nibbles 2, 3, 4: u at p = 2, 3, 4;  nibbles 5, 6, 7: u >> 12 at p = 2, 3, 4.
__device__ __forceinline__ uint4 dequant8_bf16(uint32_t u, const DqConst& d) {
  uint4 o;
  asm("{\n\t"
      ".reg .b32 v0, v1, f0, f1, f2, f3, f4, f5, f6, f7;\n\t"
      ".reg .b64 p01, p23, p45, p67;\n\t"
      ".reg .f32 a0, a1, a2, a3, a4, a5, a6, a7;\n\t"
      "shl.b32 v0, %4, 8;\n\t"
      "shr.b32 v1, %4, 12;\n\t"
      "lop3.b32 f0, v0, 0xF00, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f1, v0, 0xF000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f2, %4, 0xF00, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f3, %4, 0xF000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f4, %4, 0xF0000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f5, v1, 0xF00, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f6, v1, 0xF000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f7, v1, 0xF0000, 0x4B000000, 0xEA;\n\t"
      "mov.b64 p01, {f0, f1};\n\t"
      "mov.b64 p23, {f2, f3};\n\t"
      "mov.b64 p45, {f4, f5};\n\t"
      "mov.b64 p67, {f6, f7};\n\t"
      "fma.rn.f32x2 p01, p01, %5, %6;\n\t"
      "fma.rn.f32x2 p23, p23, %5, %6;\n\t"
      "fma.rn.f32x2 p45, p45, %7, %8;\n\t"
      "fma.rn.f32x2 p67, p67, %9, %10;\n\t"
      "mov.b64 {a0, a1}, p01;\n\t"
      "mov.b64 {a2, a3}, p23;\n\t"
      "mov.b64 {a4, a5}, p45;\n\t"
      "mov.b64 {a6, a7}, p67;\n\t"
      "cvt.rn.bf16x2.f32 %0, a1, a0;\n\t"
      "cvt.rn.bf16x2.f32 %1, a3, a2;\n\t"
      "cvt.rn.bf16x2.f32 %2, a5, a4;\n\t"
      "cvt.rn.bf16x2.f32 %3, a7, a6;\n\t"
      "}"
      : "=r"(o.x), "=r"(o.y), "=r"(o.z), "=r"(o.w)
      : "r"(u), "l"(d.s23), "l"(d.c23), "l"(d.s42), "l"(d.c42), "l"(d.s34), "l"(d.c34));
  return o;
}

// 16-byte streaming load that bypasses L1 allocation (each weight byte is used by one thread once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int BN>
__device__ __forceinline__ int64_t b_row(const GemmParams& p, int e, int nt, int r) {
  int row;
  if (p.paired) row = r < BN / 2 ? nt * (BN / 2) + r : p.pair_off + nt * (BN / 2) + (r - BN / 2);
  else row = nt * BN + r;
  return (int64_t)e * p.b_rows_per_e + row;
}

template <int MS>
__device__ __forceinline__ GemmTile load_tile(const GemmParams& p, int ti) {
  GemmTile t;
  if (p.tiles) {
    t = p.tiles[ti];
  } else {
    t.e = 0;
    t.m0 = ti * MS * kTileM;
    t.mcount = p.M - t.m0;
  }
  t.e = min(max(t.e, 0), p.E - 1);
  t.mcount = max(0, min(t.mcount, MS * kTileM));
  if (t.m0 < 0) t.mcount = 0;
  return t;
}

// Position in a ring of n stages: the stage, the parity of its current use and whether the ring has wrapped (the
// stage's previous use must be released first). Kept incrementally: g % n and g / n are runtime divisions, about
// twenty instructions each, in every role's per-k-step loop.
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  bool reused = false;
  __device__ __forceinline__ void next(int n) {
    if (++s == n) {
      s = 0;
      ph ^= 1u;
      reused = true;
    }
  }
};

template <int BN, bool INT4, int EPI, int NDW, int MS>
__global__ void __launch_bounds__(gemm_threads(NDW, MS), 1)
    moe_gemm_kernel(const __grid_constant__ GemmParams p, const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmS, const GemmCfg c) {
  constexpr int kDeqThreads = NDW * 32, kDeqWarp0 = deq_warp0(MS);
  constexpr int NB = 2 * MS * BN <= 512 ? 2 : 1;  // TMEM accumulator buffers
  constexpr uint32_t kSubBytes = kTileM * 128;    // one 128-row A sub-tile of a stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int SA = c.sa, SR = c.sr, NSC = c.nsc;
  const int nN = p.N / BN, nk = p.K / kBK;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + c.bar);
  uint64_t* full = bars;
  uint64_t* empty = full + SA;
  uint64_t* fullR = empty + SA;
  uint64_t* freeR = fullR + SR;
  uint64_t* sc_full = freeR + SR;      // [NSC <= 2]
  uint64_t* sc_free = sc_full + 2;     // [NSC <= 2]
  uint64_t* acc_full = sc_free + 2;    // [NB <= 2]
  uint64_t* acc_empty = acc_full + 2;  // [NB <= 2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t cols = (uint32_t)(NB * MS * BN);  // 128, 256 or 512
  static_assert(cols == 128 || cols == 256 || cols == 512, "TMEM allocation");

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(&full[s], (c.a_tma ? 1 : 64) + (INT4 ? kDeqThreads / 32 : 1));
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < SR; ++s) {
      mbar_init(&fullR[s], 1);
      mbar_init(&freeR[s], kDeqThreads / 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sc_full[i], c.s_tma ? 1 : 32);
      mbar_init(&sc_free[i], kDeqThreads / 32);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4 * MS);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  // everything above touches only this CTA's shared memory: it overlaps the previous kernel under PDL
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int ntiles = p.tiles ? min(*p.ntiles, 1 << 20) : (p.M + MS * kTileM - 1) / (MS * kTileM);
  const int n_items = ntiles * nN;
  if ((int)blockIdx.x >= n_items) return;  // uniform for the CTA, before any TMEM is held
  if (warp == 3) tmem_alloc(tmem_slot, cols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp <= 1) {
    // ---- A producers
    if (c.a_tma) {
      if (warp == 0 && lane == 0) {
        Ring ra;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
          const GemmTile t = load_tile<MS>(p, it / nN);
          const int nsub = MS > 1 && t.mcount > kTileM ? MS : 1;
          for (int kt = 0; kt < nk; ++kt, ra.next(SA)) {
            const int s = ra.s;
            if (ra.reused && !wait_bar(&empty[s], ra.ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
            mbar_expect_tx(&full[s], (uint32_t)nsub * kSubBytes);
            for (int u = 0; u < nsub; ++u)
              tma_load_2d(smem + c.a + ((size_t)s * MS + u) * kSubBytes, &tmA, kt * kBK, t.m0 + u * kTileM,
                          &full[s]);
          }
        }
      }
    } else {
      // gathered rows: lane l of the 64 fetches 16-byte chunk l % 8 of rows l / 8 + 8 i (i < 16 MS), so that each
      // warp instruction covers four whole 128-byte rows; sub-tile u's rows land kSubBytes further on
      const int t64 = threadIdx.x, ch = t64 & 7, r0 = t64 >> 3;
      Ring ra;
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        const GemmTile t = load_tile<MS>(p, it / nN);
        int soff[16 * MS];  // element offset of the source row of rows r0 + 8 i, or -1
#pragma unroll
        for (int i = 0; i < 16 * MS; ++i) {
          const int r = r0 + 8 * i;
          soff[i] = -1;
          if (r < t.mcount) {
            int src = p.a_rows ? __ldg(p.a_rows + min(t.m0 + r, p.list_len - 1)) / p.a_div : t.m0 + r;
            src = min(max(src, 0), p.a_nrows - 1);
            soff[i] = (int)((int64_t)src * p.lda) + ch * 8;
          }
        }
        for (int kt = 0; kt < nk; ++kt, ra.next(SA)) {
          const int s = ra.s;
          if (ra.reused && !wait_bar(&empty[s], ra.ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          uint8_t* dst = smem + c.a + (size_t)s * MS * kSubBytes;
#pragma unroll
          for (int i = 0; i < 16 * MS; ++i) {
            // rows past the tile are never loaded nor stored: their stale values are harmless
            if (soff[i] < 0) continue;
            cp_async16(dst + sw128_chunk(r0 + 8 * i, ch), p.A + soff[i] + kt * kBK);
          }
          cp_async_arrive_noinc(&full[s]);
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
  } else if (warp == 2) {
    // ---- B producer: lane 0 issues the TMA tiles; all lanes copy scales when their rows are under 16 bytes
    constexpr int HB = BN / 2;
    Ring rr, rb;  // the raw ring (INT4) or the A + B ring (bf16 B); lane 0 issues
    int j = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++j) {
      const GemmTile t = load_tile<MS>(p, it / nN);
      const int nt = it % nN;
      const int y0 = (int)((int64_t)t.e * p.b_rows_per_e + nt * BN);
      if constexpr (INT4) {
        const int sb = j % NSC;
        int freed = 1;  // one lane waits, the warp follows its verdict
        if (lane == 0 && j >= NSC) freed = wait_bar(&sc_free[sb], ((j / NSC) - 1) & 1, abort_flag, p.err) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, freed, 0)) break;
        uint8_t* sdst = smem + c.sc + (size_t)sb * BN * c.sstride;
        if (c.s_tma) {
          if (lane == 0) {
            mbar_expect_tx(&sc_full[sb], (uint32_t)(BN * c.sstride));
            if (p.paired) tma_load_4d(sdst, &tmS, 0, nt * HB, 0, t.e, &sc_full[sb]);
            else tma_load_2d(sdst, &tmS, 0, y0, &sc_full[sb]);
          }
        } else {
          const int rb = c.sstride;  // 2, 4 or 8 bytes per row
          for (int r = lane; r < BN; r += 32) {
            if (!p.paired && nt * BN + r >= p.n_valid) continue;
            const int64_t row = b_row<BN>(p, t.e, nt, r);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(p.Bs) + row * rb;
            if (rb >= 4) {
              const uint32_t d = smem_u32(sdst + r * rb);
              if (rb == 8) asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(d), "l"(src) : "memory");
              else asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
            } else {
              *reinterpret_cast<uint16_t*>(sdst + r * rb) = __ldg(reinterpret_cast<const uint16_t*>(src));
            }
          }
          if (rb >= 4) cp_async_arrive_noinc(&sc_full[sb]);
          else mbar_arrive(&sc_full[sb]);
        }
        if (lane == 0) {
          const int RB = 32 * c.rk;
          for (int kt = 0; kt < nk; kt += c.rk, rr.next(SR)) {
            const int s = rr.s;
            if (rr.reused && !wait_bar(&freeR[s], rr.ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
            uint8_t* dst = smem + c.raw + (size_t)s * BN * RB;
            mbar_expect_tx(&fullR[s], (uint32_t)(BN * RB));
            if (p.paired) tma_load_4d(dst, &tmB, kt * 32, nt * HB, 0, t.e, &fullR[s]);
            else tma_load_2d(dst, &tmB, kt * 32, y0, &fullR[s]);
          }
        }
      } else {
        if (lane == 0) {
          for (int kt = 0; kt < nk; ++kt, rb.next(SA)) {
            const int s = rb.s;
            if (rb.reused && !wait_bar(&empty[s], rb.ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
            uint8_t* dst = smem + c.b + (size_t)s * BN * 128;
            mbar_expect_tx(&full[s], (uint32_t)(BN * 128));
            if (p.paired) tma_load_4d(dst, &tmB, kt * kBK, nt * HB, 0, t.e, &full[s]);
            else tma_load_2d(dst, &tmB, kt * kBK, y0, &full[s]);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 3) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kTileM, BN);
      Ring ra;
      int j = 0;
      bool ok = true;
      // shared-memory descriptors of stage 0; a stage, sub-tile or K step is an offset added to the start-address
      // field (bits [0,14) hold address >> 4, and every address here stays below 256 KB, so no carry leaves it)
      const uint64_t a_desc0 = sw128_desc(smem_u32(smem + c.a)), b_desc0 = sw128_desc(smem_u32(smem + c.b));
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++j) {
        const int ab = j % NB, use = j / NB;
        if (use >= 1 && !wait_bar(&acc_empty[ab], (use - 1) & 1, abort_flag, p.err)) break;
        fence_after_sync();
        // sub-tiles past the tile's rows are neither loaded nor multiplied (their epilogue warps skip them)
        const int nsub = MS > 1 && load_tile<MS>(p, it / nN).mcount > kTileM ? MS : 1;
        const uint32_t d = tmem + (uint32_t)(ab * MS * BN);
        for (int kt = 0; kt < nk; ++kt, ra.next(SA)) {
          const int s = ra.s;
          ok = wait_bar(&full[s], ra.ph, abort_flag, p.err);
          if (!ok) break;
          fence_after_sync();
          const uint64_t ad = a_desc0 + (uint64_t)((s * MS * kSubBytes) >> 4);
          const uint64_t bd = b_desc0 + (uint64_t)((s * BN * 128) >> 4);
#pragma unroll
          for (int u = 0; u < MS; ++u) {
            if (u >= nsub) break;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_bf16(d + (uint32_t)(u * BN), ad + (uint64_t)((u * kSubBytes + kk * 32) >> 4),
                       bd + (uint64_t)((kk * 32) >> 4), idesc, (kt | kk) != 0);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[ab]);
      }
    }
    __syncwarp();
  } else if (warp < kDeqWarp0) {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 of sub-tile (w - 4) / 4 = tile rows
    // 128 (w - 4) / 4 + 32 (w % 4) ..
    const int q = warp & 3, u = (warp - 4) >> 2;
    int j = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++j) {
      const GemmTile t = load_tile<MS>(p, it / nN);
      const int nt = it % nN, ab = j % NB;
      if (!wait_bar(&acc_full[ab], (j / NB) & 1, abort_flag, p.err)) break;
      __syncwarp();  // lane 0's arrive of the previous item can leave the warp split until here
      fence_after_sync();
      const int r = u * kTileM + q * 32 + lane;
      const bool valid = r < t.mcount;
      // warp-uniform: a lane quarter without rows is not read (a sub-tile past the rows was not computed)
      const bool any = u * kTileM + q * 32 < t.mcount;
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((ab * MS + u) * BN);
      int64_t orow = t.m0 + r;
      float rs = 1.f;
      if constexpr (EPI == EPI_SLOT) {
        orow = valid ? (int64_t)__ldg(p.out_rows + min(t.m0 + r, p.list_len - 1)) : 0;
        orow = min(max(orow, (int64_t)0), (int64_t)p.out_nrows - 1);
        rs = valid ? __ldg(p.row_scale + orow) : 0.f;
      } else {
        orow = min(orow, (int64_t)p.out_nrows - 1);
      }
      if (!any) {
        // nothing to store
      } else if constexpr (EPI == EPI_SILU_TILE || EPI == EPI_SILU_ROUND) {
        uint16_t* out = static_cast<uint16_t*>(p.out) + orow * p.ldo + nt * (BN / 2);
#pragma unroll 1
        for (int c0 = 0; c0 < BN / 2; c0 += 16) {
          float gv[16], uv[16];
          tmem_ld16x2(tb + c0, tb + BN / 2 + c0, gv, uv);
          if (valid) {
            uint32_t o[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              float a0, a1;
              if constexpr (EPI == EPI_SILU_TILE) {
                a0 = silu(gv[2 * jj]) * uv[2 * jj];
                a1 = silu(gv[2 * jj + 1]) * uv[2 * jj + 1];
              } else {
                a0 = silu(bf2f(f2bf(gv[2 * jj]))) * bf2f(f2bf(uv[2 * jj]));
                a1 = silu(bf2f(f2bf(gv[2 * jj + 1]))) * bf2f(f2bf(uv[2 * jj + 1]));
              }
              o[jj] = (uint32_t)f2bf(a0) | ((uint32_t)f2bf(a1) << 16);
            }
            reinterpret_cast<uint4*>(out + c0)[0] = make_uint4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<uint4*>(out + c0)[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      } else if constexpr (EPI == EPI_BF16) {
        uint16_t* out = static_cast<uint16_t*>(p.out) + orow * p.ldo + nt * BN;
        const int ncol = min(BN, p.n_valid - nt * BN);
#pragma unroll 1
        for (int c2 = 0; c2 < BN; c2 += 32) {
          float vv[2][16];
          tmem_ld16x2(tb + c2, tb + c2 + 16, vv[0], vv[1]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c0 = c2 + 16 * h;
            const float* v = vv[h];
            if (valid && c0 + 16 <= ncol) {
              uint32_t o[8];
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) o[jj] = (uint32_t)f2bf(v[2 * jj]) | ((uint32_t)f2bf(v[2 * jj + 1]) << 16);
              reinterpret_cast<uint4*>(out + c0)[0] = make_uint4(o[0], o[1], o[2], o[3]);
              reinterpret_cast<uint4*>(out + c0)[1] = make_uint4(o[4], o[5], o[6], o[7]);
            } else if (valid) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                if (c0 + jj < ncol) out[c0 + jj] = f2bf(v[jj]);
            }
          }
        }
      } else {  // EPI_F32, EPI_SLOT
        float* out = static_cast<float*>(p.out) + orow * p.ldo + nt * BN;
        const int ncol = min(BN, p.n_valid - nt * BN);
#pragma unroll 1
        for (int c2 = 0; c2 < BN; c2 += 32) {
          float vv[2][16];
          tmem_ld16x2(tb + c2, tb + c2 + 16, vv[0], vv[1]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c0 = c2 + 16 * h;
            float* v = vv[h];
            if constexpr (EPI == EPI_F32) {
              if (p.col_bias) {  // fp32 add after the dot product (the router's per-expert bias)
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                  v[jj] += (c0 + jj < ncol) ? __ldg(p.col_bias + nt * BN + c0 + jj) : 0.f;
              }
            }
            if (valid && c0 + 16 <= ncol) {
#pragma unroll
              for (int jj = 0; jj < 16; jj += 4)
                *reinterpret_cast<float4*>(out + c0 + jj) =
                    make_float4(v[jj] * rs, v[jj + 1] * rs, v[jj + 2] * rs, v[jj + 3] * rs);
            } else if (valid) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj)
                if (c0 + jj < ncol) out[c0 + jj] = v[jj] * rs;
            }
          }
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  } else if constexpr (INT4) {
    // ---- dequantization: job (row r, K half h) covers 32 nibbles of row r per step; thread td owns jobs
    // td + kDeqThreads * j
    constexpr int J = (BN * 2 + kDeqThreads - 1) / kDeqThreads;  // jobs per thread (2 at BN = 256, NDW = 8)
    const int td = threadIdx.x - kDeqWarp0 * 32;
    const int RB = 32 * c.rk, gsh = __ffs(p.G) - 1;  // G is 32, 64 or 128
    Ring rr, ra;  // the raw ring (advanced every rk k-steps) and the A + B ring
    int sub = 0, j = 0;  // k-step within the raw stage
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++j) {
      const int sbuf = j % NSC;
      if (!wait_bar(&sc_full[sbuf], (j / NSC) & 1, abort_flag, p.err)) break;
      __syncwarp();
      const uint8_t* scb = smem + c.sc + (size_t)sbuf * BN * c.sstride;
      // each job keeps four consecutive group scales in a register pair and reloads them when its group leaves the
      // window (every 4 k-steps at G = 64): the rows a warp converts are sstride bytes apart, so their scale reads
      // collide in a few banks, now once per window instead of once per k-step
      const bool wide = (c.sstride & 7) == 0;
      uint2 sreg[J];
      int sbase[J];
#pragma unroll
      for (int jj = 0; jj < J; ++jj) {
        sreg[jj] = make_uint2(0, 0);
        sbase[jj] = -(1 << 20);
      }
      for (int kt = 0; kt < nk; ++kt) {
        const int sr = rr.s, s = ra.s;
        ok = wait_bar(&fullR[sr], rr.ph, abort_flag, p.err);
        ok = ok && (!ra.reused || wait_bar(&empty[s], ra.ph ^ 1u, abort_flag, p.err));
        if (!ok) break;
        __syncwarp();  // lane 0's arrives of the previous step can leave the warp split until here
        const uint8_t* rawp = smem + c.raw + (size_t)sr * BN * RB + sub * 32;
        uint8_t* bdst = smem + c.b + (size_t)s * BN * 128;
#pragma unroll
        for (int jj = 0; jj < J; ++jj) {
          const int job = td + kDeqThreads * jj, r = job >> 1, h = job & 1;
          if (job >= BN * 2) continue;
          const uint4 w = *reinterpret_cast<const uint4*>(rawp + r * RB + h * 16);
          const int gi = (kt * kBK + h * 32) >> gsh;  // this job's group scale
          float sv;
          if (wide) {
            if (gi < sbase[jj] || gi >= sbase[jj] + 4) {
              sbase[jj] = gi & ~3;
              sreg[jj] = *reinterpret_cast<const uint2*>(scb + r * c.sstride + 2 * sbase[jj]);
            }
            const int k = gi - sbase[jj];
            const uint32_t pair = k < 2 ? sreg[jj].x : sreg[jj].y;
            sv = h2f((uint16_t)((k & 1) ? (pair >> 16) : (pair & 0xffffu)));
          } else {
            sv = h2f(*reinterpret_cast<const uint16_t*>(scb + r * c.sstride + 2 * gi));
          }
          const DqConst dc = dq_const(sv);
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int qq = 0; qq < 4; ++qq)
            *reinterpret_cast<uint4*>(bdst + sw128_chunk(r, h * 4 + qq)) = dequant8_bf16(ww[qq], dc);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (sub == c.rk - 1) mbar_arrive(&freeR[sr]);  // the raw stage's last k-step
          mbar_arrive(&full[s]);
        }
        if (++sub == c.rk) {
          sub = 0;
          rr.next(SR);
        }
        ra.next(SA);
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&sc_free[sbuf]);
    }
  }

  fence_before_sync();
  __syncthreads();
  if (warp == 3) {
    fence_after_sync();
    tmem_dealloc(tmem, cols);
  }
}

// ------------------------------------------------------------------ host side

static int dev_attr(cudaDeviceAttr a, int fallback) {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&v, a, dev) != cudaSuccess || v <= 0) v = fallback;
  return v;
}

// k-steps per raw INT4 box: the preference order below, or only the value the environment sets in
// MOE_B200_GEMM_RAW_KSTEPS (1, 2 or 4; read once per process). One k-step per box makes a box row 32 bytes, so
// the 16 rows a dequantisation warp reads fall on distinct banks; wider boxes mean fewer, larger TMA copies.
static int raw_ksteps_forced() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MOE_B200_GEMM_RAW_KSTEPS");
    const int k = e ? atoi(e) : 0;
    v = (k == 1 || k == 2 || k == 4) ? k : 0;
  }
  return v;
}

static bool pick_cfg(int bn, bool int4, int K, int G, int ms, GemmCfg* out) {
  static int optin = 0;
  if (!optin) optin = dev_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin, 227 * 1024);
  // first fit in order of preference: 3+ A + B stages, double-buffered scales (single ones only for double tiles,
  // whose A stages are twice as large), wide raw boxes, raw ring depth
  const int sa_c[] = {4, 3, 2}, sr_c[] = {3, 2};
  const int forced = int4 ? raw_ksteps_forced() : 0;
  const int rk_pref[] = {4, 2, 1}, rk_one[] = {forced, forced, forced};
  const int* rk_c = forced ? rk_one : rk_pref;
  const int n_nsc = int4 && ms > 1 ? 2 : 1;
  for (int sa : sa_c)
    for (int ni = 0; ni < n_nsc; ++ni)
      for (int ri = 0; ri < 3; ++ri)
        for (int sr : sr_c) {
          const int rk = rk_c[ri];
          const GemmCfg c = gemm_cfg(bn, int4, sa, sr, rk, K, G, ms, 2 - ni);
          if ((int)c.total <= optin && (sa >= 3 || rk == 1 || forced)) {
            *out = c;
            return true;
          }
          if (!int4) break;
        }
  return false;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point: the library links no driver library, so it
// loads on machines without a GPU driver (where only its host-side checks run).
static PFN_cuTensorMapEncodeTiled encode_fn() {
  static PFN_cuTensorMapEncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(f);
  });
  return fn;
}

// 4D tensor map of a paired operand: [E][2][half_rows][inner], halves half_rows rows apart, experts e_rows apart.
static bool make_map_pair(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t half_rows,
                          uint64_t experts, uint64_t e_rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                          bool swizzle128) {
  memset(m, 0, sizeof *m);
  const PFN_cuTensorMapEncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[4] = {inner, half_rows, 2, experts};
  const cuuint64_t strides[3] = {row_bytes, half_rows * row_bytes, (e_rows ? e_rows : 2 * half_rows) * row_bytes};
  const cuuint32_t box[4] = {box_inner, box_rows, 2, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE,
                                swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2D tensor map over a row-major [outer][inner] array; rows are row_bytes apart. Out-of-range box elements read 0.
static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  memset(m, 0, sizeof *m);
  const PFN_cuTensorMapEncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE,
                                swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, bool INT4, int EPI, int NDW = 8, int MS = 1>
static cudaError_t launch_t(const GemmParams& p, int max_tiles, bool pdl, cudaStream_t st) {
  GemmCfg c;
  if (!pick_cfg(BN, INT4, p.K, p.G, MS, &c)) return cudaErrorInvalidValue;
  c.a_tma = p.a_rows ? 0 : 1;
  CUtensorMap tmA, tmB, tmS;
  memset(&tmA, 0, sizeof tmA);
  memset(&tmB, 0, sizeof tmB);
  memset(&tmS, 0, sizeof tmS);
  if (c.a_tma && !make_map(&tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.A, (uint64_t)p.K, (uint64_t)p.a_nrows,
                           (uint64_t)p.lda * 2, kBK, kTileM, true))
    return cudaErrorInvalidValue;
  const uint32_t rows_box = p.paired ? BN / 2 : BN;
  const uint64_t hr = (uint64_t)p.pair_off, ne = (uint64_t)p.E, er = (uint64_t)p.b_rows_per_e;
  if (INT4) {
    const uint64_t rows = ne * er;
    const bool okb = p.paired ? make_map_pair(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.Bq, (uint64_t)p.K / 2, hr, ne, er,
                                              (uint64_t)p.K / 2, (uint32_t)(32 * c.rk), rows_box, false)
                              : make_map(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.Bq, (uint64_t)p.K / 2, rows,
                                         (uint64_t)p.K / 2, (uint32_t)(32 * c.rk), rows_box, false);
    if (!okb) return cudaErrorInvalidValue;
    if (c.s_tma) {
      const bool oks = p.paired ? make_map_pair(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT16, p.Bs, (uint64_t)c.ksc, hr, ne, er,
                                                (uint64_t)c.sstride, (uint32_t)c.ksc, rows_box, false)
                                : make_map(&tmS, CU_TENSOR_MAP_DATA_TYPE_UINT16, p.Bs, (uint64_t)c.ksc, rows,
                                           (uint64_t)c.sstride, (uint32_t)c.ksc, rows_box, false);
      if (!oks) return cudaErrorInvalidValue;
    }
  } else {
    const bool okb = p.paired ? make_map_pair(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.Bh, (uint64_t)p.K, hr, 1, 0,
                                              (uint64_t)p.K * 2, kBK, rows_box, true)
                              : make_map(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, p.Bh, (uint64_t)p.K,
                                         (uint64_t)p.n_valid, (uint64_t)p.K * 2, kBK, rows_box, true);
    if (!okb) return cudaErrorInvalidValue;
  }
  static SmemGrant granted;
  {
    cudaError_t e = grant_smem(reinterpret_cast<const void*>(moe_gemm_kernel<BN, INT4, EPI, NDW, MS>), c.total, 0,
                               granted);
    if (e != cudaSuccess) return e;
  }
  static int sms = 0;
  if (!sms) sms = dev_attr(cudaDevAttrMultiProcessorCount, 148);
  const int64_t items = (int64_t)max_tiles * (p.N / BN);
  if (items <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min<int64_t>(items, sms));
  cfg.blockDim = dim3(gemm_threads(NDW, MS));
  cfg.dynamicSmemBytes = c.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return launched(cudaLaunchKernelEx(&cfg, moe_gemm_kernel<BN, INT4, EPI, NDW, MS>, p, tmA, tmB, tmS, c));
}

// Dequantisation warps of the routed INT4 GEMMs: 8, or 16 when the environment sets MOE_B200_GEMM_DEQ_WARPS=16
// (read once per process).
static int deq_warps() {
  static int n = 0;
  if (!n) {
    const char* v = getenv("MOE_B200_GEMM_DEQ_WARPS");
    n = (v && atoi(v) == 16) ? 16 : 8;
  }
  return n;
}

template <int BN, bool INT4>
static cudaError_t launch_epi(const GemmParams& p, int epi, int max_tiles, bool pdl, cudaStream_t st, int ms) {
  if (ms == 2) {  // double tiles: the routed INT4 expert GEMMs at BN = 256
    if constexpr (BN == 256 && INT4) {
      const bool d16 = deq_warps() == 16;
      if (epi == EPI_SILU_TILE)
        return d16 ? launch_t<BN, true, EPI_SILU_TILE, 16, 2>(p, max_tiles, pdl, st)
                   : launch_t<BN, true, EPI_SILU_TILE, 8, 2>(p, max_tiles, pdl, st);
      if (epi == EPI_SLOT)
        return d16 ? launch_t<BN, true, EPI_SLOT, 16, 2>(p, max_tiles, pdl, st)
                   : launch_t<BN, true, EPI_SLOT, 8, 2>(p, max_tiles, pdl, st);
    }
    return cudaErrorInvalidValue;
  }
  switch (epi) {
    case EPI_F32: return launch_t<BN, INT4, EPI_F32>(p, max_tiles, pdl, st);
    case EPI_BF16: return launch_t<BN, INT4, EPI_BF16>(p, max_tiles, pdl, st);
    case EPI_SILU_TILE:
      if constexpr (BN == 256 && INT4)
        if (deq_warps() == 16) return launch_t<256, true, EPI_SILU_TILE, 16>(p, max_tiles, pdl, st);
      return launch_t<BN, INT4, EPI_SILU_TILE>(p, max_tiles, pdl, st);
    case EPI_SILU_ROUND: return launch_t<BN, INT4, EPI_SILU_ROUND>(p, max_tiles, pdl, st);
    case EPI_SLOT:
      if constexpr (BN == 256 && INT4)
        if (deq_warps() == 16) return launch_t<256, true, EPI_SLOT, 16>(p, max_tiles, pdl, st);
      return launch_t<BN, INT4, EPI_SLOT>(p, max_tiles, pdl, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm(const GemmParams& p, int epi, int bn, int tile_rows, bool int4, int max_tiles, bool pdl,
                        cudaStream_t st) {
  if (p.K <= 0 || p.K % kBK || p.N <= 0 || p.N % bn || p.lda % 8 || p.ldo % 8 || !p.A || !p.out) return cudaErrorInvalidValue;
  if (tile_rows != kTileM && tile_rows != 2 * kTileM) return cudaErrorInvalidValue;
  const int ms = tile_rows / kTileM;
  if (p.n_valid <= 0 || p.n_valid > p.N || (p.paired && p.n_valid != p.N)) return cudaErrorInvalidValue;
  const void* ptrs[5] = {p.A, p.Bh, p.Bq, p.Bs, p.out};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) % 16) return cudaErrorInvalidValue;  // 16-byte copies and stores
  if (p.a_nrows <= 0 || p.out_nrows <= 0 || p.E <= 0 || (p.a_rows && p.a_div <= 0)) return cudaErrorInvalidValue;
  if ((p.a_rows || p.out_rows) && p.list_len <= 0) return cudaErrorInvalidValue;
  if ((epi == EPI_SILU_TILE || epi == EPI_SILU_ROUND) != (p.paired != 0)) return cudaErrorInvalidValue;
  if (p.paired && p.N != 2 * p.pair_off) return cudaErrorInvalidValue;
  if (epi == EPI_SLOT && (!p.out_rows || !p.row_scale)) return cudaErrorInvalidValue;
  if (!p.tiles && p.M <= 0) return cudaErrorInvalidValue;
  if (p.tiles && !p.ntiles) return cudaErrorInvalidValue;
  if (int4) {
    if (!p.Bq || !p.Bs || (p.G != 32 && p.G != 64 && p.G != 128) || p.K % p.G) return cudaErrorInvalidValue;
  } else if (!p.Bh) {
    return cudaErrorInvalidValue;
  }
  switch (bn) {
    case 64:
      return int4 ? launch_epi<64, true>(p, epi, max_tiles, pdl, st, ms)
                  : launch_epi<64, false>(p, epi, max_tiles, pdl, st, ms);
    case 128:
      return int4 ? launch_epi<128, true>(p, epi, max_tiles, pdl, st, ms)
                  : launch_epi<128, false>(p, epi, max_tiles, pdl, st, ms);
    case 256:
      return int4 ? launch_epi<256, true>(p, epi, max_tiles, pdl, st, ms)
                  : launch_epi<256, false>(p, epi, max_tiles, pdl, st, ms);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace moe
