// moe_gemm.cu -- warp-specialized tcgen05 tile GEMM for the prefill path: the dense router / shared-expert
// GEMMs (dense(), qwen.cu:298-319) and the grouped INT4 expert GEMMs (moe_gate_up_tile_kernel,
// moe_down_tile_kernel, kernels.cuh:942-1057).
//
// One CTA computes a 128 x BN tile of D = A . B^T with K-steps of 64 through a ring of shared-memory stages:
//   warp 0      A producer: gathers the tile's 128 A rows (one per token or (token, slot) pair) with cp.async
//               into the 128-byte-swizzled K-major layout, arrives on fullA[s] when its copies land;
//   warp 1      B producer: bf16 B rows straight into the swizzled layout, or INT4 rows (32 bytes per row and
//               step) into a raw staging buffer; arrives on fullB[s];
//   warp 3      INT4 only: copies the tile's fp16 group scales (all of K) once;
//   warps 4-7   INT4 only: dequantize raw[s] into bf16 B[s] exactly as dequant32_bf16 does
//               (kernels.cuh:925-940: bf16((q - 8) * scale), one rounding), fence the writes to the async proxy
//               and arrive on deq[s]; after the main loop the same warps run the epilogue from TMEM;
//   warp 2      allocates the TMEM accumulator (BN fp32 columns x 128 lanes); one lane issues the four
//               tcgen05.mma (M=128, N=BN, K=16) of each stage and commits them to empty[s] (which frees the
//               stage for the producers) and, after the last stage, to acc_full.
// Every mbarrier wait is bounded: after kWaitNs the waiting thread records MOE_ERR_TIMEOUT in the error word,
// raises the CTA's abort flag (other waits poll it) and leaves its loop; the CTA then drains its copies, frees
// TMEM and exits.
//
// Exact dequantization without a conversion instruction per nibble: a nibble q at bit position 4p of a word,
// OR-ed into 0x4B000000, is the float 2^23 + q * 2^(4p); subtracting 2^23 + 8 * 2^(4p) leaves (q - 8) * 2^(4p)
// exactly, and multiplying by scale * 2^(-4p) gives (q - 8) * scale exactly (at most 15 significant bits); one
// cvt.rn.bf16x2.f32 rounds two such values to bf16, the reference's single rounding.
#include <algorithm>

#include "moe_common.cuh"
#include "moe_gemm.h"
#include "moe_tc.cuh"

namespace moe {

using namespace tc;

constexpr int kBM = 128, kBK = 64, kGThreads = 256;
constexpr unsigned long long kWaitNs = 2000000000ull;  // 2 s: far beyond any tile's main loop

struct GemmSmem {
  size_t a, b, raw, sc, bar, total;
};

__host__ __device__ inline size_t g_align(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline GemmSmem gemm_smem(int bn, bool int4, int stages, int K, int G) {
  GemmSmem L;
  size_t o = 0;
  L.a = o;   o += (size_t)stages * kBM * 128;  // 16 KiB per stage; every stage 1024-byte aligned
  L.b = o;   o += (size_t)stages * bn * 128;
  L.raw = o; if (int4) o += (size_t)stages * bn * 32;
  L.sc = o;  if (int4) o = g_align(o + (size_t)bn * (K / G) * 2, 16);
  L.bar = g_align(o, 8);
  o = L.bar + 8 * (4 * (size_t)stages + 4);
  L.total = o + 1024;  // the dynamic base is aligned up to 1024 bytes at run time
  return L;
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

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity; bounded in time (kWaitNs from the first miss), and gives up early when
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
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitNs) {
        *abort_flag = 1;
        if (err) atomicOr(err, (uint32_t)MOE_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// 8 nibbles of u (k = 8w .. 8w + 7) times the scale -> 8 bf16 (one 16-byte chunk), exact products, RNE.
// sc01 = (s, s/16), sc23 = (s/256, s/4096), sc45 = (s/65536, s/256), sc67 = (s/4096, s/65536).
__device__ __forceinline__ uint4 dequant8_bf16(uint32_t u, u64 sc01, u64 sc23, u64 sc45, u64 sc67,
                                               const Nib8Magic& M) {
  uint4 o;
  asm("{\n\t"
      ".reg .b32 v, f0, f1, f2, f3, f4, f5, f6, f7;\n\t"
      ".reg .b64 p01, p23, p45, p67;\n\t"
      ".reg .f32 a0, a1, a2, a3, a4, a5, a6, a7;\n\t"
      "shr.b32 v, %4, 12;\n\t"
      "lop3.b32 f0, %4, 0xF, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f1, %4, 0xF0, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f2, %4, 0xF00, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f3, %4, 0xF000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f4, %4, 0xF0000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f5, v, 0xF00, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f6, v, 0xF000, 0x4B000000, 0xEA;\n\t"
      "lop3.b32 f7, v, 0xF0000, 0x4B000000, 0xEA;\n\t"
      "mov.b64 p01, {f0, f1};\n\t"
      "mov.b64 p23, {f2, f3};\n\t"
      "mov.b64 p45, {f4, f5};\n\t"
      "mov.b64 p67, {f6, f7};\n\t"
      "add.rn.f32x2 p01, p01, %9;\n\t"
      "add.rn.f32x2 p23, p23, %10;\n\t"
      "add.rn.f32x2 p45, p45, %11;\n\t"
      "add.rn.f32x2 p67, p67, %12;\n\t"
      "mul.rn.f32x2 p01, p01, %5;\n\t"
      "mul.rn.f32x2 p23, p23, %6;\n\t"
      "mul.rn.f32x2 p45, p45, %7;\n\t"
      "mul.rn.f32x2 p67, p67, %8;\n\t"
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
      : "r"(u), "l"(sc01), "l"(sc23), "l"(sc45), "l"(sc67), "l"(M.m01), "l"(M.m23), "l"(M.m45), "l"(M.m67));
  return o;
}

__device__ __forceinline__ u64 pack2f(float lo, float hi) {
  return ((u64)__float_as_uint(hi) << 32) | (u64)__float_as_uint(lo);
}

template <int BN>
__device__ __forceinline__ int64_t b_row(const GemmParams& p, int e, int nt, int r) {
  int row;
  if (p.paired) row = r < BN / 2 ? nt * (BN / 2) + r : p.pair_off + nt * (BN / 2) + (r - BN / 2);
  else row = nt * BN + r;
  return (int64_t)e * p.b_rows_per_e + row;
}

template <int BN, bool INT4, int EPI>
__global__ void __launch_bounds__(kGThreads, 1) moe_gemm_kernel(const GemmParams p, int stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int S = stages;
  const GemmSmem L = gemm_smem(BN, INT4, S, p.K, p.G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nN = p.N / BN;
  const int tix = blockIdx.x / nN, nt = blockIdx.x - tix * nN;
  GemmTile t;
  if (p.tiles) {
    if (tix >= *p.ntiles) return;
    t = p.tiles[tix];
  } else {
    t.e = 0;
    t.m0 = tix * kBM;
    t.mcount = p.M - t.m0;
  }
  t.e = min(max(t.e, 0), p.E - 1);
  t.mcount = min(t.mcount, kBM);
  if (t.mcount <= 0 || t.m0 < 0) return;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar);
  uint64_t* fullA = bars;
  uint64_t* fullB = bars + S;
  uint64_t* deq = bars + 2 * S;
  uint64_t* empty = bars + 3 * S;
  uint64_t* sc_full = bars + 4 * S;
  uint64_t* acc_full = bars + 4 * S + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * S + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 4 * S + 3);
  constexpr uint32_t kCols = BN < 32 ? 32 : BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&fullA[s], 32);
      mbar_init(&fullB[s], 32);
      mbar_init(&deq[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(sc_full, 32);
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 2) tmem_alloc(tmem_slot, kCols);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int nk = p.K / kBK;
  const int ksc = p.K / p.G;  // scales per B row

  if (warp == 0) {
    // ---- A producer: 4 rows per lane, 8 chunks each per stage
    const uint16_t* arow[4];
    bool aval[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = lane + 32 * i;
      aval[i] = r < t.mcount;
      int src = 0;
      if (aval[i]) {
        src = p.a_rows ? __ldg(p.a_rows + min(t.m0 + r, p.list_len - 1)) / p.a_div : t.m0 + r;
        src = min(max(src, 0), p.a_nrows - 1);
      }
      arow[i] = p.A + (int64_t)src * p.lda;
    }
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % S;
      if (kt >= S && !wait_bar(&empty[s], ((kt / S) - 1) & 1, abort_flag, p.err)) break;
      uint8_t* dst = smem + L.a + (size_t)s * kBM * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = lane + 32 * i;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          cp_async16_zfill(dst + sw128_chunk(r, j), arow[i] + kt * kBK + j * 8, aval[i]);
      }
      cp_async_arrive_noinc(&fullA[s]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 1) {
    // ---- B producer
    constexpr int RPL = BN / 32;  // rows per lane
    int64_t brow[RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) brow[i] = b_row<BN>(p, t.e, nt, lane + 32 * i);
    for (int kt = 0; kt < nk; ++kt) {
      const int s = kt % S;
      if (kt >= S && !wait_bar(&empty[s], ((kt / S) - 1) & 1, abort_flag, p.err)) break;
      if constexpr (INT4) {
        uint8_t* dst = smem + L.raw + (size_t)s * BN * 32;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int r = lane + 32 * i;
          const bool ok = p.paired || nt * BN + r < p.n_valid;
          const uint8_t* src = ok ? p.Bq + brow[i] * (p.K / 2) + kt * 32 : p.Bq;
          cp_async16_zfill(dst + r * 32, src, ok);
          cp_async16_zfill(dst + r * 32 + 16, src + (ok ? 16 : 0), ok);
        }
      } else {
        uint8_t* dst = smem + L.b + (size_t)s * BN * 128;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int r = lane + 32 * i;
          const bool ok = p.paired || nt * BN + r < p.n_valid;
          const uint16_t* src = ok ? p.Bh + brow[i] * p.K + kt * kBK : p.Bh;
#pragma unroll
          for (int j = 0; j < 8; ++j) cp_async16_zfill(dst + sw128_chunk(r, j), src + (ok ? j * 8 : 0), ok);
        }
      }
      cp_async_arrive_noinc(&fullB[s]);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 2) {
    // ---- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
      bool ok = true;
      for (int kt = 0; kt < nk && ok; ++kt) {
        const int s = kt % S;
        const uint32_t par = (kt / S) & 1;
        ok = wait_bar(&fullA[s], par, abort_flag, p.err) &&
             wait_bar(INT4 ? &deq[s] : &fullB[s], par, abort_flag, p.err);
        if (!ok) break;
        fence_after_sync();
        const uint32_t a_addr = smem_u32(smem + L.a + (size_t)s * kBM * 128);
        const uint32_t b_addr = smem_u32(smem + L.b + (size_t)s * BN * 128);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_bf16(tmem, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), idesc, (kt | kk) != 0);
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(acc_full);
    }
    __syncwarp();
  } else if (warp == 3) {
    // ---- scale loader (INT4): all K/G scales of the tile's BN rows
    if constexpr (INT4) {
      uint16_t* sc = reinterpret_cast<uint16_t*>(smem + L.sc);
      for (int r = lane; r < BN; r += 32) {
        if (!p.paired && nt * BN + r >= p.n_valid) continue;  // zero rows: any scale gives 0
        const uint16_t* src = p.Bs + b_row<BN>(p, t.e, nt, r) * ksc;
        if ((ksc & 7) == 0) {
          for (int g = 0; g < ksc; g += 8)
            *reinterpret_cast<uint4*>(sc + r * ksc + g) = __ldg(reinterpret_cast<const uint4*>(src + g));
        } else {
          for (int g = 0; g < ksc; ++g) sc[r * ksc + g] = __ldg(src + g);
        }
      }
      mbar_arrive(sc_full);
    }
  }

  if (warp >= 4) {
    const int td = threadIdx.x - 128;
    if constexpr (INT4) {
      // ---- dequantization
      const Nib8Magic M = nib8_magic();
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(smem + L.sc);
      bool ok = wait_bar(sc_full, 0, abort_flag, p.err);
      for (int kt = 0; kt < nk && ok; ++kt) {
        const int s = kt % S;
        if (!wait_bar(&fullB[s], (kt / S) & 1, abort_flag, p.err)) break;
        const uint8_t* raw = smem + L.raw + (size_t)s * BN * 32;
        uint8_t* bdst = smem + L.b + (size_t)s * BN * 128;
#pragma unroll
        for (int jb = 0; jb < (BN * 2) / 128; ++jb) {
          const int job = td + 128 * jb;
          const int r = job >> 1, h = job & 1;
          const uint4 w = *reinterpret_cast<const uint4*>(raw + r * 32 + h * 16);
          const float sv = h2f(sc[r * ksc + (kt * kBK + h * 32) / p.G]);
          const u64 s01 = pack2f(sv, sv * 0.0625f), s23 = pack2f(sv * (1.f / 256.f), sv * (1.f / 4096.f));
          const u64 s45 = pack2f(sv * (1.f / 65536.f), sv * (1.f / 256.f));
          const u64 s67 = pack2f(sv * (1.f / 4096.f), sv * (1.f / 65536.f));
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(bdst + sw128_chunk(r, h * 4 + q)) = dequant8_bf16(ww[q], s01, s23, s45, s67, M);
        }
        fence_proxy_async_smem();
        mbar_arrive(&deq[s]);
      }
    }
    // ---- epilogue: warp (w % 4) reads TMEM lanes 32 (w % 4) .. + 31 = tile rows
    if (wait_bar(acc_full, 0, abort_flag, p.err)) {
      fence_after_sync();
      const int q = warp & 3, r = q * 32 + lane;
      const bool valid = r < t.mcount;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16);
      int64_t orow = t.m0 + r;
      float rs = 1.f;
      if constexpr (EPI == EPI_SLOT) {
        orow = valid ? (int64_t)__ldg(p.out_rows + min(t.m0 + r, p.list_len - 1)) : 0;
        orow = min(max(orow, (int64_t)0), (int64_t)p.out_nrows - 1);
        rs = valid ? __ldg(p.row_scale + orow) : 0.f;
      } else {
        orow = min(orow, (int64_t)p.out_nrows - 1);
      }
      if constexpr (EPI == EPI_SILU_TILE || EPI == EPI_SILU_ROUND) {
        uint16_t* out = static_cast<uint16_t*>(p.out) + orow * p.ldo + nt * (BN / 2);
#pragma unroll 1
        for (int c0 = 0; c0 < BN / 2; c0 += 16) {
          float g[16], u[16];
          tmem_ld16(tbase + c0, g);
          tmem_ld16(tbase + BN / 2 + c0, u);
          if (valid) {
            uint32_t o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float a0, a1;
              if constexpr (EPI == EPI_SILU_TILE) {
                a0 = silu(g[2 * j]) * u[2 * j];
                a1 = silu(g[2 * j + 1]) * u[2 * j + 1];
              } else {
                a0 = silu(bf2f(f2bf(g[2 * j]))) * bf2f(f2bf(u[2 * j]));
                a1 = silu(bf2f(f2bf(g[2 * j + 1]))) * bf2f(f2bf(u[2 * j + 1]));
              }
              o[j] = (uint32_t)f2bf(a0) | ((uint32_t)f2bf(a1) << 16);
            }
            reinterpret_cast<uint4*>(out + c0)[0] = make_uint4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<uint4*>(out + c0)[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      } else if constexpr (EPI == EPI_BF16) {
        uint16_t* out = static_cast<uint16_t*>(p.out) + orow * p.ldo + nt * BN;
        const int ncol = min(BN, p.n_valid - nt * BN);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(tbase + c0, v);
          if (valid && c0 + 16 > ncol) {
            for (int j = 0; j < 16 && c0 + j < ncol; ++j) out[c0 + j] = f2bf(v[j]);
          } else if (valid) {
            uint32_t o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = (uint32_t)f2bf(v[2 * j]) | ((uint32_t)f2bf(v[2 * j + 1]) << 16);
            reinterpret_cast<uint4*>(out + c0)[0] = make_uint4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<uint4*>(out + c0)[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      } else {  // EPI_F32, EPI_SLOT
        float* out = static_cast<float*>(p.out) + orow * p.ldo + nt * BN;
        const int ncol = min(BN, p.n_valid - nt * BN);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(tbase + c0, v);
          if (valid && c0 + 16 <= ncol) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4*>(out + c0 + j) = make_float4(v[j] * rs, v[j + 1] * rs, v[j + 2] * rs,
                                                                     v[j + 3] * rs);
          } else if (valid) {
            for (int j = 0; j < 16 && c0 + j < ncol; ++j) out[c0 + j] = v[j] * rs;
          }
        }
      }
    }
  }

  fence_before_sync();
  __syncthreads();
  if (warp == 2) {
    fence_after_sync();
    tmem_dealloc(tmem, kCols);
  }
}

// ------------------------------------------------------------------ host side

static int smem_optin() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (n <= 0) n = 227 * 1024;
  }
  return n;
}

static int pick_stages(int bn, bool int4, int K, int G) {
  for (int s = 4; s >= 2; --s)
    if ((int)gemm_smem(bn, int4, s, K, G).total <= smem_optin()) return s;
  return 0;
}

size_t gemm_smem_bytes(int bn, bool int4, int K, int G) {
  const int s = pick_stages(bn, int4, K, G);
  return s ? gemm_smem(bn, int4, s, K, G).total : 0;
}

template <int BN, bool INT4, int EPI>
static cudaError_t launch_t(const GemmParams& p, int max_tiles, cudaStream_t st) {
  const int S = pick_stages(BN, INT4, p.K, p.G);
  if (!S) return cudaErrorInvalidValue;
  const size_t smem = gemm_smem(BN, INT4, S, p.K, p.G).total;
  static size_t granted = 0;
  if (smem > granted) {
    cudaError_t e = cudaFuncSetAttribute(moe_gemm_kernel<BN, INT4, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    granted = smem;
  }
  const int64_t grid = (int64_t)max_tiles * (p.N / BN);
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  moe_gemm_kernel<BN, INT4, EPI><<<(unsigned)grid, kGThreads, smem, st>>>(p, S);
  return cudaGetLastError();
}

template <int BN, bool INT4>
static cudaError_t launch_epi(const GemmParams& p, int epi, int max_tiles, cudaStream_t st) {
  switch (epi) {
    case EPI_F32: return launch_t<BN, INT4, EPI_F32>(p, max_tiles, st);
    case EPI_BF16: return launch_t<BN, INT4, EPI_BF16>(p, max_tiles, st);
    case EPI_SILU_TILE: return launch_t<BN, INT4, EPI_SILU_TILE>(p, max_tiles, st);
    case EPI_SILU_ROUND: return launch_t<BN, INT4, EPI_SILU_ROUND>(p, max_tiles, st);
    case EPI_SLOT: return launch_t<BN, INT4, EPI_SLOT>(p, max_tiles, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemm(const GemmParams& p, int epi, int bn, bool int4, int max_tiles, cudaStream_t st) {
  if (p.K <= 0 || p.K % kBK || p.N <= 0 || p.N % bn || p.lda % 8 || p.ldo % 8 || !p.A || !p.out) return cudaErrorInvalidValue;
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
    case 64: return int4 ? launch_epi<64, true>(p, epi, max_tiles, st) : launch_epi<64, false>(p, epi, max_tiles, st);
    case 128: return int4 ? launch_epi<128, true>(p, epi, max_tiles, st) : launch_epi<128, false>(p, epi, max_tiles, st);
    case 256: return int4 ? launch_epi<256, true>(p, epi, max_tiles, st) : launch_epi<256, false>(p, epi, max_tiles, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace moe
