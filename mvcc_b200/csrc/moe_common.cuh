// moe_common.cuh -- shared device helpers, the workspace layout and launch-parameter structs of libmoe_b200.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/moe_block.h"

namespace moe {

// ------------------------------------------------------------------ scalar conversions

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
// Same formulas as the reference's silu/sigmoid (kernels.cuh:49-50), fast exp included.
__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid(float x) { return 1.f / (1.f + __expf(-x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Streaming 16-byte load that does not allocate in L1: weights are read exactly once per call.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// Sum over the 8 nibbles of u (k = 8w + b in nibble b) of (q - 8) * x[b], accumulated into acc in k order with
// fmaf, as int4_dot32 does (kernels.cuh:812-822). The nibble becomes a float through the 2^23 exponent trick:
// 0x4B000000 | q is exactly 2^23 + q, so subtracting 2^23 + 8 yields q - 8 exactly (no int->float conversion).
__device__ __forceinline__ float dot8_int4(uint32_t u, const float* x, float acc) {
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const float q = __uint_as_float(0x4B000000u | ((u >> (4 * b)) & 0xFu)) - 8388616.0f;
    acc = fmaf(q, x[b], acc);
  }
  return acc;
}

// ---- packed (f32x2) position-scaled int4 dot, the decode kernels' inner loop.
//
// A nibble q at bit position 4p of a word, OR-ed into 0x4B000000 (one LOP3), is the float 2^23 + q * 2^(4p),
// exactly. Adding -(2^23 + 8 * 2^(4p)) (the float with bits 0xCB000000 | 8 << 4p) leaves (q - 8) * 2^(4p),
// exactly. Nibbles 0..4 of a word sit at p = 0..4 in place; nibbles 5..7 reach p = 2..4 after one 12-bit shift.
// The products with x accumulate into five position accumulators (factor 2^(4p)), folded with exact power-of-two
// factors at the end. Pairs of nibbles go through sm_100a's packed add.rn.f32x2 / fma.rn.f32x2, so one word of 8
// nibbles costs 1 shift + 8 LOP3 + 4 packed adds + 4 packed FMAs.
typedef unsigned long long u64;

struct Nib8Acc {
  u64 a01, a23, a45, a67;  // (p0, p1), (p2, p3), (p4, p2), (p3, p4)
};
struct Nib8Magic {
  u64 m01, m23, m45, m67;
};
__device__ __forceinline__ Nib8Magic nib8_magic() {
  Nib8Magic m;
  m.m01 = 0xCB000080CB000008ull;  // hi: -(2^23 + 128)   lo: -(2^23 + 8)
  m.m23 = 0xCB008000CB000800ull;  // hi: -(2^23 + 32768) lo: -(2^23 + 2048)
  m.m45 = 0xCB000800CB080000ull;  // hi: p2              lo: -(2^23 + 524288)
  m.m67 = 0xCB080000CB008000ull;  // hi: p4              lo: p3
  return m;
}
__device__ __forceinline__ void nib8_zero(Nib8Acc& A) { A.a01 = A.a23 = A.a45 = A.a67 = 0ull; }

// A += (q_b - 8) * 2^(4p_b) * x_b for the 8 nibbles of u; x01 = (x0, x1), ... packed float pairs.
__device__ __forceinline__ void nib8x2(uint32_t u, u64 x01, u64 x23, u64 x45, u64 x67, const Nib8Magic& M,
                                       Nib8Acc& A) {
  asm("{\n\t"
      ".reg .b32 v, f0, f1, f2, f3, f4, f5, f6, f7;\n\t"
      ".reg .b64 p01, p23, p45, p67;\n\t"
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
      "fma.rn.f32x2 %0, p01, %5, %0;\n\t"
      "fma.rn.f32x2 %1, p23, %6, %1;\n\t"
      "fma.rn.f32x2 %2, p45, %7, %2;\n\t"
      "fma.rn.f32x2 %3, p67, %8, %3;\n\t"
      "}"
      : "+l"(A.a01), "+l"(A.a23), "+l"(A.a45), "+l"(A.a67)
      : "r"(u), "l"(x01), "l"(x23), "l"(x45), "l"(x67), "l"(M.m01), "l"(M.m23), "l"(M.m45), "l"(M.m67));
}

__device__ __forceinline__ float lo_f(u64 v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_f(u64 v) { return __uint_as_float((uint32_t)(v >> 32)); }

// sum over positions p of acc_p * 2^(-4p): the (q - 8) . x dot of the words accumulated into A.
__device__ __forceinline__ float nib8_fold(const Nib8Acc& A) {
  const float p2 = lo_f(A.a23) + hi_f(A.a45), p3 = hi_f(A.a23) + lo_f(A.a67), p4 = lo_f(A.a45) + hi_f(A.a67);
  float d = fmaf(p4, 1.0f / 65536.0f, p3 * (1.0f / 4096.0f));
  d = fmaf(p2, 1.0f / 256.0f, d);
  d = fmaf(hi_f(A.a01), 1.0f / 16.0f, d);
  return d + lo_f(A.a01);
}

// Two packed float pairs from 16 bytes of shared memory.
__device__ __forceinline__ void lds_pairs(const void* p, u64& a, u64& b) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(s));
}

// ------------------------------------------------------------------ workspace layout

// Offsets (bytes) of the sections of the caller-owned workspace; every section is 256-byte aligned.
struct WsLayout {
  size_t ticket, err, gbar, logits, idx, wts, gate, nuniq, uniq, uoff, upairs, inter, sinter, routed, sout;
  // prefill sections (present when maxT >= kPrefillMinT): per-expert pair bitmaps and their word prefixes, expert
  // counts and offsets, the grouped-GEMM tile list, the pairs sorted by expert, the per-pair down partials
  size_t bits, wpre, counts, offsets, tiles, ntiles, tiles2, ntiles2, sorted, slot;
  size_t total;
  int maxT, nwp, max_tiles, max_tiles2;
};

// The reference switches moe() to its sort + tile path at T >= 8 (qwen.cu:347); so does this library.
constexpr int kPrefillMinT = 8;

// Rows (sorted pairs of one expert) per grouped-GEMM tile, and the upper bound of the tiles for P pairs over E
// experts: sum_e ceil(n_e / rows). Two lists are built: tiles of kTileRows rows and double tiles of 2 kTileRows
// rows (the expert GEMMs that run two 128-row sub-tiles against one dequantised B stage).
constexpr int kTileRows = 128;
__host__ __device__ inline int prefill_max_tiles(int P, int E, int rows = kTileRows) {
  return P / rows + (E < P ? E : P) + 1;
}

// Launch accounting behind moe_stats_get: `launched(e)` passes a launch's status through and counts the launch when
// it succeeded (the counters live in moe_api.cu).
void note_launches(uint64_t n);
void note_block_call();
void note_pack_bytes(uint64_t n);
inline cudaError_t launched(cudaError_t e) {
  if (e == cudaSuccess) note_launches(1);
  return e;
}

// Raises a kernel's dynamic shared-memory limit on the current device to at least `bytes`, and to `floor_bytes` at
// once so that later, larger requests rarely need another call; after a kernel's first launch on a device, its later
// launches there (including those inside CUDA-graph capture) make no attribute call. Kernel attributes belong to
// each device's context, so what was granted is recorded per device: a process that drives several GPUs raises each
// kernel's limit on each of them. One SmemGrant per kernel instantiation, as a function-local static (zero at start).
struct SmemGrant {
  static constexpr int kDevices = 64;
  std::atomic<size_t> dev[kDevices];
};
inline cudaError_t grant_smem(const void* kern, size_t bytes, size_t floor_bytes, SmemGrant& g) {
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return e;
  const bool kept = d >= 0 && d < SmemGrant::kDevices;  // devices past the table are raised on every launch
  if (kept && bytes <= g.dev[d].load(std::memory_order_relaxed)) return cudaSuccess;
  const size_t want = bytes > floor_bytes ? bytes : floor_bytes;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
  if (e == cudaSuccess && kept) g.dev[d].store(want, std::memory_order_relaxed);
  return e;
}

// Records the cudaEvent_t `ev` (nullable) on `s`; inside stream capture the record becomes a graph node that
// timestamps every replay.
inline cudaError_t record_event(void* ev, cudaStream_t s) {
  if (!ev) return cudaSuccess;
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &st);
  if (e != cudaSuccess) return e;
  if (st == cudaStreamCaptureStatusActive)
    return cudaEventRecordWithFlags(static_cast<cudaEvent_t>(ev), s, cudaEventRecordExternal);
  return cudaEventRecord(static_cast<cudaEvent_t>(ev), s);
}

__host__ __device__ inline size_t ws_align(size_t x) { return (x + 255) & ~(size_t)255; }

__host__ __device__ inline WsLayout ws_layout(int H, int E, int TOPK, int I, int Is, int maxT) {
  WsLayout L;
  size_t o = 0;
  const size_t pairs = (size_t)maxT * TOPK;
  L.maxT = maxT;
  L.ticket = o; o = ws_align(o + 16 * sizeof(uint32_t));
  L.err = o;    o = ws_align(o + sizeof(uint32_t));
  L.gbar = o;   o = ws_align(o + sizeof(unsigned long long));  // fixed offset: shared by every T
  L.logits = o; o = ws_align(o + sizeof(float) * (size_t)maxT * E);
  L.idx = o;    o = ws_align(o + sizeof(int32_t) * pairs);
  L.wts = o;    o = ws_align(o + sizeof(float) * pairs);
  L.gate = o;   o = ws_align(o + sizeof(float) * (size_t)maxT);
  L.nuniq = o;  o = ws_align(o + sizeof(int32_t));
  L.uniq = o;   o = ws_align(o + sizeof(int32_t) * (size_t)E);
  L.uoff = o;   o = ws_align(o + sizeof(int32_t) * ((size_t)E + 1));
  L.upairs = o; o = ws_align(o + sizeof(int32_t) * pairs);
  L.inter = o;  o = ws_align(o + sizeof(uint16_t) * pairs * I);
  L.sinter = o; o = ws_align(o + sizeof(uint16_t) * (size_t)maxT * Is);
  L.routed = o; o = ws_align(o + sizeof(float) * (size_t)maxT * H);
  L.sout = o;   o = ws_align(o + sizeof(uint16_t) * (size_t)maxT * H);
  L.nwp = (int)((pairs + 31) / 32);
  L.max_tiles = prefill_max_tiles((int)pairs, E);
  L.max_tiles2 = prefill_max_tiles((int)pairs, E, 2 * kTileRows);
  L.bits = L.wpre = L.counts = L.offsets = L.tiles = L.ntiles = L.tiles2 = L.ntiles2 = L.sorted = L.slot = o;
  if (maxT >= kPrefillMinT) {
    L.bits = o;    o = ws_align(o + sizeof(uint32_t) * (size_t)E * L.nwp);
    L.wpre = o;    o = ws_align(o + sizeof(uint32_t) * (size_t)E * L.nwp);
    L.counts = o;  o = ws_align(o + sizeof(int32_t) * (size_t)E);
    L.offsets = o; o = ws_align(o + sizeof(int32_t) * ((size_t)E + 1));
    L.tiles = o;   o = ws_align(o + 16 * (size_t)L.max_tiles);
    L.ntiles = o;  o = ws_align(o + sizeof(int32_t));
    L.tiles2 = o;  o = ws_align(o + 16 * (size_t)L.max_tiles2);
    L.ntiles2 = o; o = ws_align(o + sizeof(int32_t));
    L.sorted = o;  o = ws_align(o + sizeof(int32_t) * pairs);
    L.slot = o;    o = ws_align(o + sizeof(float) * pairs * H);
  }
  L.total = o;
  return L;
}

// Ticket slots (self-resetting counters for the last-block pattern).
enum { TICKET_ROUTE = 0, TICKET_COMBINE = 1, TICKET_SCAN = 2 };

// Device-side view of one call: weights, geometry and workspace pointers.
struct BlockArgs {
  moe_layer_weights w;
  int T;
  // activations
  float* hidden;            // [T,H] fp32 in/out (nullable for partial entry points)
  const uint16_t* attn_out; // [T,H] bf16
  uint16_t* normed;         // [T,H] bf16
  const uint16_t* next_rms1;
  // workspace sections
  uint32_t* ticket;
  uint32_t* err;
  float* logits;
  int32_t* idx;
  float* wts;
  float* gate;
  int32_t* nuniq;
  int32_t* uniq;
  int32_t* uoff;
  int32_t* upairs;
  uint16_t* inter;
  uint16_t* sinter;
  float* routed;
  uint16_t* sout;
  // prefill sections (null below kPrefillMinT tokens)
  uint32_t* bits;
  uint32_t* wpre;
  int32_t* counts;
  int32_t* offsets;
  void* tiles;
  int32_t* ntiles;
  void* tiles2;  // double tiles (2 kTileRows rows)
  int32_t* ntiles2;
  int32_t* sorted;
  float* slot;
  int nwp, max_tiles, max_tiles2;
  // row stride (elements) of `normed` as the routed gate/up operand; 0 = H (expert-parallel records are wider)
  int xstride;
  // expert-parallel combine (null otherwise): routed[t] = sum over ranks d < ep_world, ascending, with
  // ep_pos[t * ep_world + d] >= 0 of the returned bf16 partial row ep_ret[ep_pos[...]], in fp32
  const int32_t* ep_pos;
  const uint16_t* ep_ret;
  int ep_world;
  // expert-parallel experts stage (null otherwise): the routed rows of the records, rounded to bf16, go here
  // instead of into routed
  uint16_t* routed16;
};

}  // namespace moe
