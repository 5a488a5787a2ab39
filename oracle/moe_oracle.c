/* moe_oracle.c -- scalar CPU restatement of the Qwen3.5-MoE block of mvcc's examples/qwen.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE. This library is the parity checker for the CUDA path in
 * mvcc_b200/csrc. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm load it;
 * the product path never calls into it and has no CPU fallback.
 *
 * Each function restates one reference kernel of examples/qwen/kernels.cuh (or one host step of
 * examples/qwen/qwen.cu) and cites it. The rounding points are the reference's:
 *   - normed activations x are bf16 (kernels.cuh:112, f2bf after rms * w);
 *   - router logits are fp32 (qwen.cu:432-433 dense<float>), routing weights fp32 via exp (kernels.cuh:803-807);
 *   - routed `inter` is rounded to bf16 after silu(g)*u in fp32 (kernels.cuh:859);
 *   - shared-expert gate_up output sgu is bf16 (qwen.cu:436), sinter bf16 (kernels.cuh:1077), sout bf16 (qwen.cu:438);
 *   - routed output is fp32 (kernels.cuh:900), the combine accumulates in fp32 (kernels.cuh:1081-1121).
 * Two numerics modes exist because the reference has two MoE paths (qwen.cu:345-363):
 *   mode 0 "decode" (T < 8 in the reference): int4 dot in fp32 with (q-8) exact, the fp16 group scale applied in
 *          fp32 per 32-k chunk (gate/up, kernels.cuh:850-857) or 16-k chunk (down, kernels.cuh:879-898);
 *   mode 1 "tile" (T >= 8): weights dequantized to bf16((q-8)*scale) (dequant32_bf16, kernels.cuh:925-940),
 *          bf16 x bf16 products accumulated in fp32, per-slot weighted partials reduced in slot order
 *          (moe_down_tile_kernel kernels.cuh:1052-1055, moe_slot_reduce_kernel kernels.cuh:1059-1069).
 * The group size G is a parameter (the reference hard-codes 128 via `>>7`, kernels.cuh:842 and 1020).
 * fp32 arithmetic is IEEE single with explicit fmaf where the reference calls fmaf; build with
 * -ffp-contract=off so the compiler adds no contractions of its own.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ scalar conversions (kernels.cuh:38-48) */

static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Round-to-nearest-even float -> bf16, as __float2bfloat16 (kernels.cuh:39). */
static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* IEEE binary16 -> float, exact (kernels.cuh:42 h2f). */
static inline float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t u;
  if (e == 0) {
    float v = ldexpf((float)m, -24);
    return sign ? -v : v;
  } else if (e == 31) {
    u = sign | 0x7f800000u | (m << 13);
  } else {
    u = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline float silu(float x) { return x / (1.f + expf(-x)); }     /* kernels.cuh:49 */
static inline float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); } /* kernels.cuh:50 */

ORC_API float orc_bf16_to_f32(uint16_t b) { return bf2f(b); }
ORC_API uint16_t orc_f32_to_bf16(float f) { return f2bf(f); }
ORC_API float orc_f16_to_f32(uint16_t h) { return h2f(h); }

static int g_threads = 1;
ORC_API void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
ORC_API int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_num_procs();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ norms */

/* residual_rmsnorm_kernel<bf16> (kernels.cuh:98-114): x += d; y = bf16(x * rsqrt(mean(x^2) + eps) * w). */
ORC_API void orc_residual_rmsnorm(float* hidden, const uint16_t* d, const uint16_t* w, uint16_t* y, int T, int H,
                                  float eps) {
  for (int t = 0; t < T; ++t) {
    float* row = hidden + (int64_t)t * H;
    const uint16_t* drow = d + (int64_t)t * H;
    float ss = 0.f;
    for (int i = 0; i < H; ++i) {
      const float v = row[i] + bf2f(drow[i]);
      row[i] = v;
      ss += v * v;
    }
    const float inv = 1.f / sqrtf(ss / (float)H + eps);
    for (int i = 0; i < H; ++i) y[(int64_t)t * H + i] = f2bf(row[i] * inv * bf2f(w[i]));
  }
}

/* rmsnorm_kernel (kernels.cuh:80-93). */
ORC_API void orc_rmsnorm(const float* x, const uint16_t* w, uint16_t* y, int T, int H, float eps) {
  for (int t = 0; t < T; ++t) {
    const float* row = x + (int64_t)t * H;
    float ss = 0.f;
    for (int i = 0; i < H; ++i) ss += row[i] * row[i];
    const float inv = 1.f / sqrtf(ss / (float)H + eps);
    for (int i = 0; i < H; ++i) y[(int64_t)t * H + i] = f2bf(row[i] * inv * bf2f(w[i]));
  }
}

/* ------------------------------------------------------------------ dense bf16 projections */

/* gemv_bf16_kernel / gemm_bf16_kernel / gemm_bf16_tc_kernel (kernels.cuh:124-213, 344-361): y = x . W^T with
 * fp32 accumulation. out_bf16 != 0 rounds the result to bf16 (OutT = bf16), else stores fp32. */
static void dense_bf16(const uint16_t* x, const uint16_t* W, void* y, int out_bf16, int T, int N, int K) {
  const int64_t total = (int64_t)T * N;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && total >= 64)
  for (int64_t job = 0; job < total; ++job) {
    const int t = (int)(job / N), n = (int)(job % N);
    const uint16_t* xr = x + (int64_t)t * K;
    const uint16_t* wr = W + (int64_t)n * K;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = fmaf(bf2f(wr[k]), bf2f(xr[k]), acc);
    if (out_bf16) ((uint16_t*)y)[job] = f2bf(acc);
    else ((float*)y)[job] = acc;
  }
}

ORC_API void orc_dense_bf16_f32(const uint16_t* x, const uint16_t* W, float* y, int T, int N, int K) {
  dense_bf16(x, W, y, 0, T, N, K);
}
ORC_API void orc_dense_bf16_bf16(const uint16_t* x, const uint16_t* W, uint16_t* y, int T, int N, int K) {
  dense_bf16(x, W, y, 1, T, N, K);
}

/* ------------------------------------------------------------------ router */

/* router_topk_kernel (kernels.cuh:774-809): K rounds of argmax ordered by (value desc, index asc), then
 * w_k = exp(v_k - max) / sum over the K picks. E <= 256 and K <= 8 in the reference (kernels.cuh:773). */
ORC_API void orc_topk(const float* logits, int32_t* idx, float* wts, int T, int E, int K) {
  for (int t = 0; t < T; ++t) {
    const float* row = logits + (int64_t)t * E;
    unsigned char taken[1024];
    memset(taken, 0, sizeof taken);
    float pv[64];
    int pi[64];
    for (int kk = 0; kk < K; ++kk) {
      float bv = -1e30f;
      int bi = 0x7fffffff;
      for (int e = 0; e < E; ++e) {
        if (taken[e]) continue;
        const float v = row[e];
        if (v > bv || (v == bv && e < bi)) { bv = v; bi = e; }
      }
      if (bi == 0x7fffffff) bi = 0; /* all -inf/NaN: the reference keeps index sentinel semantics undefined */
      taken[bi] = 1;
      pv[kk] = bv;
      pi[kk] = bi;
    }
    float mx = pv[0];
    for (int kk = 1; kk < K; ++kk) mx = fmaxf(mx, pv[kk]);
    float den = 0.f;
    for (int kk = 0; kk < K; ++kk) { pv[kk] = expf(pv[kk] - mx); den += pv[kk]; }
    for (int kk = 0; kk < K; ++kk) {
      idx[(int64_t)t * K + kk] = pi[kk];
      wts[(int64_t)t * K + kk] = pv[kk] / den;
    }
  }
}

/* ------------------------------------------------------------------ routed experts, decode numerics */

/* Nibble k of an INT4 row: byte k/2, low nibble for even k (convert.py:154-156, kernels.cuh:24-26). */
static inline int nib(const uint8_t* row, int k) { return (row[k >> 1] >> ((k & 1) * 4)) & 0xF; }

/* moe_gate_up_int4_kernel (kernels.cuh:827-860): inter[t][s][i] = bf16(silu(x.Wg[e][i]) * (x.Wu[e][i])), the dot
 * taken per 32-k chunk in fp32 with (q - 8) exact, the chunk's group scale applied with fmaf. Wq [E][2I][H/2],
 * Ws [E][2I][H/G]: gate rows [0, I), up rows [I, 2I). */
ORC_API void orc_moe_gate_up_int4(const uint16_t* x, const uint8_t* Wq, const uint16_t* Ws, const int32_t* idx,
                                  uint16_t* inter, int T, int TOPK, int I, int H, int G) {
  const int64_t rowbytes = H / 2;
  const int groups = H / G;
  const int64_t total = (int64_t)T * TOPK * I;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && total >= 64)
  for (int64_t job = 0; job < total; ++job) {
    const int i = (int)(job % I);
    const int64_t row = job / I; /* t * TOPK + slot */
    const int t = (int)(row / TOPK);
    const int e = idx[row];
    const uint8_t* gw = Wq + ((int64_t)e * 2 * I + i) * rowbytes;
    const uint8_t* uw = Wq + ((int64_t)e * 2 * I + I + i) * rowbytes;
    const uint16_t* gs = Ws + ((int64_t)e * 2 * I + i) * groups;
    const uint16_t* us = Ws + ((int64_t)e * 2 * I + I + i) * groups;
    const uint16_t* xr = x + (int64_t)t * H;
    float g = 0.f, u = 0.f;
    for (int c = 0; c < H / 32; ++c) {
      float dg = 0.f, du = 0.f;
      for (int j = 0; j < 32; ++j) {
        const int k = c * 32 + j;
        const float xv = bf2f(xr[k]);
        dg = fmaf((float)(nib(gw, k) - 8), xv, dg);
        du = fmaf((float)(nib(uw, k) - 8), xv, du);
      }
      const int grp = (c * 32) / G;
      g = fmaf(dg, h2f(gs[grp]), g);
      u = fmaf(du, h2f(us[grp]), u);
    }
    inter[job] = f2bf(silu(g) * u);
  }
}

/* moe_down_int4_kernel (kernels.cuh:865-901): routed[t][h] = sum_slot w[t][slot] * (inter[t][slot] . Wd[e][h]),
 * per 16-k chunk in fp32, group scale applied with fmaf, slots accumulated in order with fmaf. */
ORC_API void orc_moe_down_int4(const uint16_t* inter, const uint8_t* Wd, const uint16_t* Sd, const int32_t* idx,
                               const float* wts, float* routed, int T, int TOPK, int H, int I, int G) {
  const int64_t rowbytes = I / 2;
  const int groups = I / G;
  const int64_t total = (int64_t)T * H;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && total >= 64)
  for (int64_t job = 0; job < total; ++job) {
    const int t = (int)(job / H), h = (int)(job % H);
    float acc = 0.f;
    for (int slot = 0; slot < TOPK; ++slot) {
      const int e = idx[(int64_t)t * TOPK + slot];
      const float w = wts[(int64_t)t * TOPK + slot];
      const uint8_t* wr = Wd + ((int64_t)e * H + h) * rowbytes;
      const uint16_t* sr = Sd + ((int64_t)e * H + h) * groups;
      const uint16_t* xr = inter + ((int64_t)t * TOPK + slot) * I;
      float part = 0.f;
      for (int c = 0; c < I / 16; ++c) {
        float d = 0.f;
        for (int j = 0; j < 16; ++j) {
          const int k = c * 16 + j;
          d = fmaf((float)(nib(wr, k) - 8), bf2f(xr[k]), d);
        }
        part = fmaf(d, h2f(sr[(c * 16) / G]), part);
      }
      acc = fmaf(w, part, acc);
    }
    routed[job] = acc;
  }
}

/* ------------------------------------------------------------------ routed experts, tile (prefill) numerics */

/* moe_sort_kernel (kernels.cuh:906-923) made stable: pairs p = t*TOPK + slot grouped by expert, ascending p
 * within an expert (the reference's order within an expert is arbitrary, kernels.cuh:922). offsets[E+1]. */
ORC_API void orc_moe_sort(const int32_t* idx, int pairs, int E, int32_t* offsets, int32_t* sorted) {
  int32_t* cnt = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
  for (int p = 0; p < pairs; ++p) cnt[idx[p]]++;
  int run = 0;
  for (int e = 0; e < E; ++e) { offsets[e] = run; run += cnt[e]; cnt[e] = offsets[e]; }
  offsets[E] = run;
  for (int p = 0; p < pairs; ++p) sorted[cnt[idx[p]]++] = p;
  free(cnt);
}

/* dequant32_bf16 (kernels.cuh:925-940): bf16((q - 8) * scale), one value. */
static inline float dq_bf16(const uint8_t* row, const uint16_t* srow, int k, int G) {
  return bf2f(f2bf((float)(nib(row, k) - 8) * h2f(srow[k / G])));
}

/* moe_gate_up_tile_kernel (kernels.cuh:942-1003): per (pair, i), g and u are fp32 sums of bf16 x times
 * bf16-dequantized weights; inter[pair][i] = bf16(silu(g) * u). */
ORC_API void orc_moe_gate_up_tile(const uint16_t* x, const uint8_t* Wq, const uint16_t* Ws, const int32_t* idx,
                                  uint16_t* inter, int T, int TOPK, int I, int H, int G) {
  const int64_t rowbytes = H / 2;
  const int groups = H / G;
  const int64_t total = (int64_t)T * TOPK * I;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && total >= 64)
  for (int64_t job = 0; job < total; ++job) {
    const int i = (int)(job % I);
    const int64_t pair = job / I;
    const int t = (int)(pair / TOPK);
    const int e = idx[pair];
    const uint8_t* gw = Wq + ((int64_t)e * 2 * I + i) * rowbytes;
    const uint8_t* uw = Wq + ((int64_t)e * 2 * I + I + i) * rowbytes;
    const uint16_t* gs = Ws + ((int64_t)e * 2 * I + i) * groups;
    const uint16_t* us = Ws + ((int64_t)e * 2 * I + I + i) * groups;
    const uint16_t* xr = x + (int64_t)t * H;
    float g = 0.f, u = 0.f;
    for (int k = 0; k < H; ++k) {
      const float xv = bf2f(xr[k]);
      g = fmaf(xv, dq_bf16(gw, gs, k, G), g);
      u = fmaf(xv, dq_bf16(uw, us, k, G), u);
    }
    inter[job] = f2bf(silu(g) * u);
  }
}

/* moe_down_tile_kernel (kernels.cuh:1005-1057): slot_out[pair][h] = (inter[pair] . bf16-dequant Wd[e][h]) * w[pair]. */
ORC_API void orc_moe_down_tile(const uint16_t* inter, const uint8_t* Wd, const uint16_t* Sd, const int32_t* idx,
                               const float* wts, float* slot_out, int T, int TOPK, int H, int I, int G) {
  const int64_t rowbytes = I / 2;
  const int groups = I / G;
  const int64_t total = (int64_t)T * TOPK * H;
#pragma omp parallel for schedule(static) num_threads(g_threads) if (g_threads > 1 && total >= 64)
  for (int64_t job = 0; job < total; ++job) {
    const int h = (int)(job % H);
    const int64_t pair = job / H;
    const int e = idx[pair];
    const uint8_t* wr = Wd + ((int64_t)e * H + h) * rowbytes;
    const uint16_t* sr = Sd + ((int64_t)e * H + h) * groups;
    const uint16_t* xr = inter + pair * I;
    float acc = 0.f;
    for (int k = 0; k < I; ++k) acc = fmaf(bf2f(xr[k]), dq_bf16(wr, sr, k, G), acc);
    slot_out[job] = acc * wts[pair];
  }
}

/* moe_slot_reduce_kernel (kernels.cuh:1059-1069): routed[t][h] = sum over slots in slot order. */
ORC_API void orc_moe_slot_reduce(const float* slot_out, float* routed, int T, int TOPK, int H) {
  for (int64_t i = 0; i < (int64_t)T * H; ++i) {
    const int t = (int)(i / H), h = (int)(i % H);
    float a = 0.f;
    for (int s = 0; s < TOPK; ++s) a += slot_out[((int64_t)t * TOPK + s) * H + h];
    routed[i] = a;
  }
}

/* ------------------------------------------------------------------ shared expert and combine */

/* silu_mul_kernel (kernels.cuh:1071-1079): out = bf16(silu(gu[:, :I]) * gu[:, I:]), gu bf16 [T, 2I]. */
ORC_API void orc_silu_mul(const uint16_t* gu, uint16_t* out, int T, int I) {
  for (int64_t i = 0; i < (int64_t)T * I; ++i) {
    const int t = (int)(i / I), j = (int)(i % I);
    const uint16_t* r = gu + (int64_t)t * 2 * I;
    out[i] = f2bf(silu(bf2f(r[j])) * bf2f(r[I + j]));
  }
}

/* shared_gate_combine_kernel (kernels.cuh:1081-1095) when w_next == NULL:
 *   gate = sigmoid(x . g); hidden += routed + gate * shared   (routed + gate*shared contracts to one fma);
 * shared_gate_combine_rmsnorm_kernel (kernels.cuh:1098-1121) when w_next != NULL:
 *   h = hidden + routed + gate * shared (the second add contracts to fma(gate, shared, hidden + routed)),
 *   then normed = bf16(h * rsqrt(mean(h^2) + eps) * w_next). gate_out (nullable) receives sigmoid(x . g). */
ORC_API void orc_shared_gate_combine(float* hidden, const float* routed, const uint16_t* shared, const uint16_t* x,
                                     const uint16_t* g, const uint16_t* w_next, uint16_t* normed, float* gate_out,
                                     int T, int H, float eps) {
  for (int t = 0; t < T; ++t) {
    float acc = 0.f;
    for (int i = 0; i < H; ++i) acc = fmaf(bf2f(x[(int64_t)t * H + i]), bf2f(g[i]), acc);
    const float gate = sigmoidf_(acc);
    if (gate_out) gate_out[t] = gate;
    float ss = 0.f;
    for (int i = 0; i < H; ++i) {
      const int64_t o = (int64_t)t * H + i;
      const float s = bf2f(shared[o]);
      float h;
      if (w_next) h = fmaf(gate, s, hidden[o] + routed[o]);
      else h = hidden[o] + fmaf(gate, s, routed[o]);
      hidden[o] = h;
      ss = fmaf(h, h, ss);
    }
    if (w_next) {
      const float inv = 1.f / sqrtf(ss / (float)H + eps);
      for (int i = 0; i < H; ++i) {
        const int64_t o = (int64_t)t * H + i;
        normed[o] = f2bf(hidden[o] * inv * bf2f(w_next[i]));
      }
    }
  }
}

/* ------------------------------------------------------------------ the block (qwen.cu:429-448) */

typedef struct orc_weights {
  const uint16_t* rms2;           /* bf16 [H]          L{i}.rms2 (1 + w folded in, convert.py:354-358) */
  const uint16_t* router;         /* bf16 [E, H]       L{i}.router */
  const uint8_t* exp_gu_q;        /* u8   [E, 2I, H/2] L{i}.exp.gate_up.q */
  const uint16_t* exp_gu_s;       /* f16  [E, 2I, H/G] L{i}.exp.gate_up.s */
  const uint8_t* exp_dn_q;        /* u8   [E, H, I/2]  L{i}.exp.down.q */
  const uint16_t* exp_dn_s;       /* f16  [E, H, I/G]  L{i}.exp.down.s */
  const uint16_t* shared_gate_up; /* bf16 [2Is, H] */
  const uint16_t* shared_down;    /* bf16 [H, Is] */
  const uint16_t* shared_gate;    /* bf16 [H] */
  int32_t H, E, TOPK, I, Is, G;
  float eps;
  const float* router_bias;       /* fp32 [E] or NULL: added to the logits as they are produced (no reference
                                   * counterpart; the prefill benchmark's per-expert Zipf skew) */
} orc_weights;

/* Optional intermediates (every pointer nullable), sized for T tokens. */
typedef struct orc_trace {
  float* logits;     /* [T, E] */
  int32_t* idx;      /* [T, TOPK] */
  float* wts;        /* [T, TOPK] */
  uint16_t* inter;   /* [T, TOPK, I] */
  float* routed;     /* [T, H] */
  uint16_t* sgu;     /* [T, 2Is] */
  uint16_t* sinter;  /* [T, Is] */
  uint16_t* sout;    /* [T, H] */
  float* gate;       /* [T] */
} orc_trace;

/* The MoE block of forward() (qwen.cu:429-448) for T tokens:
 *   hidden += attn_out; normed = rms2-norm(hidden)                       (qwen.cu:429)
 *   logits = normed . router^T; top-k                                    (qwen.cu:432-434)
 *   routed = moe(normed)                                                 (qwen.cu:435, 345-363)
 *   sout = shared_down(bf16(silu . mul(shared_gate_up(normed))))         (qwen.cu:436-438)
 *   hidden += routed + sigmoid(normed . g) * sout; normed = rms(hidden)*next_rms1 if next_rms1 (qwen.cu:444-448)
 * mode: 0 decode numerics, 1 tile numerics, -1 the reference's choice (T < 8 -> decode, qwen.cu:347).
 * Returns 0, or -1 on an unsupported shape. */
ORC_API int orc_moe_block_forward(const orc_weights* w, float* hidden, const uint16_t* attn_out, uint16_t* normed,
                                  const uint16_t* next_rms1, int T, int mode, orc_trace* tr) {
  const int H = w->H, E = w->E, K = w->TOPK, I = w->I, Is = w->Is, G = w->G;
  if (T < 1 || H % G || I % G || G % 16 || H % 32 || I % 16 || K > 64 || E > 1024 || K > E) return -1;
  if (mode < 0) mode = T < 8 ? 0 : 1;
  float* logits = (float*)malloc(sizeof(float) * (size_t)T * E);
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * K);
  float* wts = (float*)malloc(sizeof(float) * (size_t)T * K);
  uint16_t* inter = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * K * I);
  float* routed = (float*)malloc(sizeof(float) * (size_t)T * H);
  uint16_t* sgu = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * 2 * Is);
  uint16_t* sinter = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * Is);
  uint16_t* sout = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)T * H);
  float* gate = (float*)malloc(sizeof(float) * (size_t)T);

  orc_residual_rmsnorm(hidden, attn_out, w->rms2, normed, T, H, w->eps);
  dense_bf16(normed, w->router, logits, 0, T, E, H);
  if (w->router_bias)
    for (int64_t i = 0; i < (int64_t)T * E; ++i) logits[i] += w->router_bias[i % E];
  orc_topk(logits, idx, wts, T, E, K);
  if (mode == 0) {
    orc_moe_gate_up_int4(normed, w->exp_gu_q, w->exp_gu_s, idx, inter, T, K, I, H, G);
    orc_moe_down_int4(inter, w->exp_dn_q, w->exp_dn_s, idx, wts, routed, T, K, H, I, G);
  } else {
    float* slot_out = (float*)malloc(sizeof(float) * (size_t)T * K * H);
    orc_moe_gate_up_tile(normed, w->exp_gu_q, w->exp_gu_s, idx, inter, T, K, I, H, G);
    orc_moe_down_tile(inter, w->exp_dn_q, w->exp_dn_s, idx, wts, slot_out, T, K, H, I, G);
    orc_moe_slot_reduce(slot_out, routed, T, K, H);
    free(slot_out);
  }
  dense_bf16(normed, w->shared_gate_up, sgu, 1, T, 2 * Is, H);
  orc_silu_mul(sgu, sinter, T, Is);
  dense_bf16(sinter, w->shared_down, sout, 1, T, H, Is);
  orc_shared_gate_combine(hidden, routed, sout, normed, w->shared_gate, next_rms1, normed, gate, T, H, w->eps);

  if (tr) {
    if (tr->logits) memcpy(tr->logits, logits, sizeof(float) * (size_t)T * E);
    if (tr->idx) memcpy(tr->idx, idx, sizeof(int32_t) * (size_t)T * K);
    if (tr->wts) memcpy(tr->wts, wts, sizeof(float) * (size_t)T * K);
    if (tr->inter) memcpy(tr->inter, inter, sizeof(uint16_t) * (size_t)T * K * I);
    if (tr->routed) memcpy(tr->routed, routed, sizeof(float) * (size_t)T * H);
    if (tr->sgu) memcpy(tr->sgu, sgu, sizeof(uint16_t) * (size_t)T * 2 * Is);
    if (tr->sinter) memcpy(tr->sinter, sinter, sizeof(uint16_t) * (size_t)T * Is);
    if (tr->sout) memcpy(tr->sout, sout, sizeof(uint16_t) * (size_t)T * H);
    if (tr->gate) memcpy(tr->gate, gate, sizeof(float) * (size_t)T);
  }
  free(logits); free(idx); free(wts); free(inter); free(routed); free(sgu); free(sinter); free(sout); free(gate);
  return 0;
}

/* ------------------------------------------------------------------ input preparation for tests */

/* Bulk float -> bf16 (RNE) for the test-input generator. */
ORC_API void orc_f32_to_bf16_n(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f2bf(x[i]);
}

/* Rows [rows, K] of floats quantized per group of G along K (the synthetic-checkpoint recipe): scale =
 * fp16(absmax / 7), q = clamp(rint(w / scale), -7, 7) + 8, packed low nibble = even k (convert.py:154-156). */
ORC_API void orc_quantize_int4_rows(const float* w, int64_t rows, int K, int G, uint8_t* q, uint16_t* scales) {
  const int groups = K / G;
  for (int64_t r = 0; r < rows; ++r) {
    for (int g = 0; g < groups; ++g) {
      const float* src = w + r * K + (int64_t)g * G;
      float amax = 0.f;
      for (int k = 0; k < G; ++k) amax = fmaxf(amax, fabsf(src[k]));
      const _Float16 sh = (_Float16)(amax / 7.0f);
      uint16_t bits;
      memcpy(&bits, &sh, 2);
      scales[r * groups + g] = bits;
      const float s = (float)sh;
      uint8_t* dst = q + r * (K / 2) + (int64_t)g * (G / 2);
      for (int k = 0; k < G; k += 2) {
        int v[2];
        for (int j = 0; j < 2; ++j) {
          int t = s > 0.f ? (int)rintf(src[k + j] / s) : 0;
          v[j] = (t < -7 ? -7 : (t > 7 ? 7 : t)) + 8;
        }
        dst[k / 2] = (uint8_t)(v[0] | (v[1] << 4));
      }
    }
  }
}
