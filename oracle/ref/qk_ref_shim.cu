// qk_ref_shim.cu -- C-ABI launchers around the reference's own CUDA kernels (examples/qwen/kernels.cuh).
//
// TEST INFRASTRUCTURE, NOT PRODUCT CODE. oracle/Makefile compiles this file against the reference sources where
// they lie (-I <reference>/examples/qwen, and an include dir whose only entry is a symlink to
// <reference>/include/mvcc), into oracle/_ref/libqk_ref.so. Tests and tests/golden/make_golden.py use it to run
// the reference's kernels on a B200 and pin the CPU oracle to their outputs; bench.py's reference arm times them.
// Nothing here is shipped or called by the product path.
//
// The launch sequences restate the reference host code, which is static in qwen.cu and cannot be linked:
//   ref_dense_*        dense() dispatch, qwen.cu:298-319 (bf16 weights only)
//   ref_moe            moe(), qwen.cu:345-363, with the default QWEN_MOE_TK=32, QWEN_MOE_NB=128 (qwen.cu:27-33)
//   ref_block_forward  the MoE block of forward(), qwen.cu:429-448
//   ref_attn_forward   the attention branch of forward(), qwen.cu:413-425, with attention() of qwen.cu:52-64
//   ref_lm_head        the final norm, dense() and two-stage argmax of forward(), qwen.cu:451-456
// Buffers follow Work::alloc (qwen.cu:258-292): activation buffers read by the tensor-core GEMMs hold
// round_up(T, 128) rows (qwen.cu:259).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "kernels.cuh"

namespace {
inline int cdiv(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

template <typename OutT>
void dense(const qk::bf16* x, const qk::bf16* W, OutT* y, int T, int N, int K, cudaStream_t s) {
  if (T >= 32 && K % 128 == 0 && N % 32 == 0) {
    if (T >= 128 && N >= 2048) {
      dim3 grid(cdiv(T, 128), cdiv(N, 128));
      qk::gemm_bf16_tc_kernel<4, 4, OutT><<<grid, 512, 0, s>>>(x, W, y, T, N, K);
    } else {
      dim3 grid(cdiv(T, 64), cdiv(N, 64));
      qk::gemm_bf16_tc_kernel<2, 2, OutT><<<grid, 128, 0, s>>>(x, W, y, T, N, K);
    }
  } else if (T >= 8) {
    dim3 grid(cdiv(N, 64), cdiv(T, 32));
    qk::gemm_bf16_kernel<OutT><<<grid, 256, 0, s>>>(x, W, y, T, N, K);
  } else if (T == 1) {
    qk::gemv_bf16_kernel<1, OutT><<<dim3(cdiv(N, 8), 1), 256, 0, s>>>(x, W, y, T, N, K);
  } else if (T == 2) {
    qk::gemv_bf16_kernel<2, OutT><<<dim3(cdiv(N, 8), 1), 256, 0, s>>>(x, W, y, T, N, K);
  } else {
    qk::gemv_bf16_kernel<4, OutT><<<dim3(cdiv(N, 8), cdiv(T, 4)), 256, 0, s>>>(x, W, y, T, N, K);
  }
}
}  // namespace

extern "C" {

struct qkref_layer {
  const uint16_t* rms2;
  const uint16_t* router;
  const uint8_t* exp_gu_q;
  const uint16_t* exp_gu_s;
  const uint8_t* exp_dn_q;
  const uint16_t* exp_dn_s;
  const uint16_t* shared_gate_up;
  const uint16_t* shared_down;
  const uint16_t* shared_gate;
  int32_t H, E, TOPK, I, Is;
  float eps;
};

// Work fields used by the MoE block (qwen.cu:240-250).
struct qkref_work {
  float* logits_r;     // [T, E]
  int32_t* topk_i;     // [T, TOPK]
  float* topk_w;       // [T, TOPK]
  uint16_t* inter;     // [T, TOPK, I]
  float* routed;       // [T, H]
  int32_t* moe_off;    // [E + 1]
  int32_t* moe_sorted; // [T * TOPK]
  float* slot_out;     // [T * TOPK, H]
  uint16_t* sgu;       // [T, 2 Is]
  uint16_t* sinter;    // [T, Is]  (round_up(T,128) rows)
  uint16_t* sout;      // [T, H]
};

int qkref_residual_rmsnorm(float* hidden, const uint16_t* d, const uint16_t* w, uint16_t* y, int T, int H, float eps,
                           cudaStream_t s) {
  qk::residual_rmsnorm_kernel<qk::bf16><<<T, 256, 0, s>>>(hidden, d, w, y, H, eps);
  return (int)cudaGetLastError();
}

int qkref_dense_f32(const uint16_t* x, const uint16_t* W, float* y, int T, int N, int K, cudaStream_t s) {
  dense<float>(x, W, y, T, N, K, s);
  return (int)cudaGetLastError();
}

int qkref_dense_bf16(const uint16_t* x, const uint16_t* W, uint16_t* y, int T, int N, int K, cudaStream_t s) {
  dense<qk::bf16>(x, W, y, T, N, K, s);
  return (int)cudaGetLastError();
}

int qkref_router_topk(const float* logits, int32_t* idx, float* wts, int T, int E, int K, cudaStream_t s) {
  qk::router_topk_kernel<<<cdiv(T, 8), 256, 0, s>>>(logits, idx, wts, T, E, K);
  return (int)cudaGetLastError();
}

// moe() (qwen.cu:345-363): T < 8 takes the warp-per-row int4 GEMVs, else sort + tensor-core tiles + slot reduce.
int qkref_moe(const qkref_layer* l, qkref_work* w, const uint16_t* normed, int T, cudaStream_t s) {
  const int H = l->H;
  if (T < 8) {
    qk::moe_gate_up_int4_kernel<<<cdiv((int64_t)T * l->TOPK * l->I, 8), 256, 0, s>>>(
        normed, l->exp_gu_q, l->exp_gu_s, w->topk_i, w->inter, T, l->TOPK, l->I, H);
    qk::moe_down_int4_kernel<<<cdiv((int64_t)T * H, 8), 256, 0, s>>>(w->inter, l->exp_dn_q, l->exp_dn_s, w->topk_i,
                                                                      w->topk_w, w->routed, T, l->TOPK, H, l->I);
    return (int)cudaGetLastError();
  }
  const int pairs = T * l->TOPK;
  qk::moe_sort_kernel<<<1, 256, 0, s>>>(w->topk_i, pairs, l->E, w->moe_off, w->moe_sorted);
  qk::moe_gate_up_tile_kernel<32, 128><<<dim3(l->I / 64, l->E), 128, 0, s>>>(
      normed, l->exp_gu_q, l->exp_gu_s, w->moe_off, w->moe_sorted, w->inter, l->TOPK, l->I, H);
  qk::moe_down_tile_kernel<32, 128><<<dim3(H / 128, l->E), 128, 0, s>>>(
      w->inter, l->exp_dn_q, l->exp_dn_s, w->moe_off, w->moe_sorted, w->topk_w, w->slot_out, H, l->I);
  qk::moe_slot_reduce_kernel<<<std::min(cdiv((int64_t)T * H, 256), 4096), 256, 0, s>>>(w->slot_out, w->routed, T,
                                                                                        l->TOPK, H);
  return (int)cudaGetLastError();
}

// The MoE block of forward() (qwen.cu:429-448). next_rms1 == nullptr selects the last-layer combine.
int qkref_block_forward(const qkref_layer* l, qkref_work* w, float* hidden, const uint16_t* attn_out,
                        uint16_t* normed, const uint16_t* next_rms1, int T, cudaStream_t s) {
  const int H = l->H;
  qk::residual_rmsnorm_kernel<qk::bf16><<<T, 256, 0, s>>>(hidden, attn_out, l->rms2, normed, H, l->eps);
  dense<float>(normed, l->router, w->logits_r, T, l->E, H, s);
  qk::router_topk_kernel<<<cdiv(T, 8), 256, 0, s>>>(w->logits_r, w->topk_i, w->topk_w, T, l->E, l->TOPK);
  int rc = qkref_moe(l, w, normed, T, s);
  if (rc) return rc;
  dense<qk::bf16>(normed, l->shared_gate_up, w->sgu, T, 2 * l->Is, H, s);
  qk::silu_mul_kernel<<<std::min(cdiv((int64_t)T * l->Is, 256), 4096), 256, 0, s>>>(w->sgu, w->sinter, T, l->Is);
  dense<qk::bf16>(w->sinter, l->shared_down, w->sout, T, H, l->Is, s);
  if (next_rms1)
    qk::shared_gate_combine_rmsnorm_kernel<<<T, 256, 0, s>>>(hidden, w->routed, w->sout, normed, l->shared_gate,
                                                             next_rms1, normed, H, l->eps);
  else
    qk::shared_gate_combine_kernel<<<T, 256, 0, s>>>(hidden, w->routed, w->sout, normed, l->shared_gate, H);
  return (int)cudaGetLastError();
}

// The attention branch of forward() (qwen.cu:413-425) for T tokens at pos0. Buffers: qkv [T, (Hq + 2 Hkv) D],
// z [T, Hq D] (if gate), q [T, Hq, D], o [T, Hq D], part [T Hq 32][D + 2] (kMaxSplit = 32), caches [Hkv][ctx][D].
int qkref_attn_forward(const uint16_t* normed, const uint16_t* Wqkv, const uint16_t* Wgate, const uint16_t* Wo,
                       const uint16_t* q_norm, const uint16_t* k_norm, uint16_t* kc, uint16_t* vc, uint16_t* qkv,
                       uint16_t* z, uint16_t* q, uint16_t* o, float* part, uint16_t* attn_out, int T, int H, int Hq,
                       int Hkv, int D, int rope_dim, float theta, int pos0, int ctx, float eps, cudaStream_t s) {
  const int heads = Hq + 2 * Hkv;
  dense<qk::bf16>(normed, Wqkv, qkv, T, heads * D, H, s);
  if (Wgate) dense<qk::bf16>(normed, Wgate, z, T, Hq * D, H, s);
  qk::attn_qk_norm_rope_kernel<<<cdiv(T * heads, 8), 256, 0, s>>>(qkv, q_norm, k_norm, q, kc, vc, T, Hq, Hkv, D,
                                                                  rope_dim, theta, pos0, ctx, eps);
  // attention(), qwen.cu:52-64
  const int blocks = T * Hkv, jobs = T * Hq, nkeys = pos0 + T;
  const int nsplit = std::max(1, std::min({32, cdiv(nkeys, 32), cdiv(64, blocks)}));
  qk::attn_partial_kernel<256><<<dim3(blocks, nsplit), 256, 0, s>>>(q, kc, vc, part, T, Hq, Hkv, ctx, pos0, nsplit,
                                                                    1.f / sqrtf((float)D));
  qk::attn_combine_kernel<256><<<cdiv(jobs, 8), 256, 0, s>>>(part, o, jobs, nsplit);
  if (Wgate)
    qk::sigmoid_gate_kernel<<<std::min(cdiv((int64_t)T * Hq * D, 256), 4096), 256, 0, s>>>(o, z, (int64_t)T * Hq * D);
  dense<qk::bf16>(o, Wo, attn_out, T, H, Hq * D, s);
  return (int)cudaGetLastError();
}

// The LM head of forward() (qwen.cu:451-456) for the last token's fp32 residual: final RMSNorm, logits (fp32 [V]),
// argmax. Buffers: normed [H] bf16, pmax / pidx [1024].
int qkref_lm_head(const float* hidden_last, const uint16_t* final_norm, const uint16_t* lm_head, uint16_t* normed,
                  float* logits, float* pmax, int32_t* pidx, int32_t* next, int V, int H, float eps, cudaStream_t s) {
  qk::rmsnorm_kernel<<<1, 256, 0, s>>>(hidden_last, final_norm, normed, H, eps);
  dense<float>(normed, lm_head, logits, 1, V, H, s);
  qk::argmax_partial_kernel<<<1024, 256, 0, s>>>(logits, V, pmax, pidx);
  qk::argmax_final_kernel<<<1, 256, 0, s>>>(pmax, pidx, 1024, next);
  return (int)cudaGetLastError();
}

}  // extern "C"
