/* moe_stack.h -- the attention layer and LM head of a Qwen3.5-MoE decode step on a B200 (sm_100a): the pieces
 * around the MoE block (include/moe_block.h) that a whole decode stack needs. C ABI, plain pointers and sizes, every
 * call asynchronous on `stream`, returning a cudaError_t (0 on success).
 *
 * The reference has no C ABI: its attention branch is the launch sequence forward() issues at
 * examples/qwen/qwen.cu:413-425 (dense(), attn_qk_norm_rope_kernel, attention(), sigmoid_gate_kernel, dense()) and its
 * LM head the lines at qwen.cu:451-456 (rmsnorm_kernel, dense(), argmax_partial_kernel, argmax_final_kernel). These
 * entry points replace those sequences one for one; the final RMSNorm is the MoE block's next_rms1 (the last layer's
 * moe_block_forward with next_rms1 = final_norm writes the normed last token).
 */
#ifndef MOE_STACK_H
#define MOE_STACK_H

#include <stddef.h>
#include <stdint.h>

#include "moe_block.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One attention layer's weights, exactly the reference's Layer fields (qwen.cu:119-123) in the pack layout, all
 * bf16: qkv [(Hq + 2 Hkv) D, H] (q heads, then k heads, then v heads), gate [Hq D, H] (NULL when the model has no
 * attention output gate), o [H, Hq D], q_norm and k_norm [D] (the converter folds the +1 in). Geometry: H % 256 == 0,
 * H <= 8192, D == 256 (the reference's kernels hard-code it, kernels.cuh:681), Hq / Hkv divides 8, rope_dim even
 * and <= D, (Hq + 2 Hkv) D and H multiples of 8. */
typedef struct moe_attn_weights {
  const uint16_t* qkv;
  const uint16_t* gate;
  const uint16_t* o;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  int32_t H, Hq, Hkv, D, rope_dim;
  float theta, eps;
} moe_attn_weights;

/* Bytes of caller-owned workspace for attention calls of up to max_T tokens over a cache of ctx positions; 0 for an
 * unsupported geometry. One workspace per concurrently running call (it holds an error word, the qkv, q, gate and o
 * activations and the split-K partials). Zero it once before its first call (cudaMemset), as for the block's
 * workspace: the calls set bits of the error word and never clear it. */
MOE_API size_t moe_attn_workspace_bytes(const moe_attn_weights* w, int max_T, int ctx);

/* Reads and clears the attention workspace's error word, synchronising the stream: MOE_ERR_TIMEOUT (include/
 * moe_block.h) when a cache-copy wait of a call gave up (that call's attention output is invalid), else 0; a
 * negative value is -cudaError. */
MOE_API int moe_attn_workspace_error(void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* The attention branch of one layer (qwen.cu:413-425) for T new tokens at positions pos0 .. pos0 + T - 1:
 * qkv = normed . Wqkv^T (bf16); per-head RMSNorm of q and k heads and rotate-half RoPE over the first rope_dim dims
 * (attn_qk_norm_rope_kernel, kernels.cuh:608-663), the new k and v rows written into the bf16 caches
 * kc, vc [Hkv][ctx][D] at their positions; causal GQA attention of each query head over keys [0, pos] of its kv head
 * (split-K online softmax, kernels.cuh:665-761); if w->gate, o *= sigmoid(normed . Wgate^T) (kernels.cuh:765-769);
 * attn_out = o . Wo^T (bf16 [T,H]), the input of moe_block_forward. normed bf16 [T,H]. Requires 1 <= T <= 4 and
 * pos0 + T <= ctx; other shapes return cudaErrorInvalidValue before any launch. */
MOE_API int moe_attn_forward(const moe_attn_weights* w, uint16_t* kc, uint16_t* vc, int ctx, int pos0,
                             const uint16_t* normed, uint16_t* attn_out, int T, void* workspace, size_t workspace_bytes,
                             moe_stream_t stream);

/* moe_attn_forward with the layer's input RMSNorm (qwen.cu:411, rmsnorm_kernel, kernels.cuh:83-93) fused into its
 * first GEMV: the fp32 residual hidden [T,H] is normalised with rms1 (bf16 [H], eps = w->eps) by every CTA of that
 * GEMV as it stages its input, instead of a normed input being read. A decode step then needs neither the first
 * layer's separate norm launch nor the MoE block's fused next-layer norm (a serial tail: the last CTA of that kernel
 * normalises the row while the GPU waits). Same shapes and errors as moe_attn_forward; hidden and rms1 16-byte
 * aligned. */
MOE_API int moe_attn_forward_rms(const moe_attn_weights* w, const uint16_t* rms1, const float* hidden, uint16_t* kc,
                                 uint16_t* vc, int ctx, int pos0, uint16_t* attn_out, int T, void* workspace,
                                 size_t workspace_bytes, moe_stream_t stream);

/* y = bf16(x * rsqrt(mean(x^2) + eps) * w) per row (rmsnorm_kernel, kernels.cuh:83-93): a layer's input norm as a
 * launch of its own (moe_attn_forward_rms fuses it instead). x fp32 [T,H], w and y bf16. */
MOE_API int moe_rmsnorm(const float* x, const uint16_t* w, uint16_t* y, int T, int H, float eps, moe_stream_t stream);

/* Bytes of caller-owned workspace for moe_lm_head_argmax over a vocabulary of V rows of H. */
MOE_API size_t moe_lm_head_workspace_bytes(int V, int H);

/* The LM head of the last token (qwen.cu:452-456): logits = x . W^T (fp32 [V], written when `logits` is not NULL)
 * for x = normed bf16 [H] and W bf16 [V,H], and *next = the index of the largest logit, ties to the lowest index, NaN
 * never winning and 0 when nothing beats -1e30 (argmax_partial_kernel / argmax_final_kernel, kernels.cuh:1124-1164).
 * One launch: every CTA reduces its rows and the last CTA to finish reduces the CTAs' results. The workspace must
 * be zeroed once before first use (its ticket counter returns to zero by itself). */
MOE_API int moe_lm_head_argmax(const uint16_t* normed, const uint16_t* lm_head, int V, int H, float* logits,
                               int32_t* next, void* workspace, size_t workspace_bytes, moe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_STACK_H */
