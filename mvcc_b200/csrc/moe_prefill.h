// moe_prefill.h -- launch sequences of the prefill path (T >= kPrefillMinT tokens), moe_prefill.cu.
#pragma once
#include "moe_common.cuh"

namespace moe {

// Geometry the prefill path serves (the tile GEMMs need E % 16 == 0 for their row-padded router tile; every other
// constraint follows from the shapes the library accepts). Other geometries run the decode kernels chunk by chunk.
bool prefill_supported(const moe_layer_weights& w);

// Whole block (qwen.cu:429-448 at T >= 8): residual RMSNorm, router GEMM + top-k, stable expert sort, grouped INT4
// GEMMs, shared-expert GEMMs, slot-order combine (+ the next layer's RMSNorm when a.next_rms1 is set). marks
// (nullable, 4 cudaEvent_t of which [1..3] are used) are recorded after the routing stage (norm, router, top-k,
// sort), after the gate/up GEMM and at the end.
cudaError_t prefill_block(const BlockArgs& a, cudaStream_t s, void* const* marks = nullptr);
// Router GEMM + top-k from a.normed into a.logits / a.idx / a.wts.
cudaError_t prefill_router(const BlockArgs& a, cudaStream_t s);
// moe() for caller routing a.idx / a.wts: sort, grouped GEMMs, slot-order sum into a.routed; inter_out
// (nullable) receives the bf16 [T, TOPK, I] intermediate in pair order.
cudaError_t prefill_routed(const BlockArgs& a, uint16_t* inter_out, cudaStream_t s);
// Shared expert from a.normed into a.sout.
cudaError_t prefill_shared(const BlockArgs& a, cudaStream_t s);

// Pieces the expert-parallel entry points compose (moe_ep.cu):
// residual RMSNorm of a.hidden + a.attn_out into a.normed, shared-gate sigmoid into a.gate;
cudaError_t prefill_norm(const BlockArgs& a, cudaStream_t s);
// zeroing of the pair bitmaps (before a kernel of the caller marks them);
cudaError_t prefill_bits_clear(const BlockArgs& a, cudaStream_t s);
// moe() on pair bitmaps, a.idx and a.wts the caller's kernel already wrote: scan, scatter, grouped GEMMs, slot-order
// sum into a.routed (slots with an index outside [0, E) contribute nothing);
cudaError_t prefill_routed_marked(const BlockArgs& a, cudaStream_t s);
// the same without the final slot-order sum: the per-slot partials stay in a.slot;
cudaError_t prefill_routed_marked_gemms(const BlockArgs& a, cudaStream_t s);
// gated residual combine into a.hidden (+ next RMSNorm); routed rows from a.ep_pos / a.ep_ret when set.
cudaError_t prefill_combine(const BlockArgs& a, cudaStream_t s);

}  // namespace moe
