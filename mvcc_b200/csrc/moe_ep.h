// moe_ep.h -- kernels of the expert-parallel stages (moe_ep.cu) behind include/moe_ep.h.
#pragma once
#include "moe_common.cuh"

namespace moe {

constexpr int kEpMaxWorld = 8;

// Bytes of one dispatch record: H bf16 activations, TOPK int32 local expert ids, TOPK fp32 weights, 16-aligned.
inline int ep_record_bytes(int H, int TOPK) { return (2 * H + 8 * TOPK + 15) / 16 * 16; }

// Source side: from a.idx / a.wts / a.normed of T = a.T tokens, the destination plan (tok_pos [T][world], counts
// [world]) and the records in `send`, grouped by destination in rank order, tokens ascending within a rank.
cudaError_t ep_plan_pack(const BlockArgs& a, int world, uint8_t* send, int32_t* send_count, int32_t* tok_pos,
                         cudaStream_t s);
// Destination side: a.idx / a.wts of the a.T received records from their meta fields, and the pair bitmaps of the
// slots with a local expert (-1 = another rank's slot: skipped; other out-of-range ids are flagged and skipped).
cudaError_t ep_mark(const BlockArgs& a, const uint8_t* recv, cudaStream_t s);

}  // namespace moe
