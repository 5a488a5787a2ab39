// moe_ep.h -- kernels of the expert-parallel stages (moe_ep.cu) behind include/moe_ep.h.
#pragma once
#include "moe_common.cuh"

namespace moe {

constexpr int kEpMaxWorld = 8;

// Peer-memory exchange: every rank's receive records [world][cap][record] followed by its per-source counts
// [world], and its return rows [world][cap][H] fp32, as pointers valid on this device (CUDA IPC mappings of the peers'
// buffers, or the local ones); rank and cap (tokens per rank at most) of this process.
struct EpPeers {
  uint8_t* recv[kEpMaxWorld];
  int32_t* rcount[kEpMaxWorld];
  uint16_t* ret[kEpMaxWorld];  // bf16 partial rows
  int rank, cap;
};

// Bytes of one dispatch record: H bf16 activations, TOPK int32 local expert ids, TOPK fp32 weights, 16-aligned.
inline int ep_record_bytes(int H, int TOPK) { return (2 * H + 8 * TOPK + 15) / 16 * 16; }

// Source side: from a.idx / a.wts / a.normed of T = a.T tokens, the destination plan (tok_pos [T][world], counts
// [world]) and the records in `send`, grouped by destination in rank order, tokens ascending within a rank.
cudaError_t ep_plan_pack(const BlockArgs& a, int world, uint8_t* send, int32_t* send_count, int32_t* tok_pos,
                         cudaStream_t s);
// The same plan with the records stored straight into the destination ranks' receive buffers (source block `rank`,
// position = the token's index among those sent to that rank) and the counts into their count arrays; tok_pos holds
// d * cap + index, the row of the return buffer the destination will fill.
cudaError_t ep_plan_pack_peers(const BlockArgs& a, int world, const EpPeers& peers, int32_t* send_count,
                               int32_t* tok_pos, cudaStream_t s);
// Destination side: a.idx / a.wts of the a.T received records from their meta fields, and the pair bitmaps of the
// slots with a local expert (-1 = another rank's slot: skipped; other out-of-range ids are flagged and skipped).
// rcount (nullable): records of source s occupy rows [s * cap, s * cap + rcount[s]); other rows are empty.
cudaError_t ep_mark(const BlockArgs& a, const uint8_t* recv, const int32_t* rcount, int cap, cudaStream_t s);
// Destination side, peer mode: per valid record row the slot-order sum of its slot partials (a.slot), stored into
// the source rank's return buffer at row rank * cap + index.
cudaError_t ep_return_peers(const BlockArgs& a, int world, const EpPeers& peers, cudaStream_t s);

}  // namespace moe
