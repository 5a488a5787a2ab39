/* moe_ep.h -- C ABI of the expert-parallel MoE layer (libmoe_b200.so), the block of moe_block.h split over
 * `world` GPUs.
 *
 * No reference counterpart: the reference runs the whole block on one GPU (examples/qwen/qwen.cu:429-448, moe() at
 * qwen.cu:345-363). These three stages let a host runtime shard the routed experts over the GPUs of one node, rank d
 * holding experts [d * E / world, (d + 1) * E / world), and move tokens with any all-to-all that takes per-rank
 * counts (NCCL through torch.distributed in mvcc_b200/ep.py):
 *
 *   1. moe_ep_dispatch   (every rank, its own T tokens)  residual RMSNorm, router + top-k over all E experts, and
 *                        one dispatch record per (token, rank owning >= 1 of its experts) in `send`;
 *   2. all-to-all of the records (send_count per destination), then moe_ep_experts on the R records received:
 *                        one bf16 partial row per record (its local slots, in slot order, weighted, summed in fp32
 *                        and rounded once);
 *   3. all-to-all of the partial rows back (the reverse counts), then moe_ep_combine: per token the partials in rank
 *                        order, plus the gated shared expert (moe_shared_expert on the rank's own tokens).
 *
 * Numerics: those of the prefill path (tile numerics, per-slot fp32 partials) except that a token's routed sum is
 * taken per rank in slot order, rounded to bf16 (the partial row that crosses the exchange: 2 H bytes instead of
 * 4 H), and then summed over ranks in rank order in fp32; with world = 1 it equals moe_block_forward's prefill path
 * with the routed row rounded to bf16. Same conventions and error rules as moe_block.h; every call is asynchronous
 * on `stream` and allocates nothing.
 */
#ifndef MOE_EP_H
#define MOE_EP_H
#include "moe_block.h"
#ifdef __cplusplus
extern "C" {
#endif

/* Bytes of one dispatch record: H bf16 normed activations, then TOPK int32 expert ids local to the destination
 * rank (-1 = that slot's expert is on another rank), then TOPK fp32 routing weights, padded to 16 bytes. */
MOE_API size_t moe_ep_record_bytes(const moe_layer_weights* w);

/* Stage 1 on each rank. w: the full layer geometry (E = all experts; router, rms2 and shared_gate are read, the
 * expert pointers are not). hidden fp32 [T,H] and attn_out bf16 [T,H] are read (hidden is not written: the combine
 * applies the residual); normed bf16 [T,H] is written. Outputs:
 *   send        records, capacity T * world: destination d's records start at the sum of send_count[0..d), tokens
 *               ascending within a destination;
 *   send_count  int32 [world];
 *   tok_pos     int32 [T, world]: the record index of token t for rank d, -1 when t has no expert on d.
 * The shared-gate logits stay in the workspace for moe_ep_combine, which must get the same workspace. Requires
 * 1 <= world <= 8, E % world == 0, (E / world) % 16 == 0 and E / world >= TOPK; the workspace is sized by
 * moe_workspace_bytes(w, T). */
MOE_API int moe_ep_dispatch(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const float* hidden,
                            const uint16_t* attn_out, uint16_t* normed, int T, int world, void* send,
                            int32_t* send_count, int32_t* tok_pos, moe_stream_t stream);

/* Stage 2 on each rank. w_local: this rank's shard (E = E / world, the exp_* pointers at its first expert; router
 * and shared pointers unused). recv: R records (R = 0 launches nothing). part bf16 [R,H]: per record the sum, over
 * its slots whose id is a local expert and in slot order, of weight * down(bf16(silu(gate) * up)) with the prefill
 * path's tile numerics, accumulated in fp32 and rounded to bf16. Ids outside [-1, E) are flagged (MOE_ERR_EXPERT_INDEX) and skipped. The workspace is sized
 * by moe_workspace_bytes(w_local, max(R_max, 8)). */
MOE_API int moe_ep_experts(const moe_layer_weights* w_local, void* workspace, size_t workspace_bytes, const void* recv,
                           int R, uint16_t* part, moe_stream_t stream);

/* Stage 3 on each rank, on the workspace of its moe_ep_dispatch call. ret bf16 [sum of send_count, H]: the partial
 * rows returned for this rank's records, in record order; sout bf16 [T,H] the shared expert of normed
 * (moe_shared_expert). hidden += attn_out + routed + sigmoid(gate) * sout with routed[t] the sum over ranks d
 * ascending of ret[tok_pos[t, d]] (tok_pos >= 0), in fp32; then normed = rms(hidden) * next_rms1 when next_rms1 != NULL. */
MOE_API int moe_ep_combine(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, float* hidden,
                           const uint16_t* attn_out, const uint16_t* sout, uint16_t* normed,
                           const uint16_t* next_rms1, int T, int world, const int32_t* tok_pos, const uint16_t* ret,
                           moe_stream_t stream);

/* ---- peer-memory exchange: the same three stages with the data moved by the kernels themselves over NVLink.
 *
 * Every rank owns a receive buffer of moe_ep_recv_bytes(w, world, cap) bytes (records [world][cap][record], source
 * s's block at s * cap, then int32 counts [world]) and a return buffer of moe_ep_ret_bytes bytes (bf16 rows
 * [world][cap][H], destination d's block at d * cap), cap = the most tokens any rank passes per call. `peers` holds
 * every rank's buffers as addresses valid on the calling device (moe_ipc_open of the peers' handles; the local
 * buffers for this rank). moe_ep_dispatch_peers stores this rank's records and counts straight into the destination
 * ranks' receive buffers; moe_ep_experts_peers reads this rank's receive buffer and stores each record's partial
 * row straight into its source rank's return buffer; moe_ep_combine then reads the local return buffer with the
 * tok_pos of the dispatch. Between dispatch and experts, and between experts and combine, every rank must pass a
 * collective barrier (any collective, e.g. a one-element all-reduce, ordered on the same stream after the kernels):
 * the kernels end their peer stores with system-scope fences, so the barrier publishes them. No host
 * synchronisation, no per-step allocation. */
typedef struct moe_ep_peers {
  void* recv[8];
  int32_t* rcount[8];  /* inside each recv buffer (its counts) */
  uint16_t* ret[8];  /* bf16 partial rows */
  int32_t rank, cap;
} moe_ep_peers;
MOE_API size_t moe_ep_recv_bytes(const moe_layer_weights* w, int world, int cap);
MOE_API size_t moe_ep_ret_bytes(const moe_layer_weights* w, int world, int cap);
/* Offset of the counts inside a receive buffer. */
MOE_API size_t moe_ep_rcount_offset(const moe_layer_weights* w, int world, int cap);
MOE_API int moe_ep_dispatch_peers(const moe_layer_weights* w, void* workspace, size_t workspace_bytes,
                                  const float* hidden, const uint16_t* attn_out, uint16_t* normed, int T, int world,
                                  const moe_ep_peers* peers, int32_t* send_count, int32_t* tok_pos,
                                  moe_stream_t stream);
/* workspace sized by moe_workspace_bytes(w_local, max(world * cap, 8)). */
MOE_API int moe_ep_experts_peers(const moe_layer_weights* w_local, void* workspace, size_t workspace_bytes, int world,
                                 const moe_ep_peers* peers, moe_stream_t stream);

/* Setup helpers for the exchange buffers (the only calls of this library that allocate): device memory that CUDA
 * IPC can share, its 64-byte IPC handle, and the mapping of a peer's handle into this process (cudaMalloc,
 * cudaIpcGetMemHandle, cudaIpcOpenMemHandle with lazy peer access, and their releases). */
MOE_API int moe_device_alloc(size_t bytes, void** ptr);
MOE_API int moe_device_free(void* ptr);
MOE_API int moe_ipc_handle(void* ptr, void* handle64);
MOE_API int moe_ipc_open(const void* handle64, void** ptr);
MOE_API int moe_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif
#endif /* MOE_EP_H */
