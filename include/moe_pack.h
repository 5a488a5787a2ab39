/* moe_pack.h -- reader of mvcc's .mvccq weight pack that places one layer's MoE block tensors in device memory.
 *
 * Replaces, for the MoE block, the reference's `Pack` (examples/qwen/pack.hpp:111-155: mmap, parse the header, map
 * the whole file zero-copy with cudaHostRegister, hand out device pointers per tensor) and the MoE lines of
 * `Model::load` (qwen.cu:158-166, 181-190). On a B200 the weights belong in HBM: a zero-copy mapping would stream
 * every expert read over the host link. So the file is mapped read-only on the host, the header is parsed and
 * checked once, and a layer's nine block tensors are copied into ONE caller-owned device region at 256-byte
 * aligned offsets, filling a moe_layer_weights (include/moe_block.h) that points into it.
 *
 * File format (convert.py:6-9, 175-211; pack.hpp:116-139): "MVCCQ001" | u64 little-endian header length n |
 * n bytes of JSON {"config": {...}, "tensors": {name: {"off", "nbytes", "dtype", "shape"}}} | tensor blobs at the
 * absolute file offsets `off` (64-byte aligned by the writer). Block tensors of layer i (convert.py:366-415):
 * L{i}.rms2, L{i}.router, L{i}.shared.gate_up, L{i}.shared.down, L{i}.shared.gate, L{i}.exp.gate_up.q / .s,
 * L{i}.exp.down.q / .s. Geometry keys of "config" (convert.py:327-333, read at qwen.cu:161-165): hidden, layers,
 * experts, topk, inter, shared_inter, eps, and group (absent in packs written before the key existed: 128, the
 * writer's default, convert.py:311).
 *
 * int8 shared expert (convert.py --dense int8, convert.py:159-169, 376-385): L{i}.shared.gate_up.q8 / .s8 and
 * L{i}.shared.down.q8 / .s8 (int8 rows, fp16 scales per group of K/cols(s8) inputs) are dequantised on the host to
 * bf16(q * scale) -- the product is exact in fp32, so bf16 round-to-nearest-even is the only rounding -- and
 * placed where the bf16 tensors would go. These are the weights the reference's tensor-core int8 GEMM multiplies
 * (gemm_i8_tc_kernel dequantises each K step to the same bf16 values, kernels.cuh:363-400; used for T >= 32,
 * qwen.cu:321-329); its GEMV and small-T paths multiply the fp32 products unrounded (kernels.cuh:215-330), which
 * the bf16 weights match within the bf16 tolerance. When both matrices share one group size that is a multiple of
 * 32, the int8 rows and scales are also handed to the block as stored (moe_layer_weights.shared_*_q8 / _s8 /
 * shared_group): the single-launch decode kernel then reads the int8 shared expert with the GEMV numerics, half the
 * bytes of the bf16 copy, and the other paths read the bf16 rows.
 *
 * Errors: every call returns a cudaError_t value as int. A pack that cannot be used (missing tensor, wrong shape or
 * dtype, a blob outside the file) gives cudaErrorInvalidValue (1). The reason is kept as text
 * (moe_pack_last_error). The reference exits with a message instead (qwen.cu:140-153, pack.hpp:119-130).
 * A moe_pack is used by one host thread at a time.
 */
#ifndef MOE_PACK_H
#define MOE_PACK_H

#include "moe_block.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct moe_pack moe_pack; /* opaque: the read-only file mapping and its parsed header */

/* Geometry from the header's "config" object (qwen.cu:161-165) plus the INT4 group size. */
typedef struct moe_pack_geometry {
  int32_t H, L, E, TOPK, I, Is, G;
  float eps;
} moe_pack_geometry;

/* One header entry (pack.hpp:105-109). `host` points into the read-only mapping (valid until moe_pack_close). */
typedef struct moe_pack_tensor_info {
  uint64_t off, nbytes;
  const void* host;
  int32_t ndim;
  int64_t shape[6];
  char dtype[8]; /* as written: "bf16", "f16", "f32", "u8", "i8" */
} moe_pack_tensor_info;

/* Maps `path` and parses its header. Returns NULL on failure and, if err != NULL, writes the reason (truncated to
 * err_len bytes, NUL-terminated). */
MOE_API moe_pack* moe_pack_open(const char* path, char* err, size_t err_len);
MOE_API void moe_pack_close(moe_pack* pack);
/* The reason the last failing call on `pack` returned non-zero ("" if none). Valid until the next call on it. */
MOE_API const char* moe_pack_last_error(const moe_pack* pack);

MOE_API int moe_pack_geometry_get(moe_pack* pack, moe_pack_geometry* geo);
MOE_API int moe_pack_tensor_count(const moe_pack* pack);
/* Header entry by name (cudaErrorInvalidValue if absent). */
MOE_API int moe_pack_tensor(moe_pack* pack, const char* name, moe_pack_tensor_info* info);
/* Name of the i-th header entry in byte order of the names (NULL if i is out of range). */
MOE_API const char* moe_pack_tensor_name(const moe_pack* pack, int i);

/* Layer `layer`'s block weights as HOST pointers, with the pack's geometry (router_bias NULL): every tensor checked
 * for presence, dtype and shape. The pointers lie in the mapping, except an int8 shared expert's bf16 pointers,
 * which point to its dequantised rows held by the pack (its int8 pointers lie in the mapping); all stay valid until
 * moe_pack_close. For host-side checkers. */
MOE_API int moe_pack_layer_host(moe_pack* pack, int layer, moe_layer_weights* w);
/* Device bytes that moe_pack_upload_layer needs for `layer` (each tensor at a 256-byte aligned offset, an int8
 * shared expert's int8 rows and scales after the nine block tensors); 0 if the layer cannot be loaded (the reason
 * in moe_pack_last_error). */
MOE_API size_t moe_pack_layer_bytes(moe_pack* pack, int layer);
/* Copies layer `layer`'s block tensors into `dev` (device memory, 256-byte aligned, dev_bytes >=
 * moe_pack_layer_bytes) with one host-to-device copy per tensor on `stream`, and fills `w` with device pointers
 * into `dev` and the pack's geometry. Returns once every source byte has been read from the mapping, so the pack
 * may be closed afterwards; the copies complete in stream order. */
MOE_API int moe_pack_upload_layer(moe_pack* pack, int layer, void* dev, size_t dev_bytes, moe_layer_weights* w,
                                  moe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_PACK_H */
