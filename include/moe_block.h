/* moe_block.h -- C ABI of the B200-native Qwen3.5-MoE block (libmoe_b200.so).
 *
 * Drop-in boundary for the MoE block of mvcc's examples/qwen: the launch sequence forward() issues at
 * qwen.cu:429-448 (residual RMSNorm, router + top-k, moe(), shared expert, gated combine) over the weight
 * layout convert.py writes (convert.py:6-20, 133-156, 388-415). Plain pointers and sizes only; every call is
 * asynchronous on `stream`, allocates nothing and returns a cudaError_t value as int (0 = cudaSuccess).
 *
 * Conventions (the reference's, kernels.cuh:20-23): bf16 and fp16 values travel as uint16_t bit patterns;
 * matrices are row-major [out, in]; INT4 rows pack k = 2j in the low nibble and k = 2j + 1 in the high nibble of
 * byte j, value = (q - 8) * scale, one fp16 scale per G consecutive inputs of a row. Read as uint32 words this is
 * "8 nibbles per word, nibble b of word w is k = 8w + b".
 *
 * Errors: unsupported shapes or a too-small workspace return cudaErrorInvalidValue (1) before any launch (the
 * reference exits through CK(), qwen.cu:40-47, and checks geometry at load, qwen.cu:168-171). Kernels that detect
 * an invalid expert index record it in the workspace error word (moe_workspace_error) instead of faulting.
 */
#ifndef MOE_BLOCK_H
#define MOE_BLOCK_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* moe_stream_t; /* same type as cudaStream_t; NULL = the legacy default stream */

/* One layer's MoE weights: the fields of `Layer` the block reads (qwen.cu:107-113), as device pointers into the
 * pack (pack.hpp:155), plus the geometry of `Model` (qwen.cu:127-128, 160-166) and the INT4 group size. */
typedef struct moe_layer_weights {
  const uint16_t* rms2;           /* bf16 [H]           L{i}.rms2, 1 + w folded in (convert.py:354-358) */
  const uint16_t* router;         /* bf16 [E, H]        L{i}.router */
  const uint8_t* exp_gu_q;        /* u8   [E, 2I, H/2]  L{i}.exp.gate_up.q (gate rows [0,I), up rows [I,2I)) */
  const uint16_t* exp_gu_s;       /* f16  [E, 2I, H/G]  L{i}.exp.gate_up.s */
  const uint8_t* exp_dn_q;        /* u8   [E, H, I/2]   L{i}.exp.down.q */
  const uint16_t* exp_dn_s;       /* f16  [E, H, I/G]   L{i}.exp.down.s */
  const uint16_t* shared_gate_up; /* bf16 [2Is, H]      L{i}.shared.gate_up (gate rows then up rows) */
  const uint16_t* shared_down;    /* bf16 [H, Is]       L{i}.shared.down */
  const uint16_t* shared_gate;    /* bf16 [H]           L{i}.shared.gate */
  int32_t H, E, TOPK, I, Is, G;
  float eps;
  /* Optional (NULL = none): fp32 [E] added to the router logits as they are produced, before the top-k, so the
   * logits, indices and weights all carry it. No reference counterpart: it expresses the skewed expert load of
   * the prefill benchmark (router logits plus a per-expert Zipf bias). */
  const float* router_bias;
  /* Optional (NULL = none): the shared expert as stored by the reference converter's --dense int8 (convert.py:159-169,
   * 379-385): int8 rows with one fp16 scale per group of shared_group inputs. When present, the single-launch decode
   * kernel reads these instead of the bf16 matrices (half the bytes) with the reference's int8 GEMV numerics
   * (gemv_i8_kernel, kernels.cuh:215-274: per 32 inputs an fp32 dot of the raw int8 values, scaled once by its
   * group's scale); the other paths read the bf16 matrices, which must then hold bf16(q * scale). shared_group is a
   * multiple of 32 dividing H and Is. */
  const int8_t* shared_gate_up_q8;   /* i8  [2Is, H] */
  const uint16_t* shared_gate_up_s8; /* f16 [2Is, H/shared_group] */
  const int8_t* shared_down_q8;      /* i8  [H, Is] */
  const uint16_t* shared_down_s8;    /* f16 [H, Is/shared_group] */
  int32_t shared_group;
} moe_layer_weights;

/* Shapes the kernels accept: H % 256 == 0 and H <= 4096, I % 128 == 0 and I <= 2048, Is % 128 == 0 and
 * Is <= 2048, G in {32, 64, 128} dividing H and I, 1 <= TOPK <= 8, TOPK <= E <= 256 (the reference's limits:
 * qwen.cu:168-171, kernels.cuh:773, 825, 863; the Qwen3.5-MoE geometry is H=2048, E=256, TOPK=8, I=Is=512).
 * Returns 0 if supported, else cudaErrorInvalidValue. */
MOE_API int moe_check_shape(const moe_layer_weights* w);

/* Bytes of device workspace the calls below need for up to max_T tokens per call (the reference's Work buffers,
 * qwen.cu:240-250, plus routing metadata). The caller owns it; it must be zeroed once before first use
 * (moe_workspace_init) and must not be shared by calls that overlap on the GPU. */
MOE_API size_t moe_workspace_bytes(const moe_layer_weights* w, int max_T);
MOE_API int moe_workspace_init(void* workspace, size_t workspace_bytes, moe_stream_t stream);
/* Reads (synchronously) and clears the workspace error word: 0 = no error recorded, else a code of moe_errc. */
MOE_API int moe_workspace_error(void* workspace, size_t workspace_bytes, moe_stream_t stream);

/* Library counters, the counterpart of the reference's mvccGetStats (crates/mvcc-cudart/src/api.rs:546; its
 * benchmark reads the launch count, qwen.cu:479-484): kernel launches issued by this library (counted when the launch
 * call succeeds; a launch recorded into a CUDA graph counts once, when captured, not per replay), block entry-point
 * calls that passed their checks, and bytes the pack loader (moe_pack.h) copied to the device. Process-wide and
 * thread-safe; moe_stats_reset sets all three to zero. */
typedef struct moe_stats {
  uint64_t launches;
  uint64_t block_calls;
  uint64_t pack_bytes;
} moe_stats;
MOE_API void moe_stats_get(moe_stats* out);
MOE_API void moe_stats_reset(void);

/* Error-word bits. MOE_ERR_BARRIER: a grid barrier or a weight-copy wait of the fused decode kernel gave up waiting
 * (bounded); the call's results are invalid and the workspace must be re-initialised with moe_workspace_init.
 * MOE_ERR_TIMEOUT: a bounded pipeline wait inside a prefill GEMM tile, or a cache-copy wait of the attention kernel,
 * gave up; that call's results are invalid. */
enum moe_errc { MOE_ERR_NONE = 0, MOE_ERR_EXPERT_INDEX = 1, MOE_ERR_SHAPE = 2, MOE_ERR_BARRIER = 4, MOE_ERR_TIMEOUT = 8 };

/* The whole block, replacing qwen.cu:429-448 for one layer:
 *   hidden[T,H] (fp32, in/out)  += attn_out[T,H] (bf16)                      residual_rmsnorm, qwen.cu:429
 *   normed = bf16(rms(hidden) * rms2)                                         (written to `normed`)
 *   logits = normed . router^T; top-TOPK with renormalised softmax weights    qwen.cu:432-434
 *   routed = sum over the picked experts of w * down(silu(gate) * up)         moe(), qwen.cu:435, 345-363
 *   sout = shared_down(silu . mul(shared_gate_up(normed)))                    qwen.cu:436-438
 *   hidden += routed + sigmoid(normed . shared_gate) * sout                    qwen.cu:444-448
 *   if next_rms1 != NULL: normed = bf16(rms(hidden) * next_rms1)  (shared_gate_combine_rmsnorm_kernel)
 * T >= 1 and T <= the max_T the workspace was sized for. */
MOE_API int moe_block_forward(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, float* hidden,
                      const uint16_t* attn_out, uint16_t* normed, const uint16_t* next_rms1, int T,
                      moe_stream_t stream);

/* moe_block_forward that also records events[0..3] (cudaEvent_t) on `stream`: events[0] before the first launch,
 * events[1] after the routing stage (norm, router, top-k; on the prefill path also the expert sort), events[2] after
 * the routed gate/up launch, events[3] at the end (down, shared expert, combine). The fused decode kernel (T < 8) is
 * one launch: events[1..3] all follow it. Inside stream capture the records become graph nodes. Profiling hook with
 * no reference counterpart (the reference times whole launches, qwen.cu:486-498). */
MOE_API int moe_block_forward_events(const moe_layer_weights* w, void* workspace, size_t workspace_bytes,
                                     float* hidden, const uint16_t* attn_out, uint16_t* normed,
                                     const uint16_t* next_rms1, int T, void* const* events, moe_stream_t stream);
/* Timing-event helpers for callers without their own CUDA runtime binding (cudaEvent_t as void*). */
MOE_API int moe_event_create(void** event);
MOE_API int moe_event_destroy(void* event);
MOE_API int moe_event_elapsed_ms(void* start, void* stop, float* ms);

/* Router alone (qwen.cu:432-434): logits fp32 [T,E], idx int32 [T,TOPK], wts fp32 [T,TOPK] from normed bf16 [T,H]. */
MOE_API int moe_router_topk(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const uint16_t* normed,
                    float* logits, int32_t* idx, float* wts, int T, moe_stream_t stream);

/* Routed experts alone, the reference's moe() (qwen.cu:345-363): routed fp32 [T,H] from normed bf16 [T,H] and
 * the routing idx/wts. inter_out (nullable) receives the bf16 [T,TOPK,I] SiLU-gated intermediate. */
MOE_API int moe_routed_experts(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const uint16_t* normed,
                       const int32_t* idx, const float* wts, float* routed, uint16_t* inter_out, int T,
                       moe_stream_t stream);

/* Shared expert alone (qwen.cu:436-438): sout bf16 [T,H] = down(bf16(silu(g) * u)), g/u rounded to bf16 first. */
MOE_API int moe_shared_expert(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, const uint16_t* normed,
                      uint16_t* sout, int T, moe_stream_t stream);

/* moe_router_topk without a workspace, for callers that cannot allocate device memory: a host runtime that owns all
 * device memory through its own allocator and forbids allocations after start-up has no workspace of ours to pass.
 * No counterpart in the reference. It always runs the decode router kernels, in chunks of the decode chunk: below
 * the prefill threshold its outputs equal moe_router_topk's; at or above it moe_router_topk takes the tensor-core
 * router, whose fp32 sums run in another order, so logits can differ in the last bits and picks at a near tie of
 * the 8th and 9th logits can differ. Its scratch (ticket, error word, unique-expert table: at most 3.6 KiB for
 * E <= 256, TOPK <= 8) lives in a fixed 8 KiB array in the library's device memory, held on every GPU that loads
 * the library until exit; shapes whose scratch would not fit are rejected with cudaErrorInvalidValue. Each call
 * looks up the array's device address on the current device (cudaGetSymbolAddress); the first call on a device
 * loads the library's device code there, so make it before any stream capture. Launch errors come back through the
 * return code; the scratch error word, which the kernels set as in a workspace, is read by
 * moe_router_topk_noalloc_error (the router's own top-k never produces the invalid-expert condition it records).
 * All calls share the array: calls that overlap on the GPU race and must be serialised by the caller. Allocates
 * nothing. */
MOE_API int moe_router_topk_noalloc(const moe_layer_weights* w, const uint16_t* normed, float* logits, int32_t* idx,
                                    float* wts, int T, moe_stream_t stream);

/* Reads and clears the error word of moe_router_topk_noalloc's scratch on the current device, after synchronising
 * the stream: the MOE_ERR_* bits of the last call (each call clears the word before its launches), or -cudaError.
 * Allocates nothing. */
MOE_API int moe_router_topk_noalloc_error(moe_stream_t stream);

/* Intermediates of the last moe_block_forward of T tokens on this workspace (device pointers into it, valid until
 * the next call): logits [T,E], idx [T,TOPK], wts [T,TOPK], routed [T,H] fp32, sout [T,H] bf16, gate [T] fp32; on
 * the prefill path (T >= the prefill threshold) also the expert sort: sorted [T*TOPK] (pair indices t*TOPK+slot
 * grouped by expert, ascending within an expert) and offsets [E+1] (NULL on the decode path). Decode calls above the
 * decode chunk (16 tokens at the Qwen3.5-MoE geometry) return cudaErrorInvalidValue: their intermediates are
 * produced chunk by chunk. */
typedef struct moe_trace {
  const float* logits;
  const int32_t* idx;
  const float* wts;
  const float* routed;
  const uint16_t* sout;
  const float* gate;
  const int32_t* sorted;
  const int32_t* offsets;
} moe_trace;
MOE_API int moe_workspace_trace(const moe_layer_weights* w, void* workspace, size_t workspace_bytes, int T,
                        moe_trace* out);

/* Path selection. Calls with T >= the prefill threshold (default 8, the reference's switch from the GEMV kernels
 * to the sort + tile kernels in moe(), qwen.cu:347) take the prefill path: tcgen05 tile GEMMs with the reference's
 * tile numerics (weights dequantized to bf16, fp32 accumulation, per-slot partials summed in slot order). Smaller T
 * takes the decode kernels. This sets the threshold for the whole process (0 restores the default; values below 8
 * act as 8; INT_MAX keeps every call on the decode kernels, chunk by chunk). The environment variable
 * MOE_B200_PREFILL=0 makes INT_MAX the default. No reference counterpart (the reference hard-codes 8). */
MOE_API int moe_set_prefill_min_tokens(int T);

/* ---- synthetic inputs for tests and the benchmark (no reference counterpart: the reference loads GPTQ
 * checkpoints through convert.py; these fill the same layout from a counter-based generator, seeded). */

/* out[i] = bf16(mean + std * N(0,1)) for i < n, from (seed, stream_id). */
MOE_API int moe_synth_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream_id, float mean, float std,
                          moe_stream_t stream);
/* INT4 rows [rows, K] of N(0, std) bf16 weights quantized per group of G along K: scale = fp16(absmax / 7),
 * q = clamp(rint(w / scale), -7, 7) + 8 (the int8 quantizer of convert.py:162-169 restated for 4 bits). */
MOE_API int moe_synth_int4_rows(uint8_t* q, uint16_t* scales, int64_t rows, int K, int G, uint64_t seed, uint64_t stream_id,
                        float std, moe_stream_t stream);

MOE_API const char* moe_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MOE_BLOCK_H */
