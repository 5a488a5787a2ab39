// moe_decode.h -- launchers of the decode-path kernels (moe_decode.cu), used by the C-ABI in moe_api.cu.
#pragma once
#include "moe_common.cuh"

namespace moe {
// Elements per staged bf16 inter row in the down kernel: I, padded to a multiple of 512 above 512.
__host__ __device__ inline int inter_stride(int I) {
  const int nchd = I / 16, L = nchd < 32 ? nchd : 32;
  return ((nchd + L - 1) / L) * 2 * L * 8;
}
size_t down_smem_bytes(int T, int TOPK, int I, int Is, bool xf32);
size_t gate_up_smem_bytes(int T, int H);

// Largest token count one decode launch sequence handles: the gate/up kernel stages T x H fp32 activations and
// the down kernel the T x TOPK bf16 intermediates, T x Is shared intermediates and per-warp accumulators in
// shared memory (each kept under 200 KB); at most 16.
inline int decode_max_tokens(int H, int TOPK, int I, int Is) {
  const size_t budget = 200 * 1024;
  int t = 16;
  while (t > 1 && (gate_up_smem_bytes(t, H) > budget || down_smem_bytes(t, TOPK, I, Is, false) > budget)) --t;
  return t;
}

cudaError_t launch_route(const BlockArgs& a, bool from_hidden, bool with_gate, cudaStream_t s);
cudaError_t launch_route_table(const BlockArgs& a, cudaStream_t s);
cudaError_t launch_gate_up(const BlockArgs& a, bool routed, bool shared, cudaStream_t s);
// mode bits: 1 routed, 2 shared, 4 combine into hidden, 8 next-layer RMSNorm.
cudaError_t launch_down_combine(const BlockArgs& a, int mode, cudaStream_t s);
}  // namespace moe
