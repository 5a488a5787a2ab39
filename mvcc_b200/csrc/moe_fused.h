// moe_fused.h -- the fused persistent decode kernel (moe_fused.cu).
#pragma once
#include "moe_common.cuh"

namespace moe {
constexpr int kFusedMaxT = 8;
// Whether the fused kernel takes this shape and T on the current device; fills its launch parameters.
bool fused_config(const moe_layer_weights& w, int T, int* stages, size_t* smem, int* rows_per_cta);
// One cooperative launch of the whole block; gbar is the workspace's grid-barrier counter.
cudaError_t launch_fused_decode(const BlockArgs& a, unsigned long long* gbar, bool next_norm, cudaStream_t s);
}  // namespace moe
