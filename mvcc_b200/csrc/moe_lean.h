// moe_lean.h -- the compact single-launch decode kernel for one or two tokens (moe_lean.cu).
#pragma once
#include "moe_common.cuh"

namespace moe {
constexpr int kLeanMaxT = 2;
// Whether the lean kernel takes this shape and T on the current device (only when MOE_B200_LEAN=1).
bool lean_config(const moe_layer_weights& w, int T);
// One cooperative launch of the whole block; gbar is the workspace's grid-barrier counter.
cudaError_t launch_lean_decode(const BlockArgs& a, unsigned long long* gbar, bool next_norm, cudaStream_t s);
}  // namespace moe
