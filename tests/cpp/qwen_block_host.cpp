// qwen_block_host.cpp -- the MoE block driven from C++ through the C ABI, as examples/qwen/qwen.cu would drive it:
// the block tensors of one layer loaded from a .mvccq pack into HBM (moe_pack.h; replaces the block lines of
// Model::load, qwen.cu:181-190), one workspace (moe_workspace_bytes / _init; replaces the block's Work buffers,
// qwen.cu:240-292), then forward() for T tokens (moe_block_forward; replaces qwen.cu:429-448) and the error word.
//
//   qwen_block_host PACK [LAYER] [T] [IN OUT]
//       prints "ok T=<T> launches=<n> max|hidden|=<v>" and exits 0 on success. With IN and OUT, the residual (fp32
//       [T,H]) and attn_out (bf16 [T,H]) are read from the raw file IN, and the updated residual, `normed` and the
//       router logits (fp32 [T,E], from moe_workspace_trace) are written to the raw file OUT; otherwise fixed inputs
//       are used.
//
// Test infrastructure: tests/test_abi.py compiles and links it (and checks its refusals) on any host;
// tests/test_cpp_host_gpu.py runs it on a B200 against the CPU oracle.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "moe_block.h"
#include "moe_pack.h"

#define CK(x)                                                                              \
  do {                                                                                     \
    const int rc_ = (int)(x);                                                              \
    if (rc_ != 0) {                                                                        \
      std::fprintf(stderr, "%s:%d: %s failed: %d\n", __FILE__, __LINE__, #x, rc_);         \
      std::exit(1);                                                                        \
    }                                                                                      \
  } while (0)

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s PACK [LAYER] [T]\n", argv[0]);
    return 2;
  }
  const int layer = argc > 2 ? std::atoi(argv[2]) : 0;
  const int T = argc > 3 ? std::atoi(argv[3]) : 1;
  char why[512];
  moe_pack* pk = moe_pack_open(argv[1], why, sizeof why);
  if (!pk) {
    std::fprintf(stderr, "%s\n", why);
    return 1;
  }
  cudaStream_t s;
  CK(cudaStreamCreate(&s));
  const size_t wbytes = moe_pack_layer_bytes(pk, layer);
  if (wbytes == 0) {
    std::fprintf(stderr, "%s\n", moe_pack_last_error(pk));
    return 1;
  }
  void* wdev = nullptr;
  CK(cudaMalloc(&wdev, wbytes));
  moe_layer_weights w;
  if (moe_pack_upload_layer(pk, layer, wdev, wbytes, &w, (moe_stream_t)s) != 0) {
    std::fprintf(stderr, "%s\n", moe_pack_last_error(pk));
    return 1;
  }
  moe_pack_close(pk);
  CK(moe_check_shape(&w));

  const size_t ws_bytes = moe_workspace_bytes(&w, T);
  void* ws = nullptr;
  CK(cudaMalloc(&ws, ws_bytes));
  CK(moe_workspace_init(ws, ws_bytes, (moe_stream_t)s));

  const size_t n = (size_t)T * w.H;
  float* hidden = nullptr;
  uint16_t *attn = nullptr, *normed = nullptr;
  CK(cudaMalloc(&hidden, n * sizeof(float)));
  CK(cudaMalloc(&attn, n * sizeof(uint16_t)));
  CK(cudaMalloc(&normed, n * sizeof(uint16_t)));
  std::vector<float> h(n);
  std::vector<uint16_t> a16(n);
  const bool files = argc > 5;
  if (files) {
    FILE* f = std::fopen(argv[4], "rb");
    if (!f || std::fread(h.data(), sizeof(float), n, f) != n || std::fread(a16.data(), 2, n, f) != n) {
      std::fprintf(stderr, "cannot read %s\n", argv[4]);
      return 1;
    }
    std::fclose(f);
    CK(cudaMemcpyAsync(attn, a16.data(), n * 2, cudaMemcpyHostToDevice, s));
  } else {
    for (size_t i = 0; i < n; ++i) h[i] = std::sin(0.01f * (float)i);  // any finite residual
    CK(moe_synth_normal_bf16(attn, (int64_t)n, 1, 2, 0.f, 1.f, (moe_stream_t)s));
  }
  CK(cudaMemcpyAsync(hidden, h.data(), n * sizeof(float), cudaMemcpyHostToDevice, s));

  moe_stats before, after;
  moe_stats_get(&before);
  CK(moe_block_forward(&w, ws, ws_bytes, hidden, attn, normed, nullptr, T, (moe_stream_t)s));
  moe_stats_get(&after);
  CK(cudaMemcpyAsync(h.data(), hidden, n * sizeof(float), cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(a16.data(), normed, n * 2, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  CK(moe_workspace_error(ws, ws_bytes, (moe_stream_t)s));
  float mx = 0.f;
  for (float v : h) {
    if (!std::isfinite(v)) {
      std::fprintf(stderr, "non-finite output\n");
      return 1;
    }
    mx = std::fmax(mx, std::fabs(v));
  }
  if (files) {
    moe_trace tr;
    CK(moe_workspace_trace(&w, ws, ws_bytes, T, &tr));
    std::vector<float> lg((size_t)T * w.E);
    CK(cudaMemcpy(lg.data(), tr.logits, lg.size() * sizeof(float), cudaMemcpyDeviceToHost));
    FILE* f = std::fopen(argv[5], "wb");
    if (!f || std::fwrite(h.data(), sizeof(float), n, f) != n || std::fwrite(a16.data(), 2, n, f) != n ||
        std::fwrite(lg.data(), sizeof(float), lg.size(), f) != lg.size()) {
      std::fprintf(stderr, "cannot write %s\n", argv[5]);
      return 1;
    }
    std::fclose(f);
  }
  std::printf("ok T=%d launches=%llu max|hidden|=%g\n", T, (unsigned long long)(after.launches - before.launches), mx);
  cudaFree(hidden);
  cudaFree(attn);
  cudaFree(normed);
  cudaFree(ws);
  cudaFree(wdev);
  cudaStreamDestroy(s);
  return 0;
}
