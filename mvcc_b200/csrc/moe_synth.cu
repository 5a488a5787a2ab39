// moe_synth.cu -- seeded synthetic weights and activations in the reference's layout, generated on the device.
//
// The reference reads real GPTQ checkpoints (convert.py); the benchmark and the full-size tests instead fill the
// same buffers from a counter-based generator: splitmix64 over (seed, stream, element index) gives two uniforms,
// Box-Muller turns them into N(0,1), the result is rounded to bf16. INT4 rows are then quantized per group of G
// along K with scale = fp16(absmax / 7) and q = clamp(rint(w / scale), -7, 7) + 8, the 4-bit analogue of
// convert.py's int8 quantizer (convert.py:162-169).
#include <algorithm>

#include "moe_common.cuh"

namespace moe {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// N(0,1) sample number i of stream (seed, sid).
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t sid, uint64_t i) {
  const uint64_t r = splitmix64(splitmix64(seed ^ (sid * 0xD1B54A32D192ED03ull)) + i);
  const float u1 = ((float)(uint32_t)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
  const float u2 = (float)(uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);     // [0, 1)
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void synth_normal_bf16_kernel(uint16_t* out, int64_t n, uint64_t seed, uint64_t sid, float mean,
                                         float std) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f2bf(mean + std * normal_at(seed, sid, (uint64_t)i));
}

// One thread per (row, group): G bf16 samples, absmax scale, packed nibbles (low nibble = even k).
__global__ void synth_int4_rows_kernel(uint8_t* q, uint16_t* scales, int64_t rows, int K, int G, uint64_t seed,
                                       uint64_t sid, float std) {
  const int groups = K / G;
  const int64_t total = rows * groups;
  for (int64_t job = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; job < total;
       job += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = job / groups;
    const int grp = (int)(job - row * groups);
    const uint64_t base = (uint64_t)row * K + (uint64_t)grp * G;
    float amax = 0.f;
    for (int k = 0; k < G; ++k) amax = fmaxf(amax, fabsf(bf2f(f2bf(std * normal_at(seed, sid, base + k)))));
    const uint16_t sh = __half_as_ushort(__float2half_rn(amax / 7.0f));
    const float s = __half2float(__ushort_as_half(sh));
    scales[job] = sh;
    uint8_t* qrow = q + (int64_t)row * (K / 2) + grp * (G / 2);
    for (int k = 0; k < G; k += 2) {
      int qq[2];
      for (int j = 0; j < 2; ++j) {
        const float w = bf2f(f2bf(std * normal_at(seed, sid, base + k + j)));
        int v = s > 0.f ? (int)rintf(w / s) : 0;
        v = v < -7 ? -7 : (v > 7 ? 7 : v);
        qq[j] = v + 8;
      }
      qrow[k / 2] = (uint8_t)(qq[0] | (qq[1] << 4));
    }
  }
}

}  // namespace moe

extern "C" {

int moe_synth_normal_bf16(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream_id, float mean, float std,
                          moe_stream_t stream) {
  if (!out || n < 0) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  moe::synth_normal_bf16_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(out, n, seed, stream_id, mean, std);
  return (int)moe::launched(cudaGetLastError());
}

int moe_synth_int4_rows(uint8_t* q, uint16_t* scales, int64_t rows, int K, int G, uint64_t seed, uint64_t stream_id,
                        float std, moe_stream_t stream) {
  if (!q || !scales || rows < 0 || K <= 0 || G <= 0 || K % G || G % 2) return (int)cudaErrorInvalidValue;
  if (rows == 0) return 0;
  const int64_t jobs = rows * (K / G);
  const int grid = (int)std::min<int64_t>((jobs + 255) / 256, 148 * 32);
  moe::synth_int4_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(q, scales, rows, K, G, seed, stream_id, std);
  return (int)moe::launched(cudaGetLastError());
}

}  // extern "C"
