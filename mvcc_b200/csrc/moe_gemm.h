// moe_gemm.h -- host interface of the tcgen05 tile GEMM (moe_gemm.cu) behind the prefill path.
//
// D[m][n] = sum_k A[row(m)][k] * B[row(n)][k] over tiles of up to 128 or 256 A rows and BN B rows, K-major bf16 in
// shared memory (B optionally dequantized there from INT4), fp32 accumulators in TMEM, one of five epilogues.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

enum GemmEpi {
  EPI_F32 = 0,         // out fp32 [row][n]                                 (router logits, dense() fp32)
  EPI_BF16 = 1,        // out bf16 [row][n]                                 (shared down -> sout, dense() bf16)
  EPI_SILU_TILE = 2,   // paired gate/up: out bf16 = silu(g) * u            (routed gate/up -> inter)
  EPI_SILU_ROUND = 3,  // paired gate/up: out bf16 = silu(bf16 g) * bf16 u  (shared gate/up -> sinter)
  EPI_SLOT = 4,        // out fp32 [pair][n] = acc * row_scale[pair]        (routed down -> slot partials)
};

// One M tile of the grouped problem: B matrix (expert) e, first A row m0 (in the tile-row space), rows mcount
// (at most tile_rows: 128, or 256 for double tiles).
struct GemmTile {
  int e, m0, mcount, pad;
};

struct GemmParams {
  // A: bf16 rows of length K with row stride lda (elements). Tile row r reads A row
  //   a_rows ? a_rows[m0 + r] / a_div : m0 + r      (clamped to [0, a_nrows)).
  const uint16_t* A;
  int64_t lda;
  const int32_t* a_rows;
  int a_div;
  int a_nrows;
  int list_len;  // entries of a_rows / out_rows (indices into them are clamped)
  // B: rows of length K; expert e starts at row e * b_rows_per_e. Tile n-tile nt, row r reads B row
  //   paired ? (r < BN/2 ? nt*BN/2 + r : pair_off + nt*BN/2 + r - BN/2) : nt*BN + r.
  const uint16_t* Bh;  // bf16 [rows][K], or
  const uint8_t* Bq;   // INT4 [rows][K/2] (low nibble = even k)
  const uint16_t* Bs;  // fp16 scales [rows][K/G]
  int64_t b_rows_per_e;
  int paired, pair_off;
  int N, K, G, E;
  int n_valid;  // unpaired B: rows (and output columns) >= n_valid are zero / not written (N padded up to BN)
  // Tiles: a device list (grouped problems, count in *ntiles) or, when tiles == nullptr, dense M tiles over M rows.
  const GemmTile* tiles;
  const int* ntiles;
  int M;
  // Epilogue
  void* out;
  int64_t ldo;               // elements
  const int32_t* out_rows;   // EPI_SLOT: out row = out_rows[m0 + r]
  const float* row_scale;    // EPI_SLOT: scale = row_scale[out row]
  const float* col_bias;     // EPI_F32 (nullable): out = acc + col_bias[column]
  int out_nrows;             // bound of out rows (clamp)
  uint32_t* err;             // error word (bounded waits)
};

// Persistent launch over min(SMs, max_tiles x N/BN) CTAs; work item i = (tile i / (N/BN), n-tile i % (N/BN)),
// items past *ntiles x N/BN are skipped. bn in {64, 128, 256}; tile_rows is the row count the tile list was built
// with (or of the dense M tiles): 128, or 256 (two 128-row sub-tiles per dequantised B stage; INT4 at bn = 256 with
// the EPI_SILU_TILE or EPI_SLOT epilogue only); int4 selects the INT4 B path. pdl: launched as a programmatic
// dependent of the previous kernel on the stream (its prologue overlaps that kernel's tail). Returns
// cudaErrorInvalidValue for unsupported parameters.
cudaError_t launch_gemm(const GemmParams& p, int epi, int bn, int tile_rows, bool int4, int max_tiles, bool pdl,
                        cudaStream_t s);

}  // namespace moe
