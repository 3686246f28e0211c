// Tensor-core (tcgen05 + TMA) projections for multi-token chunks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace sg {

// A row-major bf16 matrix [rows][K] described for TMA (64 x 128 boxes,
// 128-byte swizzle). `bytes` holds the driver's 128-byte CUtensorMap.
struct TcMap {
  alignas(64) unsigned char bytes[128];
  int rows = 0;
  int K = 0;
};

// K must be a multiple of 8 (16-byte rows) and base 16-byte aligned.
void tc_make_map(TcMap* m, const uint16_t* base, int rows, int K);

// hi[t][k] = bf16(x[t][k]), lo[t][k] = bf16(x[t][k] - hi[t][k]) for t < T
// (hi/lo rows of K elements, x rows `ldx` floats apart).
void tc_split(const float* x, int ldx, int T, int K, uint16_t* hi, uint16_t* lo,
              cudaStream_t s);

// C[t][r] (op)= sum_k (A_hi + A_lo)[t][k] W[r][k] for t < T, r < w.rows.
// For EPI_SWIGLU, w holds gate/up rows interleaved and C has w.rows/2
// columns. `err` (device int, zero at rest) is set if a pipeline wait times
// out; the caller checks it.
void tc_gemm(const TcMap& w, const TcMap& a_hi, const TcMap& a_lo, int T, float* C, int ldc,
             Epilogue epi, int* err, cudaStream_t s);

void tc_configure();

}  // namespace sg
