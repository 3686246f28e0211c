// Tensor-core (tcgen05 + TMA) projections for multi-token chunks.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace sg {

// A row-major bf16 matrix [rows][K] described for TMA (boxes of 64 x
// box_rows elements, 128-byte swizzle). `bytes` holds the driver's 128-byte
// CUtensorMap.
struct TcMap {
  alignas(64) unsigned char bytes[128];
  int rows = 0;
  int K = 0;
  int box_rows = 0;
};

// The bf16 halves of a projection input, [rows][K] each, with one map per
// token-tile width (32, 64, 128).
struct TcAct {
  TcMap hi[3], lo[3];
  const uint16_t* hi_base = nullptr;
  const uint16_t* lo_base = nullptr;
};

// Weight matrix [rows][K]: K a multiple of 8 (16-byte rows), base 16-byte
// aligned.
void tc_make_map(TcMap* m, const uint16_t* base, int rows, int K);
void tc_make_act(TcAct* a, const uint16_t* hi, const uint16_t* lo, int rows, int K);

// hi[t][k] = bf16(x[t][k]), lo[t][k] = bf16(x[t][k] - hi[t][k]) for t < T
// (hi/lo rows of K elements, x rows `ldx` floats apart; K, ldx multiples of
// 4, x 16-byte aligned).
void tc_split(const float* x, int ldx, int T, int K, uint16_t* hi, uint16_t* lo,
              cudaStream_t s);

// C[t][r] (op)= sum_k (A_hi + A_lo)[t][k] W[r][k] for t < T, r < w.rows.
// For EPI_SWIGLU, w holds gate/up rows interleaved and C has w.rows/2
// columns. `err` (device int, zero at rest) is set if a pipeline wait times
// out; the caller checks it. `w_early`: no kernel launched before this one
// on the stream writes w (model weights), so its first tiles may be
// requested before the wait for that kernel; false when an earlier kernel
// produces w (dequantised experts, caller-owned buffers).
void tc_gemm(const TcMap& w, const TcAct& a, int T, float* C, int ldc, Epilogue epi, int* err,
             cudaStream_t s, bool w_early = true);

// Token-tile width tc_gemm uses for `rows` weight rows and T tokens.
int tc_width(int rows, int T);

void tc_configure();

}  // namespace sg
