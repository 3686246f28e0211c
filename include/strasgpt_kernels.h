// strasgpt-b200 kernel-level entry points, for unit tests and for callers
// that manage their own device buffers. All pointers are DEVICE pointers;
// `stream` is a cudaStream_t (NULL: the legacy default stream). Each call
// only enqueues work; it returns 0, or dies with "[StrasGPT] Error ..." on an
// invalid shape. None of these has a counterpart in the reference API: they
// expose the pieces of transformer_predict_chunk (source/transformer.c:
// 1186-1602) one at a time.
#ifndef STRASGPT_KERNELS_H
#define STRASGPT_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Epilogue selector shared by the projection entry points.
#define STRASGPT_EPI_STORE  0  // out = W x
#define STRASGPT_EPI_ADD    1  // out += W x (residual)
#define STRASGPT_EPI_SWIGLU 2  // out = silu(gate) * up, gate/up rows interleaved

// y = W x for one token: W bf16 [rows][K] (rows of K contiguous), x fp32
// [K]. norm_w (bf16 [K]) != NULL applies the reference RMSNorm to x first
// (source/transformer.c:978-999). For STRASGPT_EPI_SWIGLU `rows` counts
// outputs and W holds 2*rows rows: gate row f at 2f, up row f at 2f+1.
int strasgpt_k_matvec(const float* x, const uint16_t* norm_w, float eps,
                      const uint16_t* w, int k, int rows, float* out, int epi,
                      void* stream);

// C[m][n] (op)= sum_k A[m][k] W[n][k] for m < M, n < N (SIMT fp32 tiles).
// For STRASGPT_EPI_SWIGLU, N counts weight rows and C has N/2 columns.
int strasgpt_k_gemm_simt(const float* a, int lda, const uint16_t* w, int k,
                         int m, int n, float* c, int ldc, int epi,
                         void* stream);

// Same product as strasgpt_k_gemm_simt on the tcgen05 tensor cores: A is
// split into bf16 halves a_hi + a_lo (caller-provided [m][k] buffers,
// 16-byte aligned, k a multiple of 8) and both are multiplied with W in fp32
// accumulation. `err` is a device int, zero at rest, set non-zero if the
// kernel's pipeline waits time out (C is then incomplete).
int strasgpt_k_gemm_tc(const float* a, int lda, uint16_t* a_hi,
                       uint16_t* a_lo, const uint16_t* w, int k, int m, int n,
                       float* c, int ldc, int epi, int* err, void* stream);

// Causal GQA attention of a chunk (source/transformer.c:1375-1422): q
// [t][kv_heads*group][head_dim] at positions pos0.., caches
// [kv_heads][ctx][head_dim] holding keys/values 0..pos0+t-1; att gets
// [t][kv_heads*group][head_dim]. head_dim 32, 64 or 128; group divides 64.
int strasgpt_k_attn_prefill(const float* q, const float* k_cache,
                            const float* v_cache, int t, int kv_heads,
                            int group, int head_dim, int ctx, int pos0,
                            float* att, void* stream);

// y[t] = rmsnorm(x[t]) * w for t < T, rows of D floats.
int strasgpt_k_rmsnorm_rows(const float* x, int t, int d, const uint16_t* w,
                            float eps, float* y, void* stream);

// The error path of the device-side waits, for tests (no counterpart in the
// reference): runs the tensor-parallel barrier kernel of a 2-rank exchange
// on the current GPU whose second rank is a buffer that nothing writes
// (peer_posted 0: the wait can only run out) or whose post is already in
// place (peer_posted 1), with a wait limit of timeout_ms. Returns 1 when
// the wait ran out and the kernel returned with its error flag set, 0 when
// it completed, -1 on a bad argument. The GPU stays usable either way.
int strasgpt_k_tp_wait_check(int timeout_ms, int peer_posted, void* stream);

// Size of the fixed device scratch of strasgpt_k_matvec_noalloc, held by
// every GPU that loads the library until the process exits.
#define STRASGPT_NOALLOC_SCRATCH_BYTES (4 << 20)

// strasgpt_k_matvec without any allocation, for callers that own all of the
// GPU's memory through their own pools or cannot stall the device with
// cudaMalloc/cudaFree between decode steps. No counterpart in the reference:
// it is an extra way in to the same projection. Same arguments and result as
// strasgpt_k_matvec (computed split-K: fp32 sums in another order); x, w and
// norm_w must be 16-byte aligned. Its scratch is a fixed 4 MiB device array:
// the weight rows (2*rows for STRASGPT_EPI_SWIGLU) may be at most
// STRASGPT_NOALLOC_SCRATCH_BYTES / 4 - 64 = 1048512; larger shapes, and
// other invalid arguments, return -1 with a message on stderr and enqueue
// nothing. The first call on a device looks up the scratch's address, so
// make it before any stream capture on that device. All calls on a device
// share the scratch: calls that overlap on the GPU race, so serialise them
// (one stream). Returns 0 once the work is enqueued.
int strasgpt_k_matvec_noalloc(const float* x, const uint16_t* norm_w,
                              float eps, const uint16_t* w, int k, int rows,
                              float* out, int epi, void* stream);

#ifdef __cplusplus
}
#endif

#endif // STRASGPT_KERNELS_H
