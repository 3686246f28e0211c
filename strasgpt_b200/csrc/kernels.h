// Launchers for the forward-pass kernels. All pointers are device pointers;
// every launch goes on `stream`. Shapes are checked on the host by the
// callers (transformer.cu); the kernels assume:
//   - row lengths (K) are multiples of 8 bf16 (16-byte rows),
//   - gate/up weights are interleaved row by row (gate row f at 2f, up row f
//     at 2f+1; SG_GU_GROUP = 1)
//     see the layout notes in
//     transformer.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define SG_GU_GROUP 1

namespace sg {

// Row of the gate weights of SwiGLU output i in the interleaved gate/up
// matrix; the matching up row is SG_GU_GROUP rows further.
__host__ __device__ __forceinline__ int gu_gate_row(int i) {
  return (i / SG_GU_GROUP) * (2 * SG_GU_GROUP) + i % SG_GU_GROUP;
}

enum Epilogue { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

// out[t][e] = bf16->f32(emb[tok[t]][e]) for t < T.
void embed(const int* tok, int T, const uint16_t* emb, int D, float* x,
           cudaStream_t s);

// y[t][:] = rmsnorm(x[t][:]) * w   (source/transformer.c:978-999).
void rmsnorm_rows(const float* x, int T, int D, const uint16_t* w, float eps,
                  float* y, cudaStream_t s);

// Single-token matvec y = W x with W bf16 [rows][K], x fp32 [K].
// norm_w != null: x is RMS-normalised (weights norm_w, eps) first.
// EPI_STORE: out[r] = y[r]; EPI_ADD: out[r] += y[r];
// EPI_SWIGLU: `rows` counts outputs; out[p] = swiglu(gate_p, up_p) with
// gate/up rows interleaved by SG_GU_GROUP.
void matvec(const float* x, const uint16_t* norm_w, float eps,
            const uint16_t* W, int K, int rows, float* out, Epilogue epi,
            cudaStream_t s);

// Multi-token projection C[t][n] (+)= sum_k A[t][k] W[n][k], fp32 A,
// bf16 W, fp32 accumulation (SIMT tiles). ldc is the row stride of C.
void gemm_simt(const float* A, int lda, const uint16_t* W, int K, int M,
               int N, float* C, int ldc, Epilogue epi, cudaStream_t s);

// Per-head q/k RMSNorm (optional) + RoPE, then scatter:
// q heads -> q[t][qh][HD]; k heads -> k_cache[kh][pos+t][HD];
// v heads -> v_cache[kh][pos+t][HD]. qkv rows are [QHl | KHl | KHl] heads.
struct QkvPostArgs {
  const float* qkv; int T; int QHl; int KHl; int HD;
  const uint16_t* q_norm; const uint16_t* k_norm; float eps;
  const float* rope;        // [ctx][HD]
  int pair_bound, pair_offset, pair_stride;
  const int* pos;           // device: position of token 0
  float* q;                 // [T][QHl][HD]
  float* k_cache;           // this layer: [KHl][ctx][HD]
  float* v_cache;
  int ctx;
};
void qkv_post(const QkvPostArgs& a, cudaStream_t s);

// Decode attention (one token) over cache rows [0, pos]:
// att[qh][HD] for the QHl heads, GQA group G = QHl/KHl. Split over the
// sequence in `nsplit` parts; the last CTA of each kv head merges them.
struct AttnDecodeArgs {
  const float* q;           // [QHl][HD]
  const float* k_cache;     // [KHl][ctx][HD]
  const float* v_cache;
  int KHl, G, HD, ctx;
  const int* pos;           // device
  int nsplit, split_len;
  float* partial;           // [KHl*G][nsplit][HD + 2]
  int* ticket;              // [KHl], zero at rest
  float* att;               // [QHl][HD]
};
void attn_decode(const AttnDecodeArgs& a, cudaStream_t s);
// Split of a `ctx`-row cache for attn_decode (<= 64 splits, each a multiple
// of 64 positions, about two CTAs per SM).
void attn_decode_split(int ctx, int KHl, int* nsplit, int* split_len);

// Causal prefill attention for T tokens at positions pos..pos+T-1 over
// cache rows [0, pos+t]. q [T][QHl][HD] -> att [T][QHl][HD].
struct AttnPrefillArgs {
  const float* q; const float* k_cache; const float* v_cache;
  int T, KHl, G, HD, ctx;
  int pos0;                 // host-known position of token 0
  float* att;
};
void attn_prefill(const AttnPrefillArgs& a, cudaStream_t s);
// The same on the tensor cores (attn_tc.cu): operands split into bf16 hi/lo
// halves, three mma.sync per product; attn_prefill uses it when supported.
bool attn_prefill_tc_supported(const AttnPrefillArgs& a);
void attn_prefill_tc(const AttnPrefillArgs& a, cudaStream_t s);
void attn_prefill_tc_configure();

// Greedy argmax over rows [0, n): first index of the strict maximum, as
// source/sampler.c:92-102. Writes *out_token, stores it at
// tokens_out[*step] when tokens_out is set and *step < tokens_len, advances
// *step by 1 and, when pos is not null, *pos by 1.
void argmax_advance(const float* logits, int n, int* out_token, int* pos,
                    int* step, int* tokens_out, int tokens_len,
                    float* partial_val, int* partial_idx, int* ticket,
                    cudaStream_t s);

// --- Mixture of experts (MXFP4 experts) ---------------------------------
// Router top-k: per token, the k largest logits (ties -> lower index),
// weights = softmax over the selected logits.
void moe_topk(const float* router_logits, int T, int E, int k, int* idx,
              float* weight, cudaStream_t s);

// h[t][j][f] = swiglu(gate_e[f] . xn[t], up_e[f] . xn[t]) for e=idx[t][j]
// with MXFP4 gate/up (codes [E][F][D/32][16], scales [E][F][D/32]).
// Experts outside [e_begin, e_end) produce zeros.
struct MoeArgs {
  const float* xn; int T; int D; int F; int k;
  const int* idx; const float* weight;
  const uint8_t* gate_codes; const uint8_t* gate_scales;
  const uint8_t* up_codes; const uint8_t* up_scales;
  const uint8_t* down_codes; const uint8_t* down_scales;
  int e_begin, e_end;       // owned experts (global ids)
  float* h;                 // [T][k][F]
  float* out;               // [T][D], EPI_ADD target
};
void moe_gate_up(const MoeArgs& a, cudaStream_t s);
// out[t][r] += sum_j weight[t][j] * (down_e[r] . h[t][j])
void moe_down(const MoeArgs& a, cudaStream_t s);

// --- Grouped experts for multi-token chunks ------------------------------
// Groups the `slots` = T*k (token, choice) slots by expert: counts[E],
// offsets[E] (exclusive prefix), perm[pos] = slot index with the slots of
// expert e at positions [offsets[e], offsets[e] + counts[e]), and
// inv[slot] = pos. The order inside an expert is unspecified (every row of
// an expert's product is computed independently of its position).
void moe_group(const int* idx, int slots, int E, int* counts, int* offsets, int* perm, int* inv,
               cudaStream_t s);
// bf16 halves (hi, lo as in tc_split) of the rows xn[perm[r] / k] for r < n.
void moe_gather_split(const float* xn, int D, const int* perm, int k, int n, uint16_t* hi,
                      uint16_t* lo, cudaStream_t s);
// bf16 rows from MXFP4 rows (codes [rows][K/32][16], scales [rows][K/32]):
// source row r goes to out row r * row_stride + row_offset ([*][K]); the
// values e2m1 * 2^(e8m0 - 127) are exact in bf16.
void mxfp4_to_bf16(const uint8_t* codes, const uint8_t* scales, int rows, int K, uint16_t* out,
                   int row_stride, int row_offset, cudaStream_t s);
// out[t][d] += sum over j (in order) of weight[t][j] * y[inv[t*k+j]][d], for
// the slots whose expert is in [e_begin, e_end).
void moe_combine(float* out, const float* weight, const int* idx, const int* inv, const float* y,
                 int T, int k, int D, int e_begin, int e_end, cudaStream_t s);

}  // namespace sg

namespace sg {
// Raise shared-memory limits of the kernels above; once per device, before
// the first launch or stream capture.
void configure_kernels();
// One-thread kernel that spins for `cycles` SM clocks (bounded).
void gpu_sleep_cycles(long long cycles, cudaStream_t s);
}  // namespace sg
