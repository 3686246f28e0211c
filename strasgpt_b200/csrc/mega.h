// Persistent decode megakernel: one cooperative launch runs `steps` greedy
// decode steps of a dense model (all layers, LM head and argmax), one CTA per
// SM, phases separated by grid-wide barriers with bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sg {

struct MegaLayer {
  const uint16_t* attn_norm;
  const uint16_t* wqkv;   // [QKVl][D]
  const uint16_t* q_norm; // [HD] or null
  const uint16_t* k_norm;
  const uint16_t* wo;     // [D][QHl*HD]
  const uint16_t* ffn_norm;
  const uint16_t* wgu;    // [2*Fl][D], gate/up rows interleaved
  const uint16_t* wd;     // [D][Fl]
};

struct MegaArgs {
  int D, HD, QHl, KHl, G, Fl, Vl, L, QKVl, ctx;
  float eps;
  const MegaLayer* layers;  // device array [L]
  const uint16_t* emb;      // [V][D]
  const uint16_t* out_norm;
  const uint16_t* out_w;    // [Vl][D]
  const float* rope;        // [ctx][HD]
  int pair_bound, pair_offset, pair_stride;
  float* x;                 // [D] residual stream
  float* qkv;               // [QKVl]
  float* att;               // [QHl*HD]
  float* h;                 // [Fl]
  float* logits;            // [Vl]
  float* kc;                // [L][KHl][ctx][HD]
  float* vc;
  float* attn_partial;      // [QHl][nsplit][HD+2]
  int* attn_ticket;         // [KHl], zero at rest
  int nsplit, split_len;
  float* am_val;            // [gridDim] argmax partials
  int* am_idx;
  int* tok;                 // in: token of the first step; out: last argmax
  int* pos;                 // in/out: position of the next token
  int* step;                // in/out: index into gen
  int* gen;                 // generated tokens
  int gen_len;              // capacity of gen: writes at step >= gen_len are dropped
  unsigned* bar;            // [2] barrier count / generation, zero at rest
  int* err;                 // set non-zero when a barrier wait times out
  int steps;
  int write_logits;
  // Optional (null = off): per barrier and CTA, kMegaTraceWidth %globaltimer
  // stamps [barrier][cta][w]: arrival, release, input staged, first weight
  // chunk ready, phase consumed, last chunk computed, next copy issued; for
  // the first `trace_barriers` barriers.
  unsigned long long* trace;
  int trace_barriers;
};

constexpr int kMegaTraceWidth = 7;

// Dynamic shared memory the megakernel needs for these dimensions.
size_t mega_smem_bytes(int D, int QD, int Fl, int HD, int G);
// Largest grid that is co-resident (one CTA per SM); 0 if not launchable.
int mega_grid(size_t smem, int HD, int G);
// Decode split used by the megakernel (split_len a multiple of 128).
void mega_split(int ctx, int KHl, int grid, int* nsplit, int* split_len);
void mega_configure(size_t smem);
void mega_decode(const MegaArgs& a, int grid, size_t smem, cudaStream_t s);

}  // namespace sg
