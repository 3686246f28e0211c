// Persistent decode megakernel: one cooperative launch runs `steps` greedy
// decode steps of a dense model (all layers, LM head and argmax), one CTA per
// SM. Phases hand their outputs to the next phase through flagged vectors
// (every element a 64-bit word: value bits and the step's epoch), so a
// consumer waits for exactly the data it reads; there is no grid barrier.
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
  // Mixture of experts (null for a dense layer): the router [E][D] bf16 and
  // this rank's experts in MXFP4, codes [El][rows][K/2] (two per byte, low
  // nibble first) and e8m0 scales [El][rows][S] with S = K/32 rounded up to
  // 16 bytes (a row's scales start on a 16-byte boundary).
  const uint16_t* router;
  const uint8_t* gate_c;  // [El][Fe][D/2]
  const uint8_t* up_c;
  const uint8_t* down_c;  // [El][D][Fe/2]
  const uint8_t* gate_s;  // [El][Fe][S(D)]
  const uint8_t* up_s;
  const uint8_t* down_s;  // [El][D][S(Fe)]
};

// Offsets (in 64-bit words) of the flagged vectors inside MegaArgs::ll.
// Under tensor parallelism (world N > 1) the ranks write into each other's
// copies of `xpart` and `am` over NVLink.
struct MegaFlagged {
  size_t x;      // [L][2][D]     residual after o_proj (0) and after down (1)
  size_t qkv;    // [L][QKVl]
  size_t att;    // [L][QHl*HD]   merged attention output
  size_t h;      // [L][Fl]       SwiGLU output
  size_t xpart;  // [L][2][N][D]  every rank's partial o_proj / down rows (N > 1)
  size_t am;     // [2][N][grid]  per-CTA argmax value / global index of every rank
  size_t rec;    // [L][KHl][nsplit][G][HD+2]  attention split records (m, l, acc)
  size_t rl;     // [L][E]        router logits (MoE)
  size_t hm;     // [L][topk][Fe] SwiGLU outputs of the selected experts (MoE)
  size_t total;
};

MegaFlagged mega_flagged_layout(int D, int QKVl, int QD, int Fl, int L, int grid, int world,
                                int nsplit, int HD, int E, int topk, int Fe);

struct MegaArgs {
  int D, HD, QHl, KHl, G, Fl, Vl, L, QKVl, ctx;
  float eps;
  const MegaLayer* layers;  // device array [L]
  const uint16_t* emb;      // [V][D]
  const uint16_t* out_norm;
  const uint16_t* out_w;    // [Vl][D]
  const float* rope;        // [ctx][HD]
  int pair_bound, pair_offset, pair_stride;
  float* logits;            // [Vl]
  float* kc;                // [L][KHl][ctx][HD]
  float* vc;
  int nsplit, split_len;
  unsigned long long* ll;   // flagged vectors (layout: MegaFlagged)
  MegaFlagged llo;
  // Tensor parallelism: this rank of `world`, and every rank's `ll` as
  // mapped in this process (ll_peer[rank] == ll). world 1: ll_peer unused.
  int rank, world;
  unsigned long long* ll_peer[8];
  unsigned epoch;           // epoch of the first step; step s uses epoch + s
  int* tok;                 // in: token of the first step; out: last argmax
  int* pos;                 // in/out: position of the next token
  int* step;                // in/out: index into gen
  int* gen;                 // generated tokens
  int gen_len;              // capacity of gen: writes at step >= gen_len are dropped
  int* err;                 // set non-zero when a wait times out
  unsigned long long wait_ns;  // bound of every wait (ns)
  // Set by mega_decode: the ring's buffers (nbuf of buf_bytes) and the
  // activation's bf16 parts.
  int nbuf, buf_bytes, parts;
  long long layers_off;  // byte offset of the layer table in dynamic smem
  // Mixture of experts (moe != 0): E experts, topk chosen per token, expert
  // FFN width Fe, this rank owning experts [e_begin, e_end).
  int moe, E, topk, Fe, e_begin, e_end;
  int steps;
  int write_logits;
  // Optional (null = off): per phase and CTA, kMegaTraceWidth %globaltimer
  // records [phase][cta][w]: stage start, inputs complete, input staged,
  // first weight chunk ready, phase consumed, then the phase's ns spent
  // waiting for weight buffers, on its chunks in total, on warp 0's dot
  // products, and on the cross-warp sums and epilogues, then the times the
  // RMSNorm sum of squares was complete, the normalised input written and
  // the staging barrier passed, and the gains were resident; for the first
  // `trace_phases` phases.
  unsigned long long* trace;
  int trace_phases;
};

constexpr int kMegaTraceWidth = 13;

// Dynamic shared memory the megakernel needs for these dimensions (for a
// mixture of experts, Fl = 0, topk and Fe set; dense: topk = Fe = 0).
size_t mega_smem_bytes(int D, int QD, int Fl, int HD, int G, int L, int topk = 0, int Fe = 0);
// Largest grid that is co-resident (one CTA per SM); 0 if not launchable.
int mega_grid(size_t smem, int HD, int G);
// Decode split used by the megakernel (split_len a multiple of 64).
void mega_split(int ctx, int KHl, int grid, int* nsplit, int* split_len);
void mega_configure(size_t smem);
// Bytes of a row of e8m0 scales in the layout the kernel copies (K / 32
// rounded up to 16), and the copy of [rows][src_bytes] into that layout.
int mega_scale_row_bytes(int K);
void mega_pad_rows(const uint8_t* src, size_t rows, int src_bytes, int dst_bytes, uint8_t* dst,
                   cudaStream_t s);
void mega_decode(const MegaArgs& a, int grid, size_t smem, cudaStream_t s);

}  // namespace sg
