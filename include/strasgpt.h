// strasgpt-b200 extensions to the transformer C ABI. None of these has a
// counterpart in the reference's include/transformer.h; each is optional for
// a caller that only uses the reference API.
#ifndef STRASGPT_H
#define STRASGPT_H

#include <stddef.h>
#include <stdint.h>

#include "transformer.h"

#ifdef __cplusplus
extern "C" {
#endif

// Device time of the last transformer_generate_greedy() call, measured with
// CUDA events on the library's stream.
typedef struct strasgpt_timing {
  double prefill_ms;      // prompt processing (all chunks)
  double decode_ms;       // all decode steps
  size_t prefill_tokens;
  size_t decode_steps;
  size_t kernel_launches; // kernels this call launched (graph nodes counted)
  size_t decode_launches; // of which in the decode steps (1: the persistent
                          // decode kernel ran all of them)
} strasgpt_timing_t;

// Greedy generation with the token loop kept on the GPU: process the
// `prompt_count` prompt tokens, then `step_count` decode steps, each fed the
// previous argmax (first index of the strict maximum, as the reference's
// sample_argmax, source/sampler.c:92-102). Writes step_count + 1 token ids
// to out_tokens (the first comes from the prompt's last logits). Appends to
// the KV cache like transformer_predict. Returns 0; dies on errors.
int transformer_generate_greedy(
    transformer_t* transformer,
    size_t prompt_count,
    const int* prompt,
    size_t step_count,
    int* out_tokens,
    strasgpt_timing_t* timing
);

// Forget the cached tokens (the next token goes to position 0).
void transformer_reset(transformer_t* transformer);

// Number of tokens currently in the KV cache.
size_t transformer_cached_count(const transformer_t* transformer);

// Tensor-parallel placement of this process: rank `rank` of `world` GPUs
// (world 1, 2, 4 or 8), on CUDA device `device`. Must be called before
// transformer_from_safetensors(); without it the environment variables
// STRASGPT_TP_RANK / STRASGPT_TP_SIZE / STRASGPT_DEVICE are read (default:
// rank 0 of 1 on device 0). world 0 clears an earlier placement (the
// environment is read again). Returns 0, or -1 on an invalid placement.
int strasgpt_set_placement(int rank, int world, int device);

// Tensor parallelism in ONE process (no counterpart in the reference, whose
// MPI split does no work): with STRASGPT_NGPU=N (2, 4 or 8) in the
// environment and no placement set, transformer_from_safetensors() builds N
// ranks on GPUs 0..N-1, connects them through direct peer access, and
// returns one transformer_t that runs every later call on all ranks (one
// host thread per rank) and answers with rank 0's results. The stock
// strasgpt.c therefore runs tensor-parallel with no change but the
// environment variable.

// Tensor parallelism, one process per GPU of one node. Each rank's
// transformer owns an exchange buffer in its GPU's memory; the ranks map
// each other's buffers (CUDA IPC over NVLink) and run one all-reduce after
// o_proj and one after the FFN of every layer, plus a gather of the
// vocabulary slices of the logits. The library does no host networking:
// the caller moves the handles. Every rank: build the transformer, write
// its STRASGPT_TP_HANDLE_BYTES handle with strasgpt_tp_handle(), exchange
// the handles (e.g. an all-gather), then call strasgpt_tp_connect() with
// all of them in rank order. All ranks must then make the same calls with
// the same tokens; each returns the full logits. Both return 0, or -1 when
// world is 1 or an argument is NULL.
#define STRASGPT_TP_HANDLE_BYTES 64
int strasgpt_tp_handle(transformer_t* transformer, void* handle);
int strasgpt_tp_connect(transformer_t* transformer, const void* handles);

// Per-kernel-family device time of the last profiled decode steps (see
// strasgpt_profile_decode). Families: 0 matvec, 1 attention, 2 qkv_post,
// 3 lm_head, 4 argmax, 5 other.
#define STRASGPT_KERNEL_FAMILIES 6
typedef struct strasgpt_kernel_profile {
  int launches[STRASGPT_KERNEL_FAMILIES];
  double ms[STRASGPT_KERNEL_FAMILIES];
  double bytes[STRASGPT_KERNEL_FAMILIES]; // algorithmic bytes moved
} strasgpt_kernel_profile_t;

// Run `step_count` greedy decode steps launching each kernel eagerly between
// CUDA events, and accumulate per-family device time and algorithmic bytes.
// The KV cache advances as in transformer_generate_greedy (the first step
// feeds `first_token`). Returns 0.
int strasgpt_profile_decode(
    transformer_t* transformer,
    int first_token,
    size_t step_count,
    strasgpt_kernel_profile_t* profile
);

#ifdef __cplusplus
}
#endif

#endif // STRASGPT_H
