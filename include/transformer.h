// strasgpt-b200: the transformer forward pass as a C ABI over CUDA (sm_100a).
//
// This header is the drop-in boundary. It keeps the names, argument meaning
// and error behaviour of StrasGPT's include/transformer.h:87-99 so that
// source/strasgpt.c and source/sampler.c compile and link against it
// unchanged:
//   - transformer_t keeps its three members; sampler_build reads
//     transformer->config->vocabulary_len (source/sampler.c:27), so
//     transformer_configuration_t is kept field-for-field.
//   - weights and state live in GPU memory; their structs are opaque here.
//   - errors print "[StrasGPT] Error ..." and exit(EXIT_FAILURE), as the
//     reference's UTIL_DIE does (include/util.h:9-26).
#ifndef TRANSFORMER_H
#define TRANSFORMER_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#ifdef __cplusplus
extern "C" {
#endif

struct safetensors;

// Kept for source compatibility (include/transformer.h:9 of the reference).
// The GPU path is not limited to this chunk length: it sizes its own chunks.
#define TRANSFORMER_CHUNK_MAX_LEN 512

// Model hyperparameters: same fields, same order as the reference
// (include/transformer.h:11-28).
typedef struct transformer_configuration {
  size_t embedding_dim;       // token representation dimension (D)
  size_t head_dim;            // per-head dimension (HD)
  size_t hidden_dim;          // FFN intermediate dimension (F)
  size_t layer_count;         // decoder layers (L)
  size_t q_head_count;        // query heads (QH)
  size_t kv_head_count;       // key/value heads (KH)
  size_t vocabulary_len;      // vocabulary size (V)
  size_t context_len;         // maximum sequence length (KV cache rows)
  float epsilon;              // RMSNorm epsilon
  float rope_theta;           // RoPE base frequency
  size_t rope_pair_bound;     // interleaved: head_dim, half-split: head_dim/2
  size_t rope_pair_offset;    // interleaved: 1, half-split: head_dim/2
  size_t rope_pair_stride;    // interleaved: 2, half-split: 1
  size_t mrope_section_count; // multi-scale RoPE sections (0 if none)
  size_t* mrope_section;      // parsed, unused by the math (as in the reference)
  bool aliased_out_weight;    // LM head shares the embedding matrix
} transformer_configuration_t;

// Device-resident weights and state (opaque to callers).
typedef struct transformer_weights transformer_weights_t;
typedef struct transformer_state transformer_state_t;

typedef struct transformer {
  transformer_configuration_t* config; // hyperparameters (host memory)
  transformer_weights_t* weights;      // device weights (opaque)
  transformer_state_t* state;          // device KV cache + activations (opaque)
} transformer_t;

// Build a transformer from parsed safetensors metadata: reads every tensor
// from disk and uploads it to the GPU(s). The caller keeps `safetensors`
// alive until this returns. Replaces source/transformer.c:732-740.
transformer_t* transformer_from_safetensors(struct safetensors* safetensors);

// Release every host and device resource. NULL is a no-op.
// Replaces source/transformer.c:743-791.
void transformer_free(transformer_t* transformer);

// Print the configuration and weight sizes. Replaces
// source/transformer.c:877-954.
void transformer_print(FILE* f, const transformer_t* transformer);

// malloc() a host logits buffer of logits_count rows of vocabulary_len
// floats and report vocabulary_len. The caller releases it with free().
// Replaces source/transformer.c:956-970.
float* transformer_logits_malloc(
    transformer_t* transformer, size_t logits_count, size_t* vocabulary_len
);

// Append token_count tokens at position cached_count and write the logits
// of the last min(logits_count, token_count) of them, row-major
// [rows][vocabulary_len], into the host buffer `logits`. No-op on NULL
// transformer/logits or zero counts; dies when the context is exhausted.
// May be called by every thread of an OpenMP team (strasgpt.c does): one
// thread drives the GPU and all threads see the logits on return.
// Replaces source/transformer.c:1607-1727.
void transformer_predict(
    transformer_t* transformer,
    size_t token_count,
    int* token,
    size_t logits_count,
    float* logits
);

#ifdef __cplusplus
}
#endif

#endif // TRANSFORMER_H
