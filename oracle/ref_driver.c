// ORACLE — test infrastructure only (see oracle/strasgpt_oracle.c).
//
// A thin driver around the REFERENCE implementation, compiled together with
// the reference's own source/transformer.c, source/safetensors.c and
// source/util.c (unmodified, from the reference tree) by oracle/Makefile into
// oracle/_ref/. It exists because the reference's transformer_predict must
// be called by every thread of an OpenMP team (source/strasgpt.c:209-232):
// these wrappers open that team, the way strasgpt.c does.
#include "safetensors.h"
#include "transformer.h"

#include <stdio.h>
#include <stdlib.h>

typedef struct {
  safetensors_t* st;
  transformer_t* tr;
} ref_handle_t;

safetensors_t* parser_parse_safetensors(const char* path);

void* ref_load(const char* dir) {
  ref_handle_t* h = calloc(1, sizeof(*h));
  h->st = parser_parse_safetensors(dir);
  h->tr = transformer_from_safetensors(h->st);
  return h;
}

int ref_vocab(void* p) {
  return (int)((ref_handle_t*)p)->tr->config->vocabulary_len;
}

size_t ref_cached(void* p) {
  return ((ref_handle_t*)p)->tr->state->cached_count;
}

void ref_reset(void* p) { ((ref_handle_t*)p)->tr->state->cached_count = 0; }

void ref_predict(void* p, size_t n, int* tok, size_t logits_count,
                 float* logits) {
  ref_handle_t* h = p;
#pragma omp parallel
  transformer_predict(h->tr, n, tok, logits_count, logits);
}

void ref_free(void* p) {
  ref_handle_t* h = p;
  transformer_free(h->tr);
  safetensors_free(h->st);
  free(h);
}
