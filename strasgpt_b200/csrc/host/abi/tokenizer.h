// Layout mirror of StrasGPT's tokenizer_t (include/tokenizer.h:10-35 of the
// reference). parser_parse_tokenizer() fills a struct that the reference's
// source/tokenizer.c then owns and frees, so the layout must be identical.
// Only the struct is declared here: the tokenizer functions themselves stay
// in the host program (they are not part of the GPU library).
#ifndef TOKENIZER_H
#define TOKENIZER_H

#include <stdbool.h>
#include <stddef.h>
#include <stdio.h>

#define TOKENIZER_FILE             "tokenizer.json"
#define TOKENIZER_MAX_TOKEN_STRING 262144
#define TOKENIZER_MAX_BYTE_STRING  512

typedef struct {
  char* token_string;
  int id;
} tokenizer_index_t;

typedef struct tokenizer {
  size_t token_string_count;
  char* token_string[TOKENIZER_MAX_TOKEN_STRING];
  float score[TOKENIZER_MAX_TOKEN_STRING];
  tokenizer_index_t sorted_token_string[TOKENIZER_MAX_TOKEN_STRING];
  size_t max_token_string_len;
  unsigned char byte_string[TOKENIZER_MAX_BYTE_STRING];
  int bos_token_id;
  int eos_token_id;
} tokenizer_t;

#endif // TOKENIZER_H
