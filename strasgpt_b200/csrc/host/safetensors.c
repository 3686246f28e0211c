// safetensors_t helpers with the API of StrasGPT's source/safetensors.c,
// plus the U8 dtype used by MXFP4 expert tensors.
#include "safetensors.h"

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

const char* safetensors_type_str[] = {"F16", "BF16", "F32", "U8"};

// Prefix of the host program's options_t up to model_dir: the layout of the
// reference's include/options.h:18-23 (safetensors_read only needs the
// model directory).
struct options_prefix {
  bool use_prompt_file;
  char* prompt_file;
  char* prompt_string;
  bool pre_tokenized;
  char* model_dir;
};

static void die(const char* msg) {
  fprintf(stderr, "[StrasGPT] Error: %s\n", msg);
  exit(EXIT_FAILURE);
}

safetensors_t* safetensors_malloc(void) {
  safetensors_t* s = calloc(1, sizeof(*s));
  if (!s) {
    die("failed to malloc for safetensors_t");
  }
  return s;
}

void safetensors_free(safetensors_t* s) {
  if (!s) {
    return;
  }
  free(s->model_type);
  for (size_t i = 0; i < s->file_count; i++) {
    free(s->file[i]);
  }
  for (size_t i = 0; i < s->tensor_count; i++) {
    free(s->tensor[i].name);
  }
  free(s);
}

safetensors_t* safetensors_read(struct options* options) {
  if (!options) {
    die("NULL options for safetensors_read");
  }
  return parser_parse_safetensors(((struct options_prefix*)options)->model_dir);
}

safetensors_type_t safetensors_type_from_string(const char* s) {
  if (!s) {
    die("NULL string for safetensors_type_from_string");
  }
  for (size_t i = 0; i < 4; i++) {
    if (strcmp(s, safetensors_type_str[i]) == 0) {
      return (safetensors_type_t)i;
    }
  }
  die("unknown data type");
  return SAFETENSORS_TYPE_F32;
}

void safetensors_file_lookup(safetensors_t* s, char* path, char* file) {
  char full[SAFETENSORS_MAX_STRING];
  snprintf(full, sizeof(full), "%s/%s", path, file);
  for (size_t i = 0; i < s->file_count; i++) {
    if (strcmp(s->file[i], full) == 0) {
      return;
    }
  }
  if (s->file_count >= SAFETENSORS_MAX_FILE_COUNT) {
    die("too many safetensors files");
  }
  s->file[s->file_count++] = strdup(full);
}

size_t safetensors_sizeof(safetensors_type_t type) {
  switch (type) {
    case SAFETENSORS_TYPE_F16:
    case SAFETENSORS_TYPE_BF16:
      return 2;
    case SAFETENSORS_TYPE_F32:
      return 4;
    case SAFETENSORS_TYPE_U8:
      return 1;
  }
  die("unknown safetensors type");
  return 0;
}

// The LM head is tied to the embedding when "lm_head.weight" is absent
// (source/safetensors.c:421-429).
bool safetensors_aliased_out_weight(const safetensors_t* s) {
  for (size_t i = 0; i < s->tensor_count; i++) {
    if (strcmp(s->tensor[i].name, SAFETENSORS_PATTERN_OUT_WEIGHT) == 0) {
      return false;
    }
  }
  return true;
}

static void print_config(FILE* f, const safetensors_t* s) {
  fprintf(f, "--- model_type:       %s\n", s->model_type ? s->model_type : "(null)");
  fprintf(f, "--- embedding_dim:    %zu\n", s->embedding_dim);
  fprintf(f, "--- head_dim:         %zu\n", s->head_dim);
  fprintf(f, "--- hidden_dim:       %zu\n", s->hidden_dim);
  fprintf(f, "--- layer_count:      %zu\n", s->layer_count);
  fprintf(f, "--- q_head_count:     %zu\n", s->q_head_count);
  fprintf(f, "--- kv_head_count:    %zu\n", s->kv_head_count);
  fprintf(f, "--- vocabulary_len:   %zu\n", s->vocabulary_len);
  fprintf(f, "--- context_len:      %zu\n", s->context_len);
  fprintf(f, "--- epsilon:          %g\n", s->epsilon);
  fprintf(f, "--- rope_theta:       %.1f\n", s->rope_theta);
  fprintf(f, "--- rope_interleaved: %s\n", s->rope_interleaved ? "true" : "false");
  fprintf(f, "--- expert_count:     %zu (top-%zu)\n", s->expert_count, s->expert_top_k);
  fprintf(f, "--- bos_token_id:     %d\n", s->bos_token_id);
  fprintf(f, "--- eos_token_id:     %d\n", s->eos_token_id);
}

void safetensors_print(FILE* f, const safetensors_t* s) {
  if (!s) {
    fprintf(f, "safetensors: NULL\n");
    return;
  }
  fprintf(f, "Safetensors:\n- Configuration:\n");
  print_config(f, s);
  fprintf(f, "- Files (%zu):\n", s->file_count);
  for (size_t i = 0; i < s->file_count; i++) {
    fprintf(f, "--- File[%zu]: %s\n", i, s->file[i]);
  }
  fprintf(f, "- Tensors (%zu):\n", s->tensor_count);
  for (size_t i = 0; i < s->tensor_count; i++) {
    const safetensors_tensor_t* t = &s->tensor[i];
    fprintf(f, "--- Tensor[%zu]: name=%s type=%s dim=[", i, t->name,
            safetensors_type_str[t->type]);
    for (size_t d = 0; d < t->dim_count; d++) {
      fprintf(f, "%zu%s", t->dim[d], d + 1 < t->dim_count ? ", " : "");
    }
    fprintf(f, "] size=%zu file=%zu offset=%zu\n", t->size, t->file, t->offset);
  }
}

void safetensors_print_model_infos(FILE* f, const safetensors_t* s) {
  if (!s) {
    fprintf(f, "model: NULL\n");
    return;
  }
  fprintf(f, "Model:\n- Configuration:\n");
  print_config(f, s);
  double bytes = 0;
  for (size_t i = 0; i < s->tensor_count; i++) {
    bytes += (double)s->tensor[i].size;
  }
  fprintf(f, "- Tensors: %zu (%.2f GB)%s\n", s->tensor_count,
          bytes / (1024.0 * 1024.0 * 1024.0),
          safetensors_aliased_out_weight(s) ? ", LM head tied to embedding" : "");
}
