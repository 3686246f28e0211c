// Model-directory reader: config.json, model.safetensors.index.json, the
// safetensors headers and tokenizer.json.
//
// The reference generates these entry points from a yacc grammar and a lex
// scanner (source/json_parser.y:526-648, source/json_scanner.l), which need
// lex/yacc to build. This file provides the same three symbols in plain C:
//   parser_parse_safetensors(path)  source/json_parser.y:526-622
//   parser_parse_tokenizer(path)    source/json_parser.y:626-648
//   json_scanner_lex_destroy()      called by source/strasgpt.c:286
// and fills the structs the same way: which config keys are read (and inside
// "text_config"), the head_dim default, the file list order, tensor offsets
// (8 + header length + begin), and raw (unescaped) token strings scored by
// their id.
//
// It compiles against either this library's safetensors.h (which adds the
// U8 dtype and the expert fields) or the reference's own header.
#include "safetensors.h"
#include "tokenizer.h"

#include "json.h"

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static void parse_die(const json_value_t* v, const char* msg) {
  fprintf(
      stderr,
      "[StrasGPT] Error: line %zu: %s\n",
      v ? v->line : (size_t)0,
      msg
  );
  exit(EXIT_FAILURE);
}

static long long want_int(const json_value_t* v, const char* what) {
  // eos_token_id may be a list in recent configs: take its first entry.
  if (v->kind == JSON_ARRAY && v->count > 0) {
    v = &v->item[0];
  }
  if (v->kind != JSON_NUMBER || !v->is_int) {
    char msg[256];
    snprintf(msg, sizeof(msg), "non integer %s value", what);
    parse_die(v, msg);
  }
  return v->ival;
}

static double want_number(const json_value_t* v, const char* what) {
  if (v->kind != JSON_NUMBER) {
    char msg[256];
    snprintf(msg, sizeof(msg), "expected a number for %s", what);
    parse_die(v, msg);
  }
  return v->fval;
}

// Members of config.json the forward pass needs
// (source/json_parser.y:81-189, keys from source/json_scanner.l:26-50).
static void apply_config(safetensors_t* s, const json_value_t* obj) {
  if (obj->kind != JSON_OBJECT) {
    parse_die(obj, "config: expected an object");
  }
  for (size_t i = 0; i < obj->count; i++) {
    const char* k = obj->key[i];
    const json_value_t* v = &obj->item[i];
    if (strcmp(k, "bos_token_id") == 0) {
      if (v->kind != JSON_NULL) {
        s->bos_token_id = (int)want_int(v, "BOS token id");
      }
    } else if (strcmp(k, "eos_token_id") == 0) {
      if (v->kind != JSON_NULL) {
        s->eos_token_id = (int)want_int(v, "EOS token id");
      }
    } else if (strcmp(k, "hidden_size") == 0) {
      s->embedding_dim = (size_t)want_int(v, "embedding_dim");
    } else if (strcmp(k, "head_dim") == 0) {
      s->head_dim = (size_t)want_int(v, "head_dim");
    } else if (strcmp(k, "intermediate_size") == 0) {
      s->hidden_dim = (size_t)want_int(v, "hidden_dim");
    } else if (strcmp(k, "num_hidden_layers") == 0) {
      s->layer_count = (size_t)want_int(v, "layer_count");
    } else if (strcmp(k, "model_type") == 0) {
      if (v->kind != JSON_STRING) {
        parse_die(v, "model_type: expected a string");
      }
      free(s->model_type);
      s->model_type = strdup(v->string);
    } else if (strcmp(k, "num_attention_heads") == 0) {
      s->q_head_count = (size_t)want_int(v, "q_head_count");
    } else if (strcmp(k, "num_key_value_heads") == 0) {
      s->kv_head_count = (size_t)want_int(v, "kv_head_count");
    } else if (strcmp(k, "vocab_size") == 0) {
      s->vocabulary_len = (size_t)want_int(v, "vocabulary_len");
    } else if (strcmp(k, "max_position_embeddings") == 0) {
      s->context_len = (size_t)want_int(v, "context_len");
    } else if (strcmp(k, "rms_norm_eps") == 0) {
      s->epsilon = (float)want_number(v, "rms_norm_eps");
    } else if (strcmp(k, "rope_theta") == 0) {
      s->rope_theta = (float)want_number(v, "rope_theta");
    } else if (strcmp(k, "rope_scaling") == 0) {
      if (v->kind == JSON_NULL) {
        continue;
      }
      if (v->kind != JSON_OBJECT) {
        parse_die(v, "rope_scaling: expected an object or null");
      }
      for (size_t j = 0; j < v->count; j++) {
        const json_value_t* m = &v->item[j];
        if (strcmp(v->key[j], "mrope_interleaved") == 0) {
          if (m->kind != JSON_BOOL) {
            parse_die(m, "mrope_interleaved: expected a boolean");
          }
          s->rope_interleaved = m->boolean;
        } else if (strcmp(v->key[j], "mrope_section") == 0) {
          if (m->kind != JSON_ARRAY) {
            parse_die(m, "mrope_section: expected a list");
          }
          for (size_t e = 0; e < m->count; e++) {
            if (s->mrope_section_count >= SAFETENSORS_MAX_MROPE_SECTION_COUNT) {
              parse_die(m, "too many mrope sections");
            }
            s->mrope_section[s->mrope_section_count++] =
                (size_t)want_int(&m->item[e], "mrope section");
          }
        }
      }
    } else if (strcmp(k, "text_config") == 0) {
      apply_config(s, v);
#ifdef SAFETENSORS_PATTERN_MOE_ROUTER_WEIGHT
    } else if (strcmp(k, "num_local_experts") == 0) {
      s->expert_count = (size_t)want_int(v, "num_local_experts");
    } else if (strcmp(k, "num_experts_per_tok") == 0) {
      s->expert_top_k = (size_t)want_int(v, "num_experts_per_tok");
#endif
    }
  }
}

// One safetensors file: 8-byte little-endian header length, then a JSON
// object of tensors (source/json_parser.y:275-338, 590-612).
static void read_safetensors_header(safetensors_t* s, size_t file_index) {
  const char* path = s->file[file_index];
  FILE* f = fopen(path, "rb");
  if (!f) {
    fprintf(stderr, "[StrasGPT] Error: failed to open %s\n", path);
    exit(EXIT_FAILURE);
  }
  uint64_t header_len = 0;
  if (fread(&header_len, 1, 8, f) != 8) {
    fprintf(stderr, "[StrasGPT] Error: %s: short header length\n", path);
    exit(EXIT_FAILURE);
  }
  if (header_len > ((uint64_t)1 << 31)) {
    fprintf(stderr, "[StrasGPT] Error: %s: header too large\n", path);
    exit(EXIT_FAILURE);
  }
  char* text = malloc((size_t)header_len + 1);
  if (!text) {
    fprintf(stderr, "[StrasGPT] Error: out of host memory\n");
    exit(EXIT_FAILURE);
  }
  if (fread(text, 1, (size_t)header_len, f) != (size_t)header_len) {
    fprintf(stderr, "[StrasGPT] Error: %s: truncated header\n", path);
    exit(EXIT_FAILURE);
  }
  fclose(f);
  text[header_len] = '\0';
  json_value_t* root = json_parse(text, (size_t)header_len, path);
  free(text);
  if (root->kind != JSON_OBJECT) {
    parse_die(root, "safetensors header: expected an object");
  }
  for (size_t i = 0; i < root->count; i++) {
    const char* name = root->key[i];
    const json_value_t* t = &root->item[i];
    if (strcmp(name, "__metadata__") == 0 || strcmp(name, "metadata") == 0) {
      continue;
    }
    if (s->tensor_count >= SAFETENSORS_MAX_TENSOR_COUNT) {
      parse_die(t, "too many tensors");
    }
    if (t->kind != JSON_OBJECT) {
      parse_die(t, "tensor entry: expected an object");
    }
    safetensors_tensor_t* st = &s->tensor[s->tensor_count];
    memset(st, 0, sizeof(*st));
    const json_value_t* dtype = json_get(t, "dtype");
    const json_value_t* shape = json_get(t, "shape");
    const json_value_t* offs = json_get(t, "data_offsets");
    if (!dtype || dtype->kind != JSON_STRING) {
      parse_die(t, "tensor entry: missing dtype");
    }
    st->type = safetensors_type_from_string(dtype->string);
    if (shape) {
      if (shape->kind != JSON_ARRAY) {
        parse_die(shape, "shape: expected a list");
      }
      if (shape->count > SAFETENSORS_MAX_DIM_COUNT) {
        parse_die(shape, "too many tensor dimensions");
      }
      for (size_t d = 0; d < shape->count; d++) {
        st->dim[d] = (size_t)want_int(&shape->item[d], "dimension");
      }
      st->dim_count = shape->count;
    }
    if (!offs || offs->kind != JSON_ARRAY || offs->count != 2) {
      parse_die(t, "tensor entry: data_offsets must be [begin, end]");
    }
    long long begin = want_int(&offs->item[0], "offset");
    long long end = want_int(&offs->item[1], "offset");
    if (end < begin || begin < 0) {
      parse_die(offs, "data_offsets: end before begin");
    }
    st->size = (size_t)(end - begin);
    st->offset = 8 + (size_t)header_len + (size_t)begin;
    st->file = file_index;
    st->name = strdup(name);
    s->tensor_count++;
  }
  json_free(root);
}

safetensors_t* parser_parse_safetensors(const char* path) {
  char full[SAFETENSORS_MAX_STRING];
  safetensors_t* s = safetensors_malloc();

  snprintf(full, sizeof(full), "%s/%s", path, SAFETENSORS_FILE_CONFIG);
  json_value_t* config = json_parse_file(full);
  if (!config) {
    fprintf(stderr, "[StrasGPT] Error: failed to open file %s\n", full);
    fprintf(stderr, "Use \"-m <path_to_model_directory>\" option\n");
    exit(EXIT_FAILURE);
  }
  apply_config(s, config);
  json_free(config);

  snprintf(full, sizeof(full), "%s/%s", path, SAFETENSORS_FILE_INDEX);
  json_value_t* index = json_parse_file(full);
  if (!index) {
    snprintf(full, sizeof(full), "%s/%s", path, SAFETENSORS_FILE_SAFETENSORS);
    s->file_count = 1;
    s->file[0] = strdup(full);
  } else {
    const json_value_t* map = json_get(index, "weight_map");
    if (map && map->kind == JSON_OBJECT) {
      for (size_t i = 0; i < map->count; i++) {
        if (map->item[i].kind != JSON_STRING) {
          parse_die(&map->item[i], "weight_map: expected file names");
        }
        safetensors_file_lookup(s, (char*)path, map->item[i].string);
      }
    }
    json_free(index);
  }

  for (size_t i = 0; i < s->file_count; i++) {
    read_safetensors_header(s, i);
  }

  // head_dim defaults to hidden_size / num_attention_heads
  // (source/json_parser.y:614-619).
  if (s->head_dim == 0 && s->q_head_count != 0) {
    s->head_dim = s->embedding_dim / s->q_head_count;
  }
  return s;
}

tokenizer_t* parser_parse_tokenizer(const char* path) {
  char full[SAFETENSORS_MAX_STRING];
  snprintf(full, sizeof(full), "%s/%s", path, TOKENIZER_FILE);
  json_value_t* root = json_parse_file(full);
  if (!root) {
    fprintf(stderr, "[StrasGPT] Error: Failed to open tokenizer file\n");
    exit(EXIT_FAILURE);
  }
  tokenizer_t* t = calloc(1, sizeof(*t));
  if (!t) {
    fprintf(stderr, "[StrasGPT] Error: failed to malloc for tokenizer_t\n");
    exit(EXIT_FAILURE);
  }
  const json_value_t* model = json_get(root, "model");
  const json_value_t* vocab = json_get(model, "vocab");
  if (vocab && vocab->kind == JSON_OBJECT) {
    for (size_t i = 0; i < vocab->count; i++) {
      if (t->token_string_count >= TOKENIZER_MAX_TOKEN_STRING) {
        parse_die(&vocab->item[i], "too many token strings");
      }
      size_t n = t->token_string_count++;
      t->token_string[n] = strdup(vocab->key[i]);
      // The score of a token is its id (source/json_parser.y:434-446).
      t->score[n] = (float)want_number(&vocab->item[i], "token id");
    }
  }
  json_free(root);
  return t;
}

// The reference frees its flex scanner here; this reader holds no state.
int json_scanner_lex_destroy(void) { return 0; }
