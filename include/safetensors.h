// strasgpt-b200: safetensors metadata (model directory reader).
//
// Same API and struct layout as StrasGPT's include/safetensors.h:1-93, so
// that source/strasgpt.c can pass its safetensors_t straight to
// transformer_from_safetensors(). Two additions, both layout-compatible:
//   - SAFETENSORS_TYPE_U8 (appended to the enum) for packed MXFP4 expert
//     weights; the reference aborts on any dtype but F16/BF16/F32
//     (source/safetensors.c:365-378).
//   - expert_count / expert_top_k appended after the tensor table, read from
//     config.json "num_local_experts" / "num_experts_per_tok" (0 = dense).
#ifndef SAFETENSORS_H
#define SAFETENSORS_H

#include <stdbool.h>
#include <stddef.h>
#include <stdio.h>

#ifdef __cplusplus
extern "C" {
#endif

struct options;

#define SAFETENSORS_FILE_CONFIG      "config.json"
#define SAFETENSORS_FILE_INDEX       "model.safetensors.index.json"
#define SAFETENSORS_FILE_SAFETENSORS "model.safetensors"

#define SAFETENSORS_PATTERN_EMBEDDING_WEIGHT  "model.embed_tokens.weight"
#define SAFETENSORS_PATTERN_MHA_NORM_WEIGHT   "model.layers.%d.input_layernorm.weight"
#define SAFETENSORS_PATTERN_MHA_Q_WEIGHT      "model.layers.%d.self_attn.q_proj.weight"
#define SAFETENSORS_PATTERN_MHA_Q_NORM_WEIGHT "model.layers.%d.self_attn.q_norm.weight"
#define SAFETENSORS_PATTERN_MHA_K_WEIGHT      "model.layers.%d.self_attn.k_proj.weight"
#define SAFETENSORS_PATTERN_MHA_K_NORM_WEIGHT "model.layers.%d.self_attn.k_norm.weight"
#define SAFETENSORS_PATTERN_MHA_V_WEIGHT      "model.layers.%d.self_attn.v_proj.weight"
#define SAFETENSORS_PATTERN_MHA_OUT_WEIGHT    "model.layers.%d.self_attn.o_proj.weight"
#define SAFETENSORS_PATTERN_FFN_NORM_WEIGHT   "model.layers.%d.post_attention_layernorm.weight"
#define SAFETENSORS_PATTERN_FFN_FC_WEIGHT     "model.layers.%d.mlp.gate_proj.weight"
#define SAFETENSORS_PATTERN_FFN_UP_WEIGHT     "model.layers.%d.mlp.up_proj.weight"
#define SAFETENSORS_PATTERN_FFN_OUT_WEIGHT    "model.layers.%d.mlp.down_proj.weight"
#define SAFETENSORS_PATTERN_OUT_NORM_WEIGHT   "model.norm.weight"
#define SAFETENSORS_PATTERN_OUT_WEIGHT        "lm_head.weight"

// Mixture-of-experts tensors (no counterpart in the reference). Per layer:
//   router      BF16 [E][D]
//   *_blocks    U8   [E][rows][K/32][16]  two e2m1 codes per byte, the
//                                         even element in the low nibble
//   *_scales    U8   [E][rows][K/32]      e8m0 exponent per 32 values
// gate/up have rows = F (expert hidden), K = D; down has rows = D, K = F.
#define SAFETENSORS_PATTERN_MOE_ROUTER_WEIGHT "model.layers.%d.mlp.router.weight"
#define SAFETENSORS_PATTERN_MOE_GATE_BLOCKS   "model.layers.%d.mlp.experts.gate_proj_blocks"
#define SAFETENSORS_PATTERN_MOE_GATE_SCALES   "model.layers.%d.mlp.experts.gate_proj_scales"
#define SAFETENSORS_PATTERN_MOE_UP_BLOCKS     "model.layers.%d.mlp.experts.up_proj_blocks"
#define SAFETENSORS_PATTERN_MOE_UP_SCALES     "model.layers.%d.mlp.experts.up_proj_scales"
#define SAFETENSORS_PATTERN_MOE_DOWN_BLOCKS   "model.layers.%d.mlp.experts.down_proj_blocks"
#define SAFETENSORS_PATTERN_MOE_DOWN_SCALES   "model.layers.%d.mlp.experts.down_proj_scales"

#define SAFETENSORS_MAX_FILE_COUNT          64
#define SAFETENSORS_MAX_DIM_COUNT           8
#define SAFETENSORS_MAX_MROPE_SECTION_COUNT 8
#define SAFETENSORS_MAX_TENSOR_COUNT        65536
#define SAFETENSORS_MAX_STRING              1024

typedef enum {
  SAFETENSORS_TYPE_F16,  // IEEE float16
  SAFETENSORS_TYPE_BF16, // bfloat16
  SAFETENSORS_TYPE_F32,  // float
  SAFETENSORS_TYPE_U8    // raw bytes (MXFP4 codes and e8m0 scales)
} safetensors_type_t;

extern const char* safetensors_type_str[];

typedef struct safetensors_tensor_t {
  char* name;                            // tensor name
  safetensors_type_t type;               // element type
  size_t dim_count;                      // number of dimensions
  size_t dim[SAFETENSORS_MAX_DIM_COUNT]; // dimensions
  size_t size;                           // size in bytes
  size_t file;                           // index into safetensors_t.file
  size_t offset;                         // byte offset of the data in file
} safetensors_tensor_t;

typedef struct safetensors {
  // Model configuration (config.json)
  char* model_type;
  size_t embedding_dim;   // hidden_size
  size_t head_dim;        // head_dim (default hidden_size / heads)
  size_t hidden_dim;      // intermediate_size
  size_t layer_count;     // num_hidden_layers
  size_t q_head_count;    // num_attention_heads
  size_t kv_head_count;   // num_key_value_heads
  size_t vocabulary_len;  // vocab_size
  size_t context_len;     // max_position_embeddings
  float epsilon;          // rms_norm_eps
  float rope_theta;       // rope_theta
  bool rope_interleaved;  // rope_scaling.mrope_interleaved
  size_t mrope_section_count;
  size_t mrope_section[SAFETENSORS_MAX_MROPE_SECTION_COUNT];

  int bos_token_id;
  int eos_token_id;

  // Files holding the tensors ("<dir>/<name>")
  size_t file_count;
  char* file[SAFETENSORS_MAX_FILE_COUNT];

  // Tensors, in header order
  size_t tensor_count;
  safetensors_tensor_t tensor[SAFETENSORS_MAX_TENSOR_COUNT];

  // Appended (not in the reference layout): mixture-of-experts shape.
  size_t expert_count;    // num_local_experts (0: dense FFN)
  size_t expert_top_k;    // num_experts_per_tok
} safetensors_t;

safetensors_t* safetensors_malloc(void);
void safetensors_free(safetensors_t* safetensors);
void safetensors_print(FILE* f, const safetensors_t* safetensors);
void safetensors_print_model_infos(FILE* f, const safetensors_t* s);
safetensors_t* safetensors_read(struct options* options);
safetensors_type_t safetensors_type_from_string(const char* s);
void safetensors_file_lookup(safetensors_t* s, char* path, char* file);
size_t safetensors_sizeof(safetensors_type_t type);
bool safetensors_aliased_out_weight(const safetensors_t* safetensors);

// Parse <path>/config.json, the optional index and every safetensors header
// (the reference generates this from source/json_parser.y:526-622).
safetensors_t* parser_parse_safetensors(const char* path);

#ifdef __cplusplus
}
#endif

#endif // SAFETENSORS_H
