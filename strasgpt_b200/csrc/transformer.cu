// The transformer C ABI (include/transformer.h, include/strasgpt.h) over the
// sm_100a kernels: weight upload with tensor-parallel slicing, device state,
// the chunked forward pass, the CUDA-graph decode step and greedy loop.
//
// Reference: source/transformer.c (weights_from_safetensors :643-729,
// state_from_safetensors :61-149, transformer_predict_chunk :1186-1602,
// transformer_predict :1607-1727).
//
// HBM layout (per GPU, rank g of N, "l" = local shard):
//   embedding      bf16 [V][D]            replicated (row gather)
//   lm head        bf16 [V/N][D]          vocab rows of this rank (a view
//                                         into the embedding when tied)
//   wqkv[l]        bf16 [(QHl+2KHl)*HD][D]  q rows of this rank's heads,
//                                         then its k rows, then its v rows
//   wo[l]          bf16 [D][QHl*HD]       column slice of o_proj
//   wgu[l]         bf16 [2*Fl][D]         gate/up rows interleaved row by
//                                         row (g0,u0,g1,u1,...)
//   wd[l]          bf16 [D][Fl]           column slice of down_proj
//   experts[l]     u8 codes/scales of the experts this rank owns
//   k/v cache      fp32 [L][KHl][ctx][HD] this rank's kv heads
//   rope table     fp32 [ctx][HD]         computed on the host with the
//                                         reference's expressions
#include "common.cuh"
#include "gemm_tc.h"
#include "kernels.h"
#include "mega.h"
#include "tp.h"

#include <fcntl.h>
#include <omp.h>
#include <string.h>
#include <unistd.h>

#include <cmath>
#include <string>
#include <thread>
#include <vector>

extern "C" {
#include "safetensors.h"
#include "strasgpt.h"
#include "transformer.h"
}

namespace {

struct Layer {
  uint16_t* attn_norm = nullptr;
  uint16_t* wqkv = nullptr;
  uint16_t* q_norm = nullptr;
  uint16_t* k_norm = nullptr;
  uint16_t* wo = nullptr;
  uint16_t* ffn_norm = nullptr;
  uint16_t* wgu = nullptr;
  uint16_t* wd = nullptr;
  uint16_t* router = nullptr;
  uint8_t* gate_c = nullptr;
  uint8_t* gate_s = nullptr;
  uint8_t* up_c = nullptr;
  uint8_t* up_s = nullptr;
  uint8_t* down_c = nullptr;
  uint8_t* down_s = nullptr;
};

// Placement requested through strasgpt_set_placement() (-1: use env).
int g_rank = -1, g_world = -1, g_device = -1;

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

}  // namespace

struct transformer_weights {
  int device = 0, rank = 0, world = 1;
  int D = 0, HD = 0, F = 0, L = 0, QH = 0, KH = 0, V = 0;
  int QHl = 0, KHl = 0, G = 0, Fl = 0, Vl = 0, QKVl = 0;
  bool qk_norm = false, moe = false;
  int E = 0, El = 0, topk = 0, e_begin = 0, e_end = 0;
  float eps = 0.f;
  uint16_t* emb = nullptr;
  uint16_t* out_w = nullptr;
  uint16_t* out_norm = nullptr;
  std::vector<Layer> layer;
  std::vector<void*> allocs;
  size_t device_bytes = 0;
  // Single-process tensor parallelism (STRASGPT_NGPU=N): the transformer the
  // caller holds is a group of N ranks, one per GPU, each a full
  // transformer_t on its device; the C ABI runs every call on all ranks,
  // one host thread per rank, and answers with rank 0's results.
  std::vector<transformer_t*> ranks;
};

struct transformer_state {
  cudaStream_t stream = nullptr;
  int chunk_max = 0;
  int logit_rows_max = 0;
  int ctx = 0;
  float *x = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr;
  float *att = nullptr, *h = nullptr, *logits = nullptr;
  float *kc = nullptr, *vc = nullptr, *rope = nullptr;
  int *tok = nullptr, *pos = nullptr, *step = nullptr, *gen = nullptr;
  float* attn_partial = nullptr;
  int* attn_ticket = nullptr;
  int nsplit = 1, split_len = 1;
  float* am_val = nullptr;
  int *am_idx = nullptr, *am_ticket = nullptr;
  float *rl = nullptr, *ew = nullptr;
  int* eidx = nullptr;
  size_t cached_count = 0;
  float* h_logits = nullptr;  // pinned bounce buffer [logit_rows_max][V]
  // Tensor parallelism (world > 1): this rank's partial sums of o_proj and
  // the FFN ([chunk][D]) before the all-reduce, its vocabulary slice of the
  // logits before the gather, and the peer exchange buffers.
  float* part = nullptr;
  float* logits_local = nullptr;
  sg::TpComm tp;
  cudaGraphExec_t graph_logits = nullptr;
  cudaGraphExec_t graph_greedy = nullptr;
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  std::vector<void*> allocs;
  // profiling (eager launches between events)
  // persistent decode megakernel (dense models, one GPU)
  bool use_mega = false;
  int mega_grid = 0, mega_nsplit = 1, mega_split_len = 1;
  size_t mega_smem = 0;
  sg::MegaLayer* mega_layers = nullptr;  // device [L]
  unsigned long long* mega_ll = nullptr; // flagged hand-off vectors
  sg::MegaFlagged mega_llo{};
  unsigned mega_epoch = 1;               // epoch of the next launch's first step
  int* err = nullptr;
  unsigned long long* trace = nullptr;   // STRASGPT_MEGA_TRACE=<file>
  int trace_phases = 0;
  // Tensor-core prefill projections: bf16 halves of the current projection
  // input ([chunk_max][K]) with their TMA maps for K = D, QH*HD, F; weight
  // maps per layer (qkv, o, gate/up, down), then the LM head.
  bool use_tc = false;
  uint16_t *a_hi = nullptr, *a_lo = nullptr;
  sg::TcAct in[3];
  std::vector<sg::TcMap> tc_w;
  int* tc_err = nullptr;
  // MoE chunks on the tensor cores: one expert at a time, its MXFP4
  // gate/up and down dequantised to bf16 scratch (gate/up interleaved), the
  // expert's tokens gathered, two projections, then a weighted combine of
  // the per-slot outputs moe_y [T*k][D].
  uint16_t *moe_wgu = nullptr, *moe_wd = nullptr;
  float* moe_y = nullptr;
  int *moe_counts = nullptr, *moe_offsets = nullptr, *moe_perm = nullptr, *moe_inv = nullptr;
  int* h_moe_counts = nullptr;  // pinned [E]
  size_t launches = 0;        // kernels enqueued (graph nodes at capture)
  size_t graph_nodes = 0;     // kernels in one greedy-graph replay
  strasgpt_kernel_profile_t* prof = nullptr;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<int> prof_fam;
  std::vector<double> prof_bytes;
};

namespace {

typedef transformer_weights W_t;
typedef transformer_state S_t;

void* dalloc(std::vector<void*>& list, size_t bytes, size_t* counter) {
  void* p = nullptr;
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "cudaMalloc of %zu bytes failed: %s", bytes,
             cudaGetErrorString(e));
    SG_DIE(msg);
  }
  list.push_back(p);
  if (counter) *counter += bytes;
  return p;
}

// ---------------------------------------------------------------------------
// Loading
// ---------------------------------------------------------------------------
enum Kind {
  K_UNKNOWN, K_EMB, K_OUT_NORM, K_OUT, K_ATTN_NORM, K_Q, K_K, K_V, K_O,
  K_QN, K_KN, K_FFN_NORM, K_GATE, K_UP, K_DOWN, K_ROUTER, K_GATE_C, K_GATE_S,
  K_UP_C, K_UP_S, K_DOWN_C, K_DOWN_S
};

// Tensor name -> (kind, layer). Accepts the reference's base names and its
// "model.language_model." aliases (source/transformer.c:520-574).
Kind classify(const char* name, int* layer) {
  static const struct { const char* n; Kind k; } globals[] = {
      {"model.embed_tokens.weight", K_EMB},
      {"model.language_model.embed_tokens.weight", K_EMB},
      {"model.norm.weight", K_OUT_NORM},
      {"model.language_model.norm.weight", K_OUT_NORM},
      {"lm_head.weight", K_OUT}};
  for (auto& g : globals)
    if (strcmp(name, g.n) == 0) return g.k;
  const char* prefixes[] = {"model.layers.", "model.language_model.layers."};
  for (const char* p : prefixes) {
    size_t n = strlen(p);
    if (strncmp(name, p, n) != 0) continue;
    const char* s = name + n;
    if (*s < '0' || *s > '9') return K_UNKNOWN;
    long idx = 0;
    while (*s >= '0' && *s <= '9') idx = idx * 10 + (*s++ - '0');
    if (*s != '.') return K_UNKNOWN;
    s++;
    *layer = (int)idx;
    static const struct { const char* n; Kind k; } suffixes[] = {
        {"input_layernorm.weight", K_ATTN_NORM},
        {"self_attn.q_proj.weight", K_Q},
        {"self_attn.k_proj.weight", K_K},
        {"self_attn.v_proj.weight", K_V},
        {"self_attn.o_proj.weight", K_O},
        {"self_attn.q_norm.weight", K_QN},
        {"self_attn.k_norm.weight", K_KN},
        {"post_attention_layernorm.weight", K_FFN_NORM},
        {"mlp.gate_proj.weight", K_GATE},
        {"mlp.up_proj.weight", K_UP},
        {"mlp.down_proj.weight", K_DOWN},
        {"mlp.router.weight", K_ROUTER},
        {"mlp.experts.gate_proj_blocks", K_GATE_C},
        {"mlp.experts.gate_proj_scales", K_GATE_S},
        {"mlp.experts.up_proj_blocks", K_UP_C},
        {"mlp.experts.up_proj_scales", K_UP_S},
        {"mlp.experts.down_proj_blocks", K_DOWN_C},
        {"mlp.experts.down_proj_scales", K_DOWN_S}};
    for (auto& x : suffixes)
      if (strcmp(s, x.n) == 0) return x.k;
    return K_UNKNOWN;
  }
  return K_UNKNOWN;
}

struct Reader {
  std::vector<int> fd;
  explicit Reader(const safetensors_t* s) {
    for (size_t i = 0; i < s->file_count; i++) {
      int f = open(s->file[i], O_RDONLY);
      if (f < 0) {
        fprintf(stderr, "[StrasGPT] Error: failed to open file %s\n", s->file[i]);
        exit(EXIT_FAILURE);
      }
      fd.push_back(f);
    }
  }
  ~Reader() {
    for (int f : fd) close(f);
  }
  void read(const safetensors_tensor_t* t, void* dst) {
    size_t done = 0;
    char* p = (char*)dst;
    while (done < t->size) {
      ssize_t n = pread(fd[t->file], p + done, t->size - done,
                        (off_t)(t->offset + done));
      if (n <= 0) SG_DIE("failed to read from file");
      done += (size_t)n;
    }
  }
};

void check_size(const safetensors_tensor_t* t, size_t expect, const char* what) {
  if (t->size != expect) {
    char msg[512];
    snprintf(msg, sizeof(msg), "unexpected size for %s (%s): have %zu expected %zu",
             what, t->name, t->size, expect);
    SG_DIE(msg);
  }
}

void check_type(const safetensors_tensor_t* t, safetensors_type_t want) {
  if (t->type != want) {
    char msg[512];
    snprintf(msg, sizeof(msg), "tensor %s has dtype %s, expected %s", t->name,
             safetensors_type_str[t->type], safetensors_type_str[want]);
    SG_DIE(msg);
  }
}

void h2d_2d(void* dst, size_t dpitch, const void* src, size_t spitch,
            size_t width, size_t height) {
  SG_CUDA(cudaMemcpy2D(dst, dpitch, src, spitch, width, height,
                       cudaMemcpyHostToDevice));
}

void load_weights(W_t* w, const safetensors_t* s) {
  const size_t D = w->D, HD = w->HD, F = w->F, V = w->V;
  const size_t QH = w->QH, KH = w->KH, QHl = w->QHl, KHl = w->KHl;
  const size_t Fl = w->Fl, Vl = w->Vl, E = w->E, El = w->El;
  const int g = w->rank;
  size_t* cnt = &w->device_bytes;
  auto A16 = [&](size_t n) { return (uint16_t*)dalloc(w->allocs, n * 2, cnt); };
  auto A8 = [&](size_t n) { return (uint8_t*)dalloc(w->allocs, n, cnt); };

  w->emb = A16(V * D);
  w->out_norm = A16(D);
  const bool tied = safetensors_aliased_out_weight(s);
  w->out_w = tied ? w->emb + (size_t)g * Vl * D : A16(Vl * D);
  w->layer.resize(w->L);
  for (auto& ly : w->layer) {
    ly.attn_norm = A16(D);
    ly.ffn_norm = A16(D);
    ly.wqkv = A16((QHl + 2 * KHl) * HD * D);
    ly.wo = A16(D * QHl * HD);
    if (w->qk_norm) {
      ly.q_norm = A16(HD);
      ly.k_norm = A16(HD);
    }
    if (w->moe) {
      ly.router = A16(E * D);
      ly.gate_c = A8(El * F * (D / 32) * 16);
      ly.gate_s = A8(El * F * (D / 32));
      ly.up_c = A8(El * F * (D / 32) * 16);
      ly.up_s = A8(El * F * (D / 32));
      ly.down_c = A8(El * D * (F / 32) * 16);
      ly.down_s = A8(El * D * (F / 32));
    } else {
      ly.wgu = A16(2 * Fl * D);
      ly.wd = A16(D * Fl);
    }
  }

  Reader rd(s);
  std::vector<char> host;
  std::vector<unsigned char> seen((size_t)w->L * 32 + 8, 0);
  const size_t row = D * 2;  // bytes of one D-long bf16 row
  for (size_t i = 0; i < s->tensor_count; i++) {
    const safetensors_tensor_t* t = &s->tensor[i];
    int l = -1;
    Kind k = classify(t->name, &l);
    if (k == K_UNKNOWN) {
      fprintf(stderr, "[StrasGPT] Warning: unknown tensor %s\n", t->name);
      continue;
    }
    if (l >= w->L) {
      fprintf(stderr, "[StrasGPT] Warning: tensor %s beyond layer_count\n", t->name);
      continue;
    }
    const bool is_moe_t = (k >= K_ROUTER);
    if (is_moe_t && !w->moe) {
      fprintf(stderr, "[StrasGPT] Warning: expert tensor %s in a dense model\n", t->name);
      continue;
    }
    if (w->moe && (k == K_GATE || k == K_UP || k == K_DOWN)) {
      fprintf(stderr, "[StrasGPT] Warning: dense FFN tensor %s in an MoE model\n", t->name);
      continue;
    }
    if ((k == K_QN || k == K_KN) && !w->qk_norm) continue;
    check_type(t, (k >= K_GATE_C) ? SAFETENSORS_TYPE_U8 : SAFETENSORS_TYPE_BF16);
    host.resize(t->size);
    rd.read(t, host.data());
    const char* h = host.data();
    Layer* ly = (l >= 0) ? &w->layer[l] : nullptr;
    switch (k) {
      case K_EMB:
        check_size(t, V * D * 2, "embedding weight");
        h2d_2d(w->emb, row, h, row, row, V);
        break;
      case K_OUT_NORM:
        check_size(t, D * 2, "out norm weight");
        h2d_2d(w->out_norm, row, h, row, row, 1);
        break;
      case K_OUT:
        check_size(t, V * D * 2, "out weight");
        h2d_2d(w->out_w, row, h + (size_t)g * Vl * row, row, row, Vl);
        break;
      case K_ATTN_NORM:
        check_size(t, D * 2, "mha norm weight");
        h2d_2d(ly->attn_norm, row, h, row, row, 1);
        break;
      case K_FFN_NORM:
        check_size(t, D * 2, "ffn norm weight");
        h2d_2d(ly->ffn_norm, row, h, row, row, 1);
        break;
      case K_Q:
        check_size(t, QH * HD * D * 2, "mha q weight");
        h2d_2d(ly->wqkv, row, h + (size_t)g * QHl * HD * row, row, row, QHl * HD);
        break;
      case K_K:
        check_size(t, KH * HD * D * 2, "mha k weight");
        h2d_2d(ly->wqkv + QHl * HD * D, row, h + (size_t)g * KHl * HD * row,
               row, row, KHl * HD);
        break;
      case K_V:
        check_size(t, KH * HD * D * 2, "mha v weight");
        h2d_2d(ly->wqkv + (QHl + KHl) * HD * D, row,
               h + (size_t)g * KHl * HD * row, row, row, KHl * HD);
        break;
      case K_O:
        check_size(t, D * QH * HD * 2, "mha out weight");
        h2d_2d(ly->wo, QHl * HD * 2, h + (size_t)g * QHl * HD * 2, QH * HD * 2,
               QHl * HD * 2, D);
        break;
      case K_QN:
        check_size(t, HD * 2, "mha q norm weight");
        h2d_2d(ly->q_norm, HD * 2, h, HD * 2, HD * 2, 1);
        break;
      case K_KN:
        check_size(t, HD * 2, "mha k norm weight");
        h2d_2d(ly->k_norm, HD * 2, h, HD * 2, HD * 2, 1);
        break;
      case K_GATE:
      case K_UP: {
        check_size(t, F * D * 2, k == K_GATE ? "ffn fc weight" : "ffn up weight");
        const size_t grp = SG_GU_GROUP * row;
        uint16_t* dst = ly->wgu + (k == K_UP ? SG_GU_GROUP * D : 0);
        h2d_2d(dst, 2 * grp, h + (size_t)g * Fl * row, grp, grp, Fl / SG_GU_GROUP);
        break;
      }
      case K_DOWN:
        check_size(t, D * F * 2, "ffn out weight");
        h2d_2d(ly->wd, Fl * 2, h + (size_t)g * Fl * 2, F * 2, Fl * 2, D);
        break;
      case K_ROUTER:
        check_size(t, E * D * 2, "router weight");
        h2d_2d(ly->router, row, h, row, row, E);
        break;
      case K_GATE_C:
      case K_UP_C: {
        const size_t per = F * (D / 32) * 16;
        check_size(t, E * per, "expert gate/up blocks");
        h2d_2d(k == K_GATE_C ? ly->gate_c : ly->up_c, El * per,
               h + (size_t)w->e_begin * per, El * per, El * per, 1);
        break;
      }
      case K_GATE_S:
      case K_UP_S: {
        const size_t per = F * (D / 32);
        check_size(t, E * per, "expert gate/up scales");
        h2d_2d(k == K_GATE_S ? ly->gate_s : ly->up_s, El * per,
               h + (size_t)w->e_begin * per, El * per, El * per, 1);
        break;
      }
      case K_DOWN_C: {
        const size_t per = D * (F / 32) * 16;
        check_size(t, E * per, "expert down blocks");
        h2d_2d(ly->down_c, El * per, h + (size_t)w->e_begin * per, El * per,
               El * per, 1);
        break;
      }
      case K_DOWN_S: {
        const size_t per = D * (F / 32);
        check_size(t, E * per, "expert down scales");
        h2d_2d(ly->down_s, El * per, h + (size_t)w->e_begin * per, El * per,
               El * per, 1);
        break;
      }
      default:
        break;
    }
    const int slot = (l >= 0) ? l * 32 + (int)k : (int)w->L * 32 + (int)k % 8;
    seen[(size_t)slot] = 1;
  }
  // Every tensor the forward pass reads must have been present.
  auto need = [&](int slot, const char* what, int l) {
    if (!seen[(size_t)slot]) {
      char msg[256];
      if (l >= 0)
        snprintf(msg, sizeof(msg), "missing tensor: layer %d %s", l, what);
      else
        snprintf(msg, sizeof(msg), "missing tensor: %s", what);
      SG_DIE(msg);
    }
  };
  need(w->L * 32 + K_EMB % 8, "embedding", -1);
  need(w->L * 32 + K_OUT_NORM % 8, "model.norm.weight", -1);
  if (!tied) need(w->L * 32 + K_OUT % 8, "lm_head.weight", -1);
  for (int l = 0; l < w->L; l++) {
    int b = l * 32;
    need(b + K_ATTN_NORM, "input_layernorm", l);
    need(b + K_Q, "q_proj", l);
    need(b + K_K, "k_proj", l);
    need(b + K_V, "v_proj", l);
    need(b + K_O, "o_proj", l);
    need(b + K_FFN_NORM, "post_attention_layernorm", l);
    if (w->qk_norm) {
      need(b + K_QN, "q_norm", l);
      need(b + K_KN, "k_norm", l);
    }
    if (w->moe) {
      need(b + K_ROUTER, "router", l);
      need(b + K_GATE_C, "gate_proj_blocks", l);
      need(b + K_GATE_S, "gate_proj_scales", l);
      need(b + K_UP_C, "up_proj_blocks", l);
      need(b + K_UP_S, "up_proj_scales", l);
      need(b + K_DOWN_C, "down_proj_blocks", l);
      need(b + K_DOWN_S, "down_proj_scales", l);
    } else {
      need(b + K_GATE, "gate_proj", l);
      need(b + K_UP, "up_proj", l);
      need(b + K_DOWN, "down_proj", l);
    }
  }
}

bool has_qk_norm(const safetensors_t* s) {
  for (size_t i = 0; i < s->tensor_count; i++) {
    int l;
    if (classify(s->tensor[i].name, &l) == K_QN) return true;
  }
  return false;
}

// RoPE table with the reference's expressions (source/transformer.c:126-146).
std::vector<float> rope_table(const transformer_configuration_t* c) {
  const size_t ctx = c->context_len, hd = c->head_dim;
  std::vector<float> t(ctx * hd, 0.f);
  const bool interleaved = c->rope_pair_stride == 2;
  const float coef = interleaved ? 1.0f : 2.0f;
  for (size_t i = 0; i < ctx; i++) {
    for (size_t j = 0; j < c->rope_pair_bound; j += c->rope_pair_stride) {
      float freq = 1.0f / powf(c->rope_theta, (coef * j) / hd);
      float val = i * freq;
      t[i * hd + j] = cosf(val);
      t[i * hd + j + c->rope_pair_offset] = sinf(val);
    }
  }
  return t;
}

void alloc_state(const W_t* w, const transformer_configuration_t* c, S_t* s) {
  const int dev = w->device;
  (void)dev;
  s->ctx = (int)c->context_len;
  s->chunk_max = env_int("STRASGPT_CHUNK", 2048);
  if (s->chunk_max > s->ctx) s->chunk_max = s->ctx;
  if (s->chunk_max < 1) s->chunk_max = 1;
  s->logit_rows_max = 64;
  const size_t T = s->chunk_max, D = w->D, HD = w->HD;
  const size_t qkv = (size_t)w->QKVl;
  const size_t hid = w->moe ? (size_t)w->topk * w->F : (size_t)w->Fl;
  auto F32 = [&](size_t n) { return (float*)dalloc(s->allocs, n * 4, nullptr); };
  auto I32 = [&](size_t n) { return (int*)dalloc(s->allocs, n * 4, nullptr); };
  s->x = F32(T * D);
  s->xn = F32(T * D);
  s->qkv = F32(T * qkv);
  s->q = F32(T * w->QHl * HD);
  s->att = F32(T * w->QHl * HD);
  s->h = F32(T * hid);
  s->logits = F32((size_t)s->logit_rows_max * w->V);
  if (w->world > 1) {
    s->part = F32(T * D);
    s->logits_local = F32((size_t)s->logit_rows_max * w->Vl);
  }
  const size_t kv = (size_t)w->L * w->KHl * s->ctx * HD;
  s->kc = F32(kv);
  s->vc = F32(kv);
  SG_CUDA(cudaMemset(s->kc, 0, kv * 4));
  SG_CUDA(cudaMemset(s->vc, 0, kv * 4));
  s->rope = F32((size_t)s->ctx * HD);
  std::vector<float> rt = rope_table(c);
  SG_CUDA(cudaMemcpy(s->rope, rt.data(), rt.size() * 4, cudaMemcpyHostToDevice));
  s->tok = I32(T);
  s->pos = I32(1);
  s->step = I32(1);
  s->gen = I32((size_t)s->ctx + 1);
  // Device-side token loop state starts at zero (cudaMalloc memory is not).
  SG_CUDA(cudaMemset(s->tok, 0, T * 4));
  SG_CUDA(cudaMemset(s->pos, 0, 4));
  SG_CUDA(cudaMemset(s->step, 0, 4));
  SG_CUDA(cudaMemset(s->gen, 0, ((size_t)s->ctx + 1) * 4));
  sg::attn_decode_split(s->ctx, w->KHl, &s->nsplit, &s->split_len);
  // Megakernel decode (dense and mixture-of-experts models), when a CTA fits
  // on every SM (under tensor parallelism too: the LM-head slices are then
  // gathered after the kernel when predict needs full logits).
  const bool moe_ok = !w->moe || (w->E % 2 == 0 && w->E <= 128 && w->topk >= 1 &&
                                  w->topk <= 8 && w->F % 32 == 0 && w->D % 32 == 0);
  const int mega_Fl = w->moe ? 0 : w->Fl;
  s->use_mega = moe_ok && (w->Vl % 2 == 0) && w->L <= 96 && w->world <= 8 && w->D <= 8192 &&
                env_int("STRASGPT_MEGA", 1) != 0;
  if (s->use_mega) {
    s->mega_smem = sg::mega_smem_bytes(w->D, w->QHl * w->HD, mega_Fl, w->HD, w->G, w->L,
                                       w->moe ? w->topk : 0, w->moe ? w->F : 0);
    if (s->mega_smem == 0) s->use_mega = false;
  }
  if (s->use_mega) {
    sg::mega_configure(s->mega_smem);
    s->mega_grid = sg::mega_grid(s->mega_smem, w->HD, w->G);
    if (s->mega_grid <= 0) s->use_mega = false;
  }
  if (s->use_mega) {
    sg::mega_split(s->ctx, w->KHl, s->mega_grid, &s->mega_nsplit, &s->mega_split_len);
    std::vector<sg::MegaLayer> ml(w->L);
    const int sgD = sg::mega_scale_row_bytes(w->D), sgF = sg::mega_scale_row_bytes(w->F);
    for (int l = 0; l < w->L; l++) {
      const Layer& y = w->layer[l];
      ml[l] = {y.attn_norm, y.wqkv, y.q_norm, y.k_norm, y.wo, y.ffn_norm, y.wgu, y.wd,
               nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
      if (w->moe) {
        // The expert scales again, each row on a 16-byte boundary (one bulk
        // copy per row), next to the unchanged codes.
        const size_t gu_rows = (size_t)w->El * w->F, d_rows = (size_t)w->El * w->D;
        uint8_t* gs = (uint8_t*)dalloc(s->allocs, gu_rows * sgD, nullptr);
        uint8_t* us = (uint8_t*)dalloc(s->allocs, gu_rows * sgD, nullptr);
        uint8_t* ds = (uint8_t*)dalloc(s->allocs, d_rows * sgF, nullptr);
        sg::mega_pad_rows(y.gate_s, gu_rows, w->D / 32, sgD, gs, 0);
        sg::mega_pad_rows(y.up_s, gu_rows, w->D / 32, sgD, us, 0);
        sg::mega_pad_rows(y.down_s, d_rows, w->F / 32, sgF, ds, 0);
        ml[l].router = y.router;
        ml[l].gate_c = y.gate_c;
        ml[l].up_c = y.up_c;
        ml[l].down_c = y.down_c;
        ml[l].gate_s = gs;
        ml[l].up_s = us;
        ml[l].down_s = ds;
      }
    }
    SG_CUDA(cudaDeviceSynchronize());
    s->mega_layers = (sg::MegaLayer*)dalloc(s->allocs, sizeof(sg::MegaLayer) * w->L, nullptr);
    SG_CUDA(cudaMemcpy(s->mega_layers, ml.data(), sizeof(sg::MegaLayer) * w->L,
                       cudaMemcpyHostToDevice));
    s->err = I32(1);
    if (getenv("STRASGPT_MEGA_TRACE")) {
      // Phase timestamps of the first two decode steps of a launch.
      s->trace_phases = 2 * ((w->moe ? 6 : 5) * w->L + 1);
      const size_t n = (size_t)s->trace_phases * s->mega_grid * sg::kMegaTraceWidth;
      s->trace = (unsigned long long*)dalloc(s->allocs, n * 8, nullptr);
      SG_CUDA(cudaMemset(s->trace, 0, n * 8));
    }
    SG_CUDA(cudaMemset(s->err, 0, 4));
    // Flagged hand-off vectors, zero (epoch 0: never written) at rest. Under
    // tensor parallelism they live in the exchange buffer the ranks map.
    s->mega_llo = sg::mega_flagged_layout(w->D, w->QKVl, w->QHl * w->HD, mega_Fl, w->L,
                                          s->mega_grid, w->world, s->mega_nsplit, w->HD,
                                          w->moe ? w->E : 0, w->moe ? w->topk : 0,
                                          w->moe ? w->F : 0);
    if (w->world == 1) {
      s->mega_ll = (unsigned long long*)dalloc(s->allocs, s->mega_llo.total * 8, nullptr);
      SG_CUDA(cudaMemset(s->mega_ll, 0, s->mega_llo.total * 8));
    }
    s->mega_epoch = 1;
  }
  if (w->world > 1) {
    sg::tp_alloc(&s->tp, w->rank, w->world, std::max(T * D, (size_t)s->logit_rows_max * w->Vl),
                 s->use_mega ? s->mega_llo.total * 8 : 0);
    if (s->use_mega) s->mega_ll = (unsigned long long*)(s->tp.local + s->tp.extra_off);
  }
  // Split records and tickets of the per-op decode kernel (the persistent
  // kernel keeps its records among its flagged vectors).
  s->attn_partial = F32((size_t)w->QHl * s->nsplit * (HD + 4));
  s->attn_ticket = I32(w->KHl);
  SG_CUDA(cudaMemset(s->attn_ticket, 0, (size_t)w->KHl * 4));
  s->am_val = F32(1024);
  s->am_idx = I32(1024);
  s->am_ticket = I32(1);
  SG_CUDA(cudaMemset(s->am_ticket, 0, 4));
  if (w->moe) {
    s->rl = F32(T * w->E);
    s->ew = F32(T * w->topk);
    s->eidx = I32(T * w->topk);
  }
  const int QD = w->QHl * w->HD;
  s->use_tc = env_int("STRASGPT_TC", 1) != 0 && w->D % 8 == 0 && QD % 8 == 0 &&
              (w->moe || w->Fl % 8 == 0);
  if (s->use_tc) {
    sg::tc_configure();
    // K of the three projection inputs: D, QH*HD, and F (this rank's FFN
    // rows; a whole expert's F for MoE).
    const int ks[3] = {w->D, QD, w->Fl};
    const size_t kmax = (size_t)std::max(ks[0], std::max(ks[1], ks[2]));
    s->a_hi = (uint16_t*)dalloc(s->allocs, T * kmax * 2, nullptr);
    s->a_lo = (uint16_t*)dalloc(s->allocs, T * kmax * 2, nullptr);
    for (int i = 0; i < 3; i++) sg::tc_make_act(&s->in[i], s->a_hi, s->a_lo, (int)T, ks[i]);
    s->tc_w.resize((size_t)4 * w->L + 3);
    if (w->moe) {
      const size_t F = w->F;
      s->moe_wgu = (uint16_t*)dalloc(s->allocs, 2 * F * D * 2, nullptr);
      s->moe_wd = (uint16_t*)dalloc(s->allocs, D * F * 2, nullptr);
      s->moe_y = F32(T * w->topk * D);
      s->moe_counts = I32(w->E);
      s->moe_offsets = I32(w->E);
      s->moe_perm = I32(T * w->topk);
      s->moe_inv = I32(T * w->topk);
      SG_CUDA(cudaMallocHost(&s->h_moe_counts, (size_t)w->E * sizeof(int)));
      sg::tc_make_map(&s->tc_w[4 * w->L + 1], s->moe_wgu, 2 * w->F, w->D);
      sg::tc_make_map(&s->tc_w[4 * w->L + 2], s->moe_wd, w->D, w->F);
    }
    for (int l = 0; l < w->L; l++) {
      const Layer& y = w->layer[l];
      sg::tc_make_map(&s->tc_w[4 * l + 0], y.wqkv, w->QKVl, w->D);
      sg::tc_make_map(&s->tc_w[4 * l + 1], y.wo, w->D, QD);
      if (!w->moe) {
        sg::tc_make_map(&s->tc_w[4 * l + 2], y.wgu, 2 * w->Fl, w->D);
        sg::tc_make_map(&s->tc_w[4 * l + 3], y.wd, w->D, w->Fl);
      }
    }
    sg::tc_make_map(&s->tc_w[4 * w->L], w->out_w, w->Vl, w->D);
    s->tc_err = I32(1);
    SG_CUDA(cudaMemset(s->tc_err, 0, 4));
  }
  SG_CUDA(cudaMallocHost(&s->h_logits, (size_t)s->logit_rows_max * w->V * 4));
  SG_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  for (auto& e : s->ev) SG_CUDA(cudaEventCreate(&e));
}

// ---------------------------------------------------------------------------
// Forward pass
// ---------------------------------------------------------------------------
enum Family { FAM_MATVEC = 0, FAM_ATTN, FAM_QKV, FAM_LMHEAD, FAM_ARGMAX, FAM_OTHER };

struct Runner {
  const W_t* w;
  S_t* s;
  const transformer_configuration_t* c;
  cudaStream_t st;

  template <typename Fn>
  void launch(int fam, double bytes, Fn&& fn) {
    s->launches++;
    if (!s->prof) {
      fn();
      return;
    }
    const size_t n = s->prof_fam.size();
    while (s->prof_ev.size() < 2 * n + 2) {
      cudaEvent_t e;
      SG_CUDA(cudaEventCreate(&e));
      s->prof_ev.push_back(e);
    }
    SG_CUDA(cudaEventRecord(s->prof_ev[2 * n], st));
    fn();
    SG_CUDA(cudaEventRecord(s->prof_ev[2 * n + 1], st));
    s->prof_fam.push_back(fam);
    s->prof_bytes.push_back(bytes);
  }

  float* kc(int l) const { return s->kc + (size_t)l * w->KHl * s->ctx * w->HD; }
  float* vc(int l) const { return s->vc + (size_t)l * w->KHl * s->ctx * w->HD; }

  sg::QkvPostArgs qkv_args(int l, int T) const {
    sg::QkvPostArgs a;
    a.qkv = s->qkv; a.T = T; a.QHl = w->QHl; a.KHl = w->KHl; a.HD = w->HD;
    a.q_norm = w->layer[l].q_norm; a.k_norm = w->layer[l].k_norm; a.eps = w->eps;
    a.rope = s->rope;
    a.pair_bound = (int)c->rope_pair_bound;
    a.pair_offset = (int)c->rope_pair_offset;
    a.pair_stride = (int)c->rope_pair_stride;
    a.pos = s->pos; a.q = s->q; a.k_cache = kc(l); a.v_cache = vc(l); a.ctx = s->ctx;
    return a;
  }

  sg::MoeArgs moe_args(int l, int T) const {
    const Layer& ly = w->layer[l];
    sg::MoeArgs a;
    a.xn = s->xn; a.T = T; a.D = w->D; a.F = w->F; a.k = w->topk;
    a.idx = s->eidx; a.weight = s->ew;
    a.gate_codes = ly.gate_c; a.gate_scales = ly.gate_s;
    a.up_codes = ly.up_c; a.up_scales = ly.up_s;
    a.down_codes = ly.down_c; a.down_scales = ly.down_s;
    a.e_begin = w->e_begin; a.e_end = w->e_end;
    a.h = s->h; a.out = rp_out();
    return a;
  }

  bool tp() const { return w->world > 1; }
  // Target and epilogue of a row-parallel projection (o_proj, down): the
  // residual directly on one GPU, this rank's partial sum under TP.
  float* rp_out() const { return tp() ? s->part : s->x; }
  sg::Epilogue rp_epi() const { return tp() ? sg::EPI_STORE : sg::EPI_ADD; }
  // Under TP: x += sum over ranks of `part` ([T][D]).
  void rp_reduce(int T) {
    if (!tp()) return;
    s->launches++;  // stage + reduce
    launch(FAM_OTHER, 0, [&] {
      sg::tp_allreduce_add(s->tp, s->part, s->x, (size_t)T * w->D, st);
    });
  }
  // LM head target ([rows][Vl] of this rank) and, under TP, the gather of the
  // vocabulary slices into s->logits ([rows][V]).
  float* lm_out() const { return tp() ? s->logits_local : s->logits; }
  void lm_gather(int rows) {
    if (!tp()) return;
    s->launches++;
    launch(FAM_OTHER, 0, [&] {
      sg::tp_gather_rows(s->tp, s->logits_local, rows, w->Vl, s->logits, st);
    });
  }
  void moe_zero_part(int T) {
    if (tp()) SG_CUDA(cudaMemsetAsync(s->part, 0, (size_t)T * w->D * 4, st));
  }

  double moe_bytes_per_token() const {
    const double blocks = (double)w->F * (w->D / 32) * 17.0;
    return w->topk * 3.0 * blocks;
  }

  // One token at the device position *s->pos (graph-capturable).
  void decode_layers() {
    const int D = w->D, HD = w->HD;
    launch(FAM_OTHER, D * 2.0 + D * 4.0, [&] { sg::embed(s->tok, 1, w->emb, D, s->x, st); });
    for (int l = 0; l < w->L; l++) {
      const Layer& ly = w->layer[l];
      launch(FAM_MATVEC, (double)w->QKVl * D * 2, [&] {
        sg::matvec(s->x, ly.attn_norm, w->eps, ly.wqkv, D, w->QKVl, s->qkv,
                   sg::EPI_STORE, st);
      });
      launch(FAM_QKV, 0, [&] { sg::qkv_post(qkv_args(l, 1), st); });
      sg::AttnDecodeArgs a;
      a.q = s->q; a.k_cache = kc(l); a.v_cache = vc(l);
      a.KHl = w->KHl; a.G = w->G; a.HD = HD; a.ctx = s->ctx; a.pos = s->pos;
      a.nsplit = s->nsplit; a.split_len = s->split_len;
      a.partial = s->attn_partial; a.ticket = s->attn_ticket; a.att = s->att;
      launch(FAM_ATTN, 0, [&] { sg::attn_decode(a, st); });
      launch(FAM_MATVEC, (double)D * w->QHl * HD * 2, [&] {
        sg::matvec(s->att, nullptr, 0.f, ly.wo, w->QHl * HD, D, rp_out(), rp_epi(), st);
      });
      rp_reduce(1);
      if (w->moe) {
        launch(FAM_OTHER, 0, [&] { sg::rmsnorm_rows(s->x, 1, D, ly.ffn_norm, w->eps, s->xn, st); });
        launch(FAM_MATVEC, (double)w->E * D * 2, [&] {
          sg::matvec(s->xn, nullptr, 0.f, ly.router, D, w->E, s->rl, sg::EPI_STORE, st);
        });
        launch(FAM_OTHER, 0, [&] { sg::moe_topk(s->rl, 1, w->E, w->topk, s->eidx, s->ew, st); });
        sg::MoeArgs m = moe_args(l, 1);
        moe_zero_part(1);
        launch(FAM_MATVEC, moe_bytes_per_token() * 2 / 3, [&] { sg::moe_gate_up(m, st); });
        launch(FAM_MATVEC, moe_bytes_per_token() / 3, [&] { sg::moe_down(m, st); });
      } else {
        launch(FAM_MATVEC, 2.0 * w->Fl * D * 2, [&] {
          sg::matvec(s->x, ly.ffn_norm, w->eps, ly.wgu, D, w->Fl, s->h,
                     sg::EPI_SWIGLU, st);
        });
        launch(FAM_MATVEC, (double)D * w->Fl * 2, [&] {
          sg::matvec(s->h, nullptr, 0.f, ly.wd, w->Fl, D, rp_out(), rp_epi(), st);
        });
      }
      rp_reduce(1);
    }
    launch(FAM_LMHEAD, (double)w->Vl * D * 2, [&] {
      sg::matvec(s->x, w->out_norm, w->eps, w->out_w, D, w->Vl, lm_out(),
                 sg::EPI_STORE, st);
    });
    lm_gather(1);
  }

  void argmax(int advance_pos) {
    launch(FAM_ARGMAX, (double)w->V * 4, [&] {
      sg::argmax_advance(s->logits, w->V, s->tok, advance_pos ? s->pos : nullptr,
                         s->step, s->gen, s->ctx + 1, s->am_val, s->am_idx,
                         s->am_ticket, st);
    });
  }

  // `steps` decode steps in one persistent launch, starting from the token
  // in s->tok at position *s->pos (see decode_mega.cu).
  void mega(int steps, bool write_logits) {
    sg::MegaArgs a;
    a.D = w->D; a.HD = w->HD; a.QHl = w->QHl; a.KHl = w->KHl; a.G = w->G;
    a.Fl = w->moe ? 0 : w->Fl; a.Vl = w->Vl; a.L = w->L; a.QKVl = w->QKVl; a.ctx = s->ctx;
    a.moe = w->moe ? 1 : 0;
    a.E = w->moe ? w->E : 0; a.topk = w->moe ? w->topk : 0; a.Fe = w->moe ? w->F : 0;
    a.e_begin = w->e_begin; a.e_end = w->e_end;
    a.eps = w->eps; a.layers = s->mega_layers;
    a.emb = w->emb; a.out_norm = w->out_norm; a.out_w = w->out_w;
    a.rope = s->rope;
    a.pair_bound = (int)c->rope_pair_bound;
    a.pair_offset = (int)c->rope_pair_offset;
    a.pair_stride = (int)c->rope_pair_stride;
    a.logits = lm_out();
    a.kc = s->kc; a.vc = s->vc;
    a.nsplit = s->mega_nsplit; a.split_len = s->mega_split_len;
    a.ll = s->mega_ll; a.llo = s->mega_llo; a.epoch = s->mega_epoch;
    a.rank = w->rank; a.world = w->world;
    for (int p = 0; p < 8; p++) a.ll_peer[p] = nullptr;
    if (w->world == 1) {
      a.ll_peer[0] = s->mega_ll;
    } else {
      for (int p = 0; p < w->world; p++)
        a.ll_peer[p] = (unsigned long long*)(s->tp.peer[p] + s->tp.extra_off);
    }
    a.tok = s->tok; a.pos = s->pos; a.step = s->step; a.gen = s->gen;
    a.gen_len = s->ctx + 1;
    a.err = s->err;
    a.wait_ns = sg::wait_limit_ns(2000);
    a.steps = steps; a.write_logits = write_logits ? 1 : 0;
    a.trace = s->trace; a.trace_phases = s->trace_phases;
    if (s->trace)
      SG_CUDA(cudaMemsetAsync(s->trace, 0,
                              (size_t)s->trace_phases * s->mega_grid * sg::kMegaTraceWidth * 8,
                              st));
    s->launches++;
    sg::mega_decode(a, s->mega_grid, s->mega_smem, st);
    // Every step of a launch has its own epoch; the next launch starts
    // after them (a CUDA graph would freeze this value, so the kernel is
    // launched directly, never captured).
    s->mega_epoch += (unsigned)steps;
  }

  // Chunk projection C[t] (op)= W a[t] for t < T: on the tensor cores when
  // the state has them (input split into bf16 halves, `ki` selects the
  // input maps by K), else on the SIMT tiles.
  void proj(const float* a, int K, int ki, const uint16_t* wraw, int wmap, int N, float* C,
            int ldc, sg::Epilogue epi, int T) {
    if (s->use_tc) {
      launch(FAM_OTHER, 0, [&] { sg::tc_split(a, K, T, K, s->a_hi, s->a_lo, st); });
      launch(FAM_OTHER, 0, [&] {
        sg::tc_gemm(s->tc_w[wmap], s->in[ki], T, C, ldc, epi, s->tc_err, st);
      });
    } else {
      launch(FAM_OTHER, 0, [&] { sg::gemm_simt(a, K, wraw, K, T, N, C, ldc, epi, st); });
    }
  }

  // MoE FFN of a chunk on the tensor cores, expert by expert (this rank's
  // experts). The tokens routed to each expert are known on the host after
  // one small read-back of the per-expert counts.
  void moe_experts_tc(int l, int T) {
    const Layer& ly = w->layer[l];
    const int D = w->D, F = w->F, k = w->topk, E = w->E;
    launch(FAM_OTHER, 0, [&] {
      sg::moe_group(s->eidx, T * k, E, s->moe_counts, s->moe_offsets, s->moe_perm, s->moe_inv,
                    st);
    });
    SG_CUDA(cudaMemcpyAsync(s->h_moe_counts, s->moe_counts, (size_t)E * sizeof(int),
                            cudaMemcpyDeviceToHost, st));
    SG_CUDA(cudaStreamSynchronize(st));
    const size_t gu_codes = (size_t)F * (D / 32) * 16, gu_scales = (size_t)F * (D / 32);
    const size_t d_codes = (size_t)D * (F / 32) * 16, d_scales = (size_t)D * (F / 32);
    int off = 0;
    for (int e = 0; e < E; e++) {
      const int n = s->h_moe_counts[e];
      if (n > 0 && e >= w->e_begin && e < w->e_end) {
        const size_t el = (size_t)(e - w->e_begin);
        launch(FAM_OTHER, 0, [&] {
          sg::mxfp4_to_bf16(ly.gate_c + el * gu_codes, ly.gate_s + el * gu_scales, F, D,
                            s->moe_wgu, 2, 0, st);
        });
        launch(FAM_OTHER, 0, [&] {
          sg::mxfp4_to_bf16(ly.up_c + el * gu_codes, ly.up_s + el * gu_scales, F, D, s->moe_wgu,
                            2, 1, st);
        });
        launch(FAM_OTHER, 0, [&] {
          sg::mxfp4_to_bf16(ly.down_c + el * d_codes, ly.down_s + el * d_scales, D, F,
                            s->moe_wd, 1, 0, st);
        });
        launch(FAM_OTHER, 0, [&] {
          sg::moe_gather_split(s->xn, D, s->moe_perm + off, k, n, s->a_hi, s->a_lo, st);
        });
        launch(FAM_OTHER, 0, [&] {
          sg::tc_gemm(s->tc_w[4 * w->L + 1], s->in[0], n, s->h, F, sg::EPI_SWIGLU, s->tc_err, st,
                      false);
        });
        launch(FAM_OTHER, 0, [&] { sg::tc_split(s->h, F, n, F, s->a_hi, s->a_lo, st); });
        launch(FAM_OTHER, 0, [&] {
          sg::tc_gemm(s->tc_w[4 * w->L + 2], s->in[2], n, s->moe_y + (size_t)off * D, D,
                      sg::EPI_STORE, s->tc_err, st, false);
        });
      }
      off += n;
    }
    launch(FAM_OTHER, 0, [&] {
      sg::moe_combine(rp_out(), s->ew, s->eidx, s->moe_inv, s->moe_y, T, k, D, w->e_begin,
                      w->e_end, st);
    });
  }

  // T > 1 tokens already in s->tok at host-known position pos0.
  void prefill_layers(int T, int pos0) {
    const int D = w->D, HD = w->HD, QD = w->QHl * HD;
    launch(FAM_OTHER, 0, [&] { sg::embed(s->tok, T, w->emb, D, s->x, st); });
    for (int l = 0; l < w->L; l++) {
      const Layer& ly = w->layer[l];
      launch(FAM_OTHER, 0, [&] { sg::rmsnorm_rows(s->x, T, D, ly.attn_norm, w->eps, s->xn, st); });
      proj(s->xn, D, 0, ly.wqkv, 4 * l + 0, w->QKVl, s->qkv, w->QKVl, sg::EPI_STORE, T);
      launch(FAM_QKV, 0, [&] { sg::qkv_post(qkv_args(l, T), st); });
      sg::AttnPrefillArgs a;
      a.q = s->q; a.k_cache = kc(l); a.v_cache = vc(l);
      a.T = T; a.KHl = w->KHl; a.G = w->G; a.HD = HD; a.ctx = s->ctx;
      a.pos0 = pos0; a.att = s->att;
      launch(FAM_ATTN, 0, [&] { sg::attn_prefill(a, st); });
      proj(s->att, QD, 1, ly.wo, 4 * l + 1, D, rp_out(), D, rp_epi(), T);
      rp_reduce(T);
      launch(FAM_OTHER, 0, [&] { sg::rmsnorm_rows(s->x, T, D, ly.ffn_norm, w->eps, s->xn, st); });
      if (w->moe) {
        launch(FAM_OTHER, 0, [&] { sg::gemm_simt(s->xn, D, ly.router, D, T, w->E, s->rl, w->E, sg::EPI_STORE, st); });
        launch(FAM_OTHER, 0, [&] { sg::moe_topk(s->rl, T, w->E, w->topk, s->eidx, s->ew, st); });
        moe_zero_part(T);
        if (s->use_tc) {
          moe_experts_tc(l, T);
        } else {
          sg::MoeArgs m = moe_args(l, T);
          launch(FAM_OTHER, 0, [&] { sg::moe_gate_up(m, st); });
          launch(FAM_OTHER, 0, [&] { sg::moe_down(m, st); });
        }
      } else {
        proj(s->xn, D, 0, ly.wgu, 4 * l + 2, 2 * w->Fl, s->h, w->Fl, sg::EPI_SWIGLU, T);
        proj(s->h, w->Fl, 2, ly.wd, 4 * l + 3, D, rp_out(), D, rp_epi(), T);
      }
      rp_reduce(T);
    }
  }

  // LM head for rows [r0, r0+n) of the chunk (n <= logit_rows_max); the
  // logits land in s->logits ([n][V]).
  void lm_head_rows(int r0, int n) {
    const int D = w->D;
    if (n == 1) {
      launch(FAM_LMHEAD, 0, [&] {
        sg::matvec(s->x + (size_t)r0 * D, w->out_norm, w->eps, w->out_w, D,
                   w->Vl, lm_out(), sg::EPI_STORE, st);
      });
    } else {
      launch(FAM_OTHER, 0, [&] { sg::rmsnorm_rows(s->x + (size_t)r0 * D, n, D, w->out_norm, w->eps, s->xn, st); });
      proj(s->xn, D, 0, w->out_w, 4 * w->L, w->Vl, lm_out(), w->Vl, sg::EPI_STORE, n);
    }
    lm_gather(n);
  }
};

void set_pos(S_t* s, int pos) {
  SG_CUDA(cudaMemcpyAsync(s->pos, &pos, sizeof(int), cudaMemcpyHostToDevice, s->stream));
}

void upload_tokens(const W_t* w, S_t* s, const int* tok, int T) {
  for (int i = 0; i < T; i++) {
    if (tok[i] < 0 || tok[i] >= w->V) {
      char msg[128];
      snprintf(msg, sizeof(msg), "token id %d out of range [0, %d)", tok[i], w->V);
      SG_DIE(msg);
    }
  }
  SG_CUDA(cudaMemcpyAsync(s->tok, tok, (size_t)T * sizeof(int),
                          cudaMemcpyHostToDevice, s->stream));
}

cudaGraphExec_t capture(Runner& r, bool greedy) {
  cudaGraph_t g;
  const size_t before = r.s->launches;
  SG_CUDA(cudaStreamBeginCapture(r.st, cudaStreamCaptureModeThreadLocal));
  r.decode_layers();
  if (greedy) r.argmax(1);
  SG_CUDA(cudaStreamEndCapture(r.st, &g));
  if (greedy) r.s->graph_nodes = r.s->launches - before;
  r.s->launches = before;
  cudaGraphExec_t e;
  SG_CUDA(cudaGraphInstantiate(&e, g, 0));
  SG_CUDA(cudaGraphDestroy(g));
  return e;
}

W_t* weights_of(transformer_t* t) { return (W_t*)t->weights; }
S_t* state_of(transformer_t* t) { return (S_t*)t->state; }

void require_connected(const W_t* w, const S_t* s) {
  if (w->world > 1 && !s->tp.connected)
    SG_DIE("tensor-parallel forward before strasgpt_tp_connect (world > 1)");
}

// After a synchronize: a megakernel barrier that timed out is fatal. With
// STRASGPT_MEGA_TRACE=<file>, the barrier timestamps of the last launch
// ([barrier][cta][arrive, release], uint64 ns) are written to <file>.
void check_device_errors(S_t* s) {
  if (s->use_tc) {
    int err = 0;
    SG_CUDA(cudaMemcpy(&err, s->tc_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) SG_DIE("tensor-core projection: a TMA or MMA pipeline wait timed out");
  }
  if (s->tp.world > 1) {
    int err = 0;
    SG_CUDA(cudaMemcpy(&err, s->tp.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err) SG_DIE("tensor-parallel exchange: a peer did not post within the time limit");
  }
  if (!s->use_mega) return;
  int err = 0;
  SG_CUDA(cudaMemcpy(&err, s->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) SG_DIE("decode megakernel: an input or weight copy wait timed out");
  if (s->trace) {
    const size_t n = (size_t)s->trace_phases * s->mega_grid * sg::kMegaTraceWidth;
    std::vector<unsigned long long> h(n);
    SG_CUDA(cudaMemcpy(h.data(), s->trace, n * 8, cudaMemcpyDeviceToHost));
    FILE* f = fopen(getenv("STRASGPT_MEGA_TRACE"), "wb");
    if (f) {
      const int hdr[3] = {s->trace_phases, s->mega_grid, sg::kMegaTraceWidth};
      fwrite(hdr, sizeof(hdr), 1, f);
      fwrite(h.data(), 8, n, f);
      fclose(f);
    }
  }
}

// Process `T` host tokens as chunks; copy logits of the last `n` of them to
// the host buffer `out` (row-major [n][V]).
void predict_impl(transformer_t* t, size_t T, const int* tok, size_t n,
                  float* out) {
  W_t* w = weights_of(t);
  S_t* s = state_of(t);
  const transformer_configuration_t* c = t->config;
  require_connected(w, s);
  SG_CUDA(cudaSetDevice(w->device));
  Runner r{w, s, c, s->stream};
  const size_t V = (size_t)w->V;
  const size_t lstart = T - n;
  for (size_t c0 = 0; c0 < T; c0 += (size_t)s->chunk_max) {
    const size_t Tc = std::min((size_t)s->chunk_max, T - c0);
    upload_tokens(w, s, tok + c0, (int)Tc);
    set_pos(s, (int)s->cached_count);
    const size_t lo = std::max(c0, lstart);
    if (Tc == 1) {
      if (s->use_mega) {
        // Under tensor parallelism each rank's LM-head rows land in its
        // slice; the gather puts every rank's slice into s->logits.
        r.mega(1, true);
        r.lm_gather(1);
      } else {
        if (!s->graph_logits) s->graph_logits = capture(r, false);
        SG_CUDA(cudaGraphLaunch(s->graph_logits, s->stream));
      }
      SG_CUDA(cudaMemcpyAsync(s->h_logits, s->logits, V * 4,
                              cudaMemcpyDeviceToHost, s->stream));
      SG_CUDA(cudaStreamSynchronize(s->stream));
      check_device_errors(s);
      memcpy(out + (lo - lstart) * V, s->h_logits, V * 4);
    } else {
      r.prefill_layers((int)Tc, (int)s->cached_count);
      for (size_t row = lo; row < c0 + Tc; row += (size_t)s->logit_rows_max) {
        const size_t nb = std::min((size_t)s->logit_rows_max, c0 + Tc - row);
        r.lm_head_rows((int)(row - c0), (int)nb);
        SG_CUDA(cudaMemcpyAsync(s->h_logits, s->logits, nb * V * 4,
                                cudaMemcpyDeviceToHost, s->stream));
        SG_CUDA(cudaStreamSynchronize(s->stream));
        memcpy(out + (row - lstart) * V, s->h_logits, nb * V * 4);
      }
    }
    s->cached_count += Tc;
  }
  SG_CUDA(cudaStreamSynchronize(s->stream));
  SG_CUDA(cudaGetLastError());
  if (T > 1) check_device_errors(s);
}

// Runs fn(rank, transformer) for every rank of a single-process group, rank
// 0 on the calling thread and each other rank on a thread of its own (the
// ranks' kernels wait for one another, so they must run concurrently).
template <typename Fn>
void on_ranks(W_t* g, Fn&& fn) {
  std::vector<std::thread> th;
  for (size_t r = 1; r < g->ranks.size(); r++)
    th.emplace_back([&fn, g, r] { fn((int)r, g->ranks[r]); });
  fn(0, g->ranks[0]);
  for (auto& x : th) x.join();
}

bool is_group(transformer_t* t) { return t && !weights_of(t)->ranks.empty(); }

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int strasgpt_set_placement(int rank, int world, int device) {
  if (world == 0) {
    g_rank = g_world = g_device = -1;
    return 0;
  }
  if (world != 1 && world != 2 && world != 4 && world != 8) return -1;
  if (rank < 0 || rank >= world || device < 0) return -1;
  g_rank = rank;
  g_world = world;
  g_device = device;
  return 0;
}

int strasgpt_tp_handle(transformer_t* t, void* handle) {
  if (!t || !handle) return -1;
  W_t* w = weights_of(t);
  S_t* s = state_of(t);
  if (w->world == 1) return -1;
  SG_CUDA(cudaSetDevice(w->device));
  sg::tp_handle(s->tp, handle);
  return 0;
}

int strasgpt_tp_connect(transformer_t* t, const void* handles) {
  if (!t || !handles) return -1;
  W_t* w = weights_of(t);
  S_t* s = state_of(t);
  if (w->world == 1) return -1;
  SG_CUDA(cudaSetDevice(w->device));
  sg::tp_connect(&s->tp, handles);
  return 0;
}

// STRASGPT_NGPU=N (2, 4 or 8, without strasgpt_set_placement): N ranks of
// a tensor-parallel group on GPUs 0..N-1 of this process, connected through
// direct peer access; the caller gets one transformer_t that runs them all.
static transformer_t* group_from_safetensors(struct safetensors* st, int n) {
  if (n != 2 && n != 4 && n != 8) SG_DIE("STRASGPT_NGPU must be 1, 2, 4 or 8");
  int ndev = 0;
  SG_CUDA(cudaGetDeviceCount(&ndev));
  if (ndev < n) SG_DIE("STRASGPT_NGPU is larger than the number of visible GPUs");
  W_t* g = new W_t();
  for (int r = 0; r < n; r++) {
    g_rank = r;
    g_world = n;
    g_device = r;
    g->ranks.push_back(transformer_from_safetensors(st));
  }
  g_rank = g_world = g_device = -1;
  std::vector<unsigned char*> bufs(n);
  std::vector<int> devs(n);
  for (int r = 0; r < n; r++) {
    bufs[r] = state_of(g->ranks[r])->tp.local;
    devs[r] = weights_of(g->ranks[r])->device;
  }
  for (int r = 0; r < n; r++) {
    SG_CUDA(cudaSetDevice(devs[r]));
    sg::tp_connect_local(&state_of(g->ranks[r])->tp, bufs.data(), devs.data());
  }
  SG_CUDA(cudaSetDevice(devs[0]));
  transformer_t* t = (transformer_t*)calloc(1, sizeof(*t));
  if (!t) SG_DIE("failed to malloc for transformer_t");
  // The configuration and state the caller may read are rank 0's.
  t->config = g->ranks[0]->config;
  t->weights = (transformer_weights_t*)g;
  t->state = g->ranks[0]->state;
  return t;
}

transformer_t* transformer_from_safetensors(struct safetensors* st) {
  if (!st) SG_DIE("NULL safetensors");
  if (g_world < 0 && env_int("STRASGPT_NGPU", 1) > 1)
    return group_from_safetensors(st, env_int("STRASGPT_NGPU", 1));
  transformer_t* t = (transformer_t*)calloc(1, sizeof(*t));
  transformer_configuration_t* c = (transformer_configuration_t*)calloc(1, sizeof(*c));
  if (!t || !c) SG_DIE("failed to malloc for transformer_t");
  // Configuration, as source/transformer.c:17-58.
  c->embedding_dim = st->embedding_dim;
  c->head_dim = st->head_dim;
  c->hidden_dim = st->hidden_dim;
  c->layer_count = st->layer_count;
  c->q_head_count = st->q_head_count;
  c->kv_head_count = st->kv_head_count;
  c->vocabulary_len = st->vocabulary_len;
  c->context_len = st->context_len;
  c->epsilon = st->epsilon;
  c->rope_theta = st->rope_theta;
  if (st->rope_interleaved) {
    c->rope_pair_bound = st->head_dim;
    c->rope_pair_offset = 1;
    c->rope_pair_stride = 2;
  } else {
    c->rope_pair_bound = st->head_dim / 2;
    c->rope_pair_offset = st->head_dim / 2;
    c->rope_pair_stride = 1;
  }
  c->mrope_section_count = st->mrope_section_count;
  if (c->mrope_section_count) {
    c->mrope_section = (size_t*)calloc(c->mrope_section_count, sizeof(size_t));
    for (size_t i = 0; i < c->mrope_section_count; i++)
      c->mrope_section[i] = st->mrope_section[i];
  }
  c->aliased_out_weight = safetensors_aliased_out_weight(st);
  t->config = c;

  W_t* w = new W_t();
  w->rank = g_rank >= 0 ? g_rank : env_int("STRASGPT_TP_RANK", 0);
  w->world = g_world >= 0 ? g_world : env_int("STRASGPT_TP_SIZE", 1);
  w->device = g_device >= 0 ? g_device : env_int("STRASGPT_DEVICE", 0);
  w->D = (int)c->embedding_dim;
  w->HD = (int)c->head_dim;
  w->F = (int)c->hidden_dim;
  w->L = (int)c->layer_count;
  w->QH = (int)c->q_head_count;
  w->KH = (int)c->kv_head_count;
  w->V = (int)c->vocabulary_len;
  w->eps = c->epsilon;
  w->moe = st->expert_count > 0;
  w->E = (int)st->expert_count;
  w->topk = (int)st->expert_top_k;
  w->qk_norm = has_qk_norm(st);
  const int N = w->world;
  if (w->D <= 0 || w->HD <= 0 || w->L <= 0 || w->QH <= 0 || w->KH <= 0 ||
      w->V <= 0 || w->F <= 0 || c->context_len == 0)
    SG_DIE("invalid model configuration");
  if (w->QH % w->KH) SG_DIE("q_head_count must be a multiple of kv_head_count");
  if (w->D % 32 || w->F % 32 || (w->QH * w->HD) % 32)
    SG_DIE("embedding, hidden and attention dims must be multiples of 32");
  if (w->HD != 32 && w->HD != 64 && w->HD != 128)
    SG_DIE("head_dim must be 32, 64 or 128");
  if (w->KH % N || w->V % N) SG_DIE("kv heads and vocabulary must divide by the GPU count");
  w->G = w->QH / w->KH;
  if (w->G != 1 && w->G != 2 && w->G != 4 && w->G != 8)
    SG_DIE("GQA group (q heads per kv head) must be 1, 2, 4 or 8");
  w->KHl = w->KH / N;
  w->QHl = w->KHl * w->G;
  w->Vl = w->V / N;
  w->QKVl = (w->QHl + 2 * w->KHl) * w->HD;
  if (w->moe) {
    if (w->topk <= 0 || w->topk > w->E || w->topk > 16 || w->E > 256)
      SG_DIE("unsupported expert count / top-k");
    if (w->E % N) SG_DIE("expert count must divide by the GPU count");
    w->El = w->E / N;
    w->e_begin = w->rank * w->El;
    w->e_end = w->e_begin + w->El;
    w->Fl = w->F;
  } else {
    if ((w->F / N) % SG_GU_GROUP) SG_DIE("FFN shard must be a multiple of the gate/up group");
    w->Fl = w->F / N;
  }
  SG_CUDA(cudaSetDevice(w->device));
  sg::configure_kernels();
  load_weights(w, st);
  t->weights = (transformer_weights_t*)w;

  S_t* s = new S_t();
  alloc_state(w, c, s);
  t->state = (transformer_state_t*)s;
  SG_CUDA(cudaDeviceSynchronize());
  return t;
}

void transformer_free(transformer_t* t) {
  if (!t) return;
  if (is_group(t)) {
    // Every rank's final barrier exchange needs the others running.
    W_t* g = weights_of(t);
    on_ranks(g, [](int, transformer_t* r) { transformer_free(r); });
    delete g;
    free(t);
    return;
  }
  W_t* w = weights_of(t);
  S_t* s = state_of(t);
  if (w) SG_CUDA(cudaSetDevice(w->device));
  if (s) {
    if (s->graph_logits) cudaGraphExecDestroy(s->graph_logits);
    if (s->graph_greedy) cudaGraphExecDestroy(s->graph_greedy);
    for (auto e : s->ev)
      if (e) cudaEventDestroy(e);
    if (s->h_logits) cudaFreeHost(s->h_logits);
    if (s->h_moe_counts) cudaFreeHost(s->h_moe_counts);
    for (auto e : s->prof_ev) cudaEventDestroy(e);
    if (s->tp.local) sg::tp_free(&s->tp, s->stream);
    if (s->stream) cudaStreamDestroy(s->stream);
    for (void* p : s->allocs) cudaFree(p);
    delete s;
  }
  if (w) {
    for (void* p : w->allocs) cudaFree(p);
    delete w;
  }
  if (t->config) {
    free(t->config->mrope_section);
    free(t->config);
  }
  free(t);
}

void transformer_print(FILE* f, const transformer_t* t) {
  if (!t) {
    fprintf(f, "transformer: NULL\n");
    return;
  }
  if (is_group(const_cast<transformer_t*>(t))) {
    const W_t* g = (const W_t*)t->weights;
    fprintf(f, "Tensor-parallel group of %zu GPUs in this process (STRASGPT_NGPU):\n",
            g->ranks.size());
    for (transformer_t* r : g->ranks) transformer_print(f, r);
    return;
  }
  const transformer_configuration_t* c = t->config;
  const W_t* w = (const W_t*)t->weights;
  fprintf(f, "Transformer (strasgpt-b200, CUDA sm_100a):\n");
  fprintf(f, "- Configuration:\n");
  fprintf(f, "--- embedding_dim:      %zu\n", c->embedding_dim);
  fprintf(f, "--- head_dim:           %zu\n", c->head_dim);
  fprintf(f, "--- hidden_dim:         %zu\n", c->hidden_dim);
  fprintf(f, "--- layer_count:        %zu\n", c->layer_count);
  fprintf(f, "--- q_head_count:       %zu\n", c->q_head_count);
  fprintf(f, "--- kv_head_count:      %zu\n", c->kv_head_count);
  fprintf(f, "--- vocabulary_len:     %zu\n", c->vocabulary_len);
  fprintf(f, "--- context_len:        %zu\n", c->context_len);
  fprintf(f, "--- epsilon:            %g\n", c->epsilon);
  fprintf(f, "--- rope_theta:         %.1f\n", c->rope_theta);
  fprintf(f, "--- rope_pair_bound     %zu\n", c->rope_pair_bound);
  fprintf(f, "--- rope_pair_offset    %zu\n", c->rope_pair_offset);
  fprintf(f, "--- rope_pair_stride    %zu\n", c->rope_pair_stride);
  fprintf(f, "--- aliased_out_weight: %s\n", c->aliased_out_weight ? "true" : "false");
  if (w) {
    if (w->moe) fprintf(f, "--- experts:            %d (top-%d)\n", w->E, w->topk);
    fprintf(f, "- Placement: rank %d of %d on CUDA device %d\n", w->rank, w->world,
            w->device);
    fprintf(f, "- Device weights: %.4f GB\n",
            (double)w->device_bytes / (1024.0 * 1024.0 * 1024.0));
  }
}

float* transformer_logits_malloc(transformer_t* t, size_t logits_count,
                                 size_t* vocabulary_len) {
  if (!t || !vocabulary_len) return NULL;
  *vocabulary_len = t->config->vocabulary_len;
  float* p = (float*)malloc(logits_count * (*vocabulary_len) * sizeof(float));
  if (!p) SG_DIE("failed to malloc for logits");
  return p;
}

void transformer_predict(transformer_t* t, size_t token_count, int* token,
                         size_t logits_count, float* logits) {
  if (!t || !logits || !token || token_count == 0 || logits_count == 0) return;
#pragma omp single
  {
    S_t* s = state_of(t);
    if (token_count + s->cached_count > t->config->context_len)
      SG_DIE("context length exhausted");
    if (logits_count > token_count) logits_count = token_count;
    if (is_group(t)) {
      // Every rank ends with the full logits; rank 0's go to the caller.
      W_t* g = weights_of(t);
      const size_t n = logits_count * t->config->vocabulary_len;
      std::vector<std::vector<float>> spare(g->ranks.size());
      for (size_t r = 1; r < spare.size(); r++) spare[r].resize(n);
      on_ranks(g, [&](int r, transformer_t* tr) {
        predict_impl(tr, token_count, token, logits_count, r == 0 ? logits : spare[r].data());
      });
    } else {
      predict_impl(t, token_count, token, logits_count, logits);
    }
  }
}

int transformer_generate_greedy(transformer_t* t, size_t P, const int* prompt,
                                size_t S, int* out_tokens,
                                strasgpt_timing_t* timing) {
  if (!t || !prompt || P == 0 || !out_tokens) SG_DIE("invalid arguments");
  if (is_group(t)) {
    W_t* g = weights_of(t);
    std::vector<std::vector<int>> toks(g->ranks.size());
    std::vector<strasgpt_timing_t> tms(g->ranks.size());
    for (size_t r = 1; r < toks.size(); r++) toks[r].resize(S + 1);
    on_ranks(g, [&](int r, transformer_t* tr) {
      transformer_generate_greedy(tr, P, prompt, S, r == 0 ? out_tokens : toks[r].data(),
                                  &tms[r]);
    });
    if (timing) {
      // Device times: the slowest rank.
      *timing = tms[0];
      for (const auto& x : tms) {
        timing->prefill_ms = std::max(timing->prefill_ms, x.prefill_ms);
        timing->decode_ms = std::max(timing->decode_ms, x.decode_ms);
      }
    }
    return 0;
  }
  W_t* w = weights_of(t);
  S_t* st = state_of(t);
  require_connected(w, st);
  if (P + S + st->cached_count > t->config->context_len)
    SG_DIE("context length exhausted");
  SG_CUDA(cudaSetDevice(w->device));
  Runner r{w, st, t->config, st->stream};
  if (!st->use_mega && !st->graph_greedy) st->graph_greedy = capture(r, true);
  const int zero = 0;
  SG_CUDA(cudaMemcpyAsync(st->step, &zero, 4, cudaMemcpyHostToDevice, st->stream));
  const size_t launches0 = st->launches;
  SG_CUDA(cudaEventRecord(st->ev[0], st->stream));
  for (size_t c0 = 0; c0 < P; c0 += (size_t)st->chunk_max) {
    const size_t Tc = std::min((size_t)st->chunk_max, P - c0);
    upload_tokens(w, st, prompt + c0, (int)Tc);
    set_pos(st, (int)st->cached_count);
    if (Tc == 1) {
      r.decode_layers();
    } else {
      r.prefill_layers((int)Tc, (int)st->cached_count);
      if (c0 + Tc == P) r.lm_head_rows((int)Tc - 1, 1);
    }
    st->cached_count += Tc;
  }
  // First generated token from the prompt's last logits; the position is
  // already past the prompt.
  set_pos(st, (int)st->cached_count);
  r.argmax(0);
  SG_CUDA(cudaEventRecord(st->ev[1], st->stream));
  size_t graph_replays = 0;
  const size_t launches_prefill = st->launches;
  if (st->use_mega) {
    if (S > 0) r.mega((int)S, false);
  } else {
    for (size_t i = 0; i < S; i++) SG_CUDA(cudaGraphLaunch(st->graph_greedy, st->stream));
    graph_replays = S;
  }
  SG_CUDA(cudaEventRecord(st->ev[2], st->stream));
  SG_CUDA(cudaMemcpyAsync(out_tokens, st->gen, (S + 1) * sizeof(int),
                          cudaMemcpyDeviceToHost, st->stream));
  SG_CUDA(cudaStreamSynchronize(st->stream));
  SG_CUDA(cudaGetLastError());
  check_device_errors(st);
  st->cached_count += S;
  if (timing) {
    float a = 0, b = 0;
    SG_CUDA(cudaEventElapsedTime(&a, st->ev[0], st->ev[1]));
    SG_CUDA(cudaEventElapsedTime(&b, st->ev[1], st->ev[2]));
    timing->prefill_ms = a;
    timing->decode_ms = b;
    timing->prefill_tokens = P;
    timing->decode_steps = S;
    timing->kernel_launches = st->launches - launches0 + graph_replays * st->graph_nodes;
    timing->decode_launches = st->launches - launches_prefill + graph_replays * st->graph_nodes;
  }
  return 0;
}

void transformer_reset(transformer_t* t) {
  if (is_group(t))
    for (transformer_t* r : weights_of(t)->ranks) transformer_reset(r);
  else if (t)
    state_of(t)->cached_count = 0;
}

size_t transformer_cached_count(const transformer_t* t) {
  return t ? ((const S_t*)t->state)->cached_count : 0;
}

int strasgpt_profile_decode(transformer_t* t, int first_token, size_t steps,
                            strasgpt_kernel_profile_t* prof) {
  if (!t || !prof) SG_DIE("invalid arguments");
  if (is_group(t)) {
    W_t* g = weights_of(t);
    std::vector<strasgpt_kernel_profile_t> spare(g->ranks.size());
    on_ranks(g, [&](int r, transformer_t* tr) {
      strasgpt_profile_decode(tr, first_token, steps, r == 0 ? prof : &spare[r]);
    });
    return 0;
  }
  W_t* w = weights_of(t);
  S_t* st = state_of(t);
  require_connected(w, st);
  if (st->cached_count + steps > t->config->context_len)
    SG_DIE("context length exhausted");
  SG_CUDA(cudaSetDevice(w->device));
  memset(prof, 0, sizeof(*prof));
  Runner r{w, st, t->config, st->stream};
  upload_tokens(w, st, &first_token, 1);
  set_pos(st, (int)st->cached_count);
  const int zero = 0;
  SG_CUDA(cudaMemcpyAsync(st->step, &zero, 4, cudaMemcpyHostToDevice, st->stream));
  for (size_t i = 0; i < steps; i++) {
    // Hold the GPU ~2 ms so the host enqueues the whole step first: the
    // event pairs then time the kernels, not the host's launch rate.
    sg::gpu_sleep_cycles(4000000LL, st->stream);
    st->prof = prof;
    r.decode_layers();
    r.argmax(1);
    st->prof = nullptr;
    SG_CUDA(cudaStreamSynchronize(st->stream));
    for (size_t j = 0; j < st->prof_fam.size(); j++) {
      float ms = 0;
      SG_CUDA(cudaEventElapsedTime(&ms, st->prof_ev[2 * j], st->prof_ev[2 * j + 1]));
      const int f = st->prof_fam[j];
      prof->launches[f] += 1;
      prof->ms[f] += ms;
      prof->bytes[f] += st->prof_bytes[j];
    }
    // attention bytes: K and V rows [0, pos] of every layer
    const double pos = (double)(st->cached_count + i);
    prof->bytes[FAM_ATTN] += 2.0 * w->L * w->KHl * (pos + 1) * w->HD * 4;
    st->prof_fam.clear();
    st->prof_bytes.clear();
  }
  st->cached_count += steps;
  SG_CUDA(cudaGetLastError());
  return 0;
}

}  // extern "C"
