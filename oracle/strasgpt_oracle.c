// ORACLE — test infrastructure only. Nothing in the product path links,
// loads or calls this file; tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline leg use it as the checker.
//
// A plain-C restatement of StrasGPT's forward pass (source/transformer.c of
// the reference) on the CPU, in fp32 like the reference, extended with the
// mixture-of-experts FFN over MXFP4 experts that the reference lacks:
//   embedding gather                  source/transformer.c:1247-1255
//   rmsnorm                           source/transformer.c:978-999
//   K/V/Q projections into the cache  source/transformer.c:1271-1291,1327-1338
//   q/k per-head rmsnorm              source/transformer.c:1293-1307,1340-1356
//   RoPE table and rotation           source/transformer.c:126-146,1309-1323,1358-1373
//   causal GQA attention              source/transformer.c:1375-1422
//   o_proj + residual                 source/transformer.c:1426-1445
//   FFN gate/up, SwiGLU, down         source/transformer.c:1449-1504
//   final norm + LM head              source/transformer.c:1580-1601
//   logits row placement              source/transformer.c:1637-1666
// MoE (no reference counterpart; semantics fixed by this project):
//   router logits r = W_r . ffn_norm(x) (bf16 W, fp32 accumulation);
//   top-k by value, ties to the lower expert index; weights = softmax over
//   the k selected logits; out = sum_j w_j * down_j(silu(gate_j x) * up_j x)
//   with MXFP4 weights: value = e2m1(code) * 2^(e8m0 - 127), 32 values per
//   scale along the input dimension, even element in the low nibble
//   (OCP Microscaling Formats v1.0, e2m1 and e8m0 element/scale types).
//
// Pinning: the dense path is checked against the reference's own
// transformer_predict compiled from its sources (oracle/Makefile ->
// oracle/_ref/) by tests/test_oracle.py. The MoE path has no reference and
// is pinned only by a float64 numpy restatement in the same test.
#include "safetensors.h"

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_CHUNK 512

typedef struct {
  uint16_t *attn_norm, *q, *k, *v, *o, *qn, *kn, *ffn_norm, *gate, *up, *down;
  uint16_t* router;
  uint8_t *gate_c, *gate_s, *up_c, *up_s, *down_c, *down_s;
} olayer_t;

typedef struct oracle {
  int D, HD, F, L, QH, KH, V, ctx, E, topk;
  float eps;
  bool interleaved, qk_norm, tied;
  float rope_theta;
  uint16_t *emb, *out, *out_norm;
  olayer_t* layer;
  float *kc, *vc, *rope;  // [L][KH][ctx][HD], [ctx][HD]
  size_t cached;
  // Smallest gap, over the tokens and layers of the last oracle_predict,
  // between the k-th selected router logit and the best unselected one
  // (INFINITY for dense models): below ~1e-5 the expert choice depends on
  // the fp32 summation order, so two correct implementations may differ.
  float min_router_gap;
} oracle_t;

static void die(const char* m) {
  fprintf(stderr, "[oracle] Error: %s\n", m);
  exit(EXIT_FAILURE);
}

static inline float bf(uint16_t w) {
  union { uint32_t u; float f; } u = {(uint32_t)w << 16};
  return u.f;
}

static void* xcalloc(size_t n) {
  void* p = calloc(1, n ? n : 1);
  if (!p) die("out of memory");
  return p;
}

static void* read_tensor(const safetensors_t* s, const char* name,
                         size_t expect) {
  for (size_t i = 0; i < s->tensor_count; i++) {
    if (strcmp(s->tensor[i].name, name) != 0) continue;
    const safetensors_tensor_t* t = &s->tensor[i];
    if (t->size != expect) {
      fprintf(stderr, "[oracle] %s: size %zu, expected %zu\n", name, t->size,
              expect);
      die("bad tensor size");
    }
    void* p = xcalloc(t->size);
    FILE* f = fopen(s->file[t->file], "rb");
    if (!f || fseek(f, (long)t->offset, SEEK_SET) != 0 ||
        fread(p, 1, t->size, f) != t->size)
      die("cannot read tensor");
    fclose(f);
    return p;
  }
  return NULL;
}

static void* need_tensor(const safetensors_t* s, const char* name,
                         size_t expect) {
  void* p = read_tensor(s, name, expect);
  if (!p) {
    fprintf(stderr, "[oracle] missing tensor %s\n", name);
    die("missing tensor");
  }
  return p;
}

oracle_t* oracle_load(const char* dir) {
  safetensors_t* s = parser_parse_safetensors(dir);
  oracle_t* o = xcalloc(sizeof(*o));
  o->D = (int)s->embedding_dim;
  o->HD = (int)s->head_dim;
  o->F = (int)s->hidden_dim;
  o->L = (int)s->layer_count;
  o->QH = (int)s->q_head_count;
  o->KH = (int)s->kv_head_count;
  o->V = (int)s->vocabulary_len;
  o->ctx = (int)s->context_len;
  o->eps = s->epsilon;
  o->rope_theta = s->rope_theta;
  o->interleaved = s->rope_interleaved;
  o->E = (int)s->expert_count;
  o->topk = (int)s->expert_top_k;
  o->min_router_gap = INFINITY;
  const size_t D = o->D, HD = o->HD, F = o->F, V = o->V;
  const size_t QD = (size_t)o->QH * HD, KD = (size_t)o->KH * HD;
  o->emb = need_tensor(s, "model.embed_tokens.weight", V * D * 2);
  o->out_norm = need_tensor(s, "model.norm.weight", D * 2);
  o->out = read_tensor(s, "lm_head.weight", V * D * 2);
  o->tied = (o->out == NULL);
  if (o->tied) o->out = o->emb;
  o->layer = xcalloc(sizeof(olayer_t) * (size_t)o->L);
  char n[512];
#define P(fmt) (snprintf(n, sizeof(n), "model.layers.%d." fmt, l), n)
  for (int l = 0; l < o->L; l++) {
    olayer_t* y = &o->layer[l];
    y->attn_norm = need_tensor(s, P("input_layernorm.weight"), D * 2);
    y->q = need_tensor(s, P("self_attn.q_proj.weight"), QD * D * 2);
    y->k = need_tensor(s, P("self_attn.k_proj.weight"), KD * D * 2);
    y->v = need_tensor(s, P("self_attn.v_proj.weight"), KD * D * 2);
    y->o = need_tensor(s, P("self_attn.o_proj.weight"), D * QD * 2);
    y->qn = read_tensor(s, P("self_attn.q_norm.weight"), HD * 2);
    y->kn = read_tensor(s, P("self_attn.k_norm.weight"), HD * 2);
    y->ffn_norm = need_tensor(s, P("post_attention_layernorm.weight"), D * 2);
    if (o->E) {
      const size_t E = o->E;
      y->router = need_tensor(s, P("mlp.router.weight"), E * D * 2);
      y->gate_c = need_tensor(s, P("mlp.experts.gate_proj_blocks"), E * F * D / 2);
      y->gate_s = need_tensor(s, P("mlp.experts.gate_proj_scales"), E * F * D / 32);
      y->up_c = need_tensor(s, P("mlp.experts.up_proj_blocks"), E * F * D / 2);
      y->up_s = need_tensor(s, P("mlp.experts.up_proj_scales"), E * F * D / 32);
      y->down_c = need_tensor(s, P("mlp.experts.down_proj_blocks"), E * D * F / 2);
      y->down_s = need_tensor(s, P("mlp.experts.down_proj_scales"), E * D * F / 32);
    } else {
      y->gate = need_tensor(s, P("mlp.gate_proj.weight"), F * D * 2);
      y->up = need_tensor(s, P("mlp.up_proj.weight"), F * D * 2);
      y->down = need_tensor(s, P("mlp.down_proj.weight"), D * F * 2);
    }
  }
#undef P
  o->qk_norm = o->layer[0].qn != NULL;
  safetensors_free(s);
  const size_t kv = (size_t)o->L * KD * o->ctx;
  o->kc = xcalloc(kv * 4);
  o->vc = xcalloc(kv * 4);
  // RoPE table (source/transformer.c:126-146)
  o->rope = xcalloc((size_t)o->ctx * HD * 4);
  size_t bound = HD / 2, off = HD / 2, stride = 1;
  float coef = 2.0f;
  if (o->interleaved) {
    bound = HD;
    off = 1;
    stride = 2;
    coef = 1.0f;
  }
  for (size_t i = 0; i < (size_t)o->ctx; i++)
    for (size_t j = 0; j < bound; j += stride) {
      float freq = 1.0f / powf(o->rope_theta, (coef * j) / HD);
      float val = i * freq;
      o->rope[i * HD + j] = cosf(val);
      o->rope[i * HD + j + off] = sinf(val);
    }
  return o;
}

int oracle_vocab(const oracle_t* o) { return o->V; }
float oracle_min_router_gap(const oracle_t* o) { return o->min_router_gap; }
size_t oracle_cached(const oracle_t* o) { return o->cached; }
void oracle_reset(oracle_t* o) { o->cached = 0; }

// fp32 dot with eight running partial sums.
static float dot_bf16(const float* a, const uint16_t* w, size_t n) {
  float acc[8] = {0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; j++) acc[j] += a[i + j] * bf(w[i + j]);
  float s = 0;
  for (; i < n; i++) s += a[i] * bf(w[i]);
  for (int j = 0; j < 8; j++) s += acc[j];
  return s;
}

static float dot_f32(const float* a, const float* b, size_t n) {
  float acc[8] = {0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; j++) acc[j] += a[i + j] * b[i + j];
  float s = 0;
  for (; i < n; i++) s += a[i] * b[i];
  for (int j = 0; j < 8; j++) s += acc[j];
  return s;
}

static void rmsnorm(size_t n, float* y, const float* x, const uint16_t* w,
                    float eps) {
  float ss = 0.0f;
  for (size_t j = 0; j < n; j++) ss += x[j] * x[j];
  ss /= n;
  ss = (float)(1. / sqrtf(ss + eps));
  for (size_t j = 0; j < n; j++) y[j] = (x[j] * ss) * bf(w[j]);
}

// out[t][r] (op)= dot(in[t], W[r]) for T rows of input, R rows of W.
static void project(size_t T, size_t K, const float* in, size_t ldi,
                    const uint16_t* W, size_t R, float* out, size_t ldo,
                    int add) {
#pragma omp parallel for schedule(static)
  for (size_t r = 0; r < R; r++) {
    for (size_t t = 0; t < T; t++) {
      float v = dot_bf16(in + t * ldi, W + r * K, K);
      if (add)
        out[t * ldo + r] += v;
      else
        out[t * ldo + r] = v;
    }
  }
}

static const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

static float e8m0(uint8_t e) { return ldexpf(1.0f, (int)e - 127); }

// Dequantise one MXFP4 row of K values.
static void mxfp4_row(const uint8_t* codes, const uint8_t* scales, size_t K,
                      float* out) {
  for (size_t b = 0; b < K / 32; b++) {
    const float s = e8m0(scales[b]);
    for (size_t j = 0; j < 16; j++) {
      const uint8_t byte = codes[b * 16 + j];
      out[b * 32 + 2 * j] = kE2M1[byte & 0xF] * s;
      out[b * 32 + 2 * j + 1] = kE2M1[byte >> 4] * s;
    }
  }
}

static void rope_rotate(const oracle_t* o, float* v, size_t pos) {
  const size_t HD = o->HD;
  size_t bound = HD / 2, off = HD / 2, stride = 1;
  if (o->interleaved) {
    bound = HD;
    off = 1;
    stride = 2;
  }
  const float* cs = o->rope + pos * HD;
  for (size_t h = 0; h < bound; h += stride) {
    float fr = cs[h], fi = cs[h + off];
    float v0 = v[h], v1 = v[h + off];
    v[h] = v0 * fr - v1 * fi;
    v[h + off] = v0 * fi + v1 * fr;
  }
}

static void moe_ffn(const oracle_t* o, const olayer_t* y, size_t T,
                    const float* xn, float* x) {
  const size_t D = o->D, F = o->F, E = o->E, K = o->topk;
  float* rl = xcalloc(T * E * 4);
  project(T, D, xn, D, y->router, E, rl, E, 0);
  int* idx = xcalloc(T * K * sizeof(int));
  float* wt = xcalloc(T * K * 4);
  for (size_t t = 0; t < T; t++) {
    float r[256];
    for (size_t e = 0; e < E; e++) r[e] = rl[t * E + e];
    float sel[16];
    for (size_t j = 0; j < K; j++) {
      size_t best = 0;
      int found = 0;
      for (size_t e = 0; e < E; e++) {
        if (r[e] == -INFINITY) continue;
        if (!found || r[e] > r[best]) {
          best = e;
          found = 1;
        }
      }
      idx[t * K + j] = (int)best;
      sel[j] = r[best];
      r[best] = -INFINITY;
    }
    float next = -INFINITY;
    for (size_t e = 0; e < E; e++)
      if (r[e] > next) next = r[e];
    const float gap = sel[K - 1] - next;
#pragma omp critical
    if (gap < ((oracle_t*)o)->min_router_gap) ((oracle_t*)o)->min_router_gap = gap;
    float sum = 0, ex[16];
    for (size_t j = 0; j < K; j++) {
      ex[j] = expf(sel[j] - sel[0]);
      sum += ex[j];
    }
    for (size_t j = 0; j < K; j++) wt[t * K + j] = ex[j] / sum;
  }
  // h[t][j][f]; computed expert by expert so each expert row is decoded once.
  float* h = xcalloc(T * K * F * 4);
  float* y_out = xcalloc(T * K * D * 4);
  for (size_t e = 0; e < E; e++) {
    size_t cnt = 0;
    for (size_t q = 0; q < T * K; q++) cnt += (idx[q] == (int)e);
    if (!cnt) continue;
#pragma omp parallel
    {
      float* wg = xcalloc(D * 4);
      float* wu = xcalloc(D * 4);
#pragma omp for schedule(static)
      for (size_t f = 0; f < F; f++) {
        const size_t row = e * F + f;
        mxfp4_row(y->gate_c + row * D / 2, y->gate_s + row * D / 32, D, wg);
        mxfp4_row(y->up_c + row * D / 2, y->up_s + row * D / 32, D, wu);
        for (size_t q = 0; q < T * K; q++) {
          if (idx[q] != (int)e) continue;
          const float* xt = xn + (q / K) * D;
          float g = dot_f32(xt, wg, D);
          float u = dot_f32(xt, wu, D);
          g *= (1.0f / (1.0f + expf(-g)));
          h[q * F + f] = g * u;
        }
      }
      free(wg);
      free(wu);
      float* wd = xcalloc(F * 4);
#pragma omp for schedule(static)
      for (size_t r = 0; r < D; r++) {
        const size_t row = e * D + r;
        mxfp4_row(y->down_c + row * F / 2, y->down_s + row * F / 32, F, wd);
        for (size_t q = 0; q < T * K; q++) {
          if (idx[q] != (int)e) continue;
          y_out[q * D + r] = dot_f32(h + q * F, wd, F);
        }
      }
      free(wd);
    }
  }
  for (size_t t = 0; t < T; t++)
    for (size_t r = 0; r < D; r++) {
      float acc = 0.0f;
      for (size_t j = 0; j < K; j++) acc += wt[t * K + j] * y_out[(t * K + j) * D + r];
      x[t * D + r] += acc;
    }
  free(rl);
  free(idx);
  free(wt);
  free(h);
  free(y_out);
}

// One chunk of T tokens at position o->cached; logits of the last n rows.
static void predict_chunk(oracle_t* o, size_t T, const int* tok, size_t n,
                          float* logits) {
  const size_t D = o->D, HD = o->HD, F = o->F, QH = o->QH, KH = o->KH;
  const size_t G = QH / KH, ctx = o->ctx, c0 = o->cached;
  float* x = xcalloc(T * D * 4);
  float* xn = xcalloc(T * D * 4);
  float* q = xcalloc(T * QH * HD * 4);
  float* kv = xcalloc(T * KH * HD * 4);
  float* att = xcalloc(T * QH * HD * 4);
  float* fc = o->E ? NULL : xcalloc(T * F * 4);
  float* up = o->E ? NULL : xcalloc(T * F * 4);
  for (size_t t = 0; t < T; t++)
    for (size_t e = 0; e < D; e++) x[t * D + e] = bf(o->emb[(size_t)tok[t] * D + e]);
  for (int l = 0; l < o->L; l++) {
    const olayer_t* y = &o->layer[l];
    float* kc = o->kc + (size_t)l * KH * ctx * HD;
    float* vc = o->vc + (size_t)l * KH * ctx * HD;
    for (size_t t = 0; t < T; t++) rmsnorm(D, xn + t * D, x + t * D, y->attn_norm, o->eps);
    // K and V rows into the cache
    project(T, D, xn, D, y->k, KH * HD, kv, KH * HD, 0);
    for (size_t t = 0; t < T; t++)
      for (size_t k = 0; k < KH; k++) {
        float* dst = kc + (k * ctx + c0 + t) * HD;
        memcpy(dst, kv + (t * KH + k) * HD, HD * 4);
        if (y->kn) rmsnorm(HD, dst, dst, y->kn, o->eps);
        rope_rotate(o, dst, c0 + t);
      }
    project(T, D, xn, D, y->v, KH * HD, kv, KH * HD, 0);
    for (size_t t = 0; t < T; t++)
      for (size_t k = 0; k < KH; k++)
        memcpy(vc + (k * ctx + c0 + t) * HD, kv + (t * KH + k) * HD, HD * 4);
    // Q (head order kv-major: head = k*G + g)
    project(T, D, xn, D, y->q, QH * HD, q, QH * HD, 0);
    for (size_t t = 0; t < T; t++)
      for (size_t h = 0; h < QH; h++) {
        float* v = q + (t * QH + h) * HD;
        if (y->qn) rmsnorm(HD, v, v, y->qn, o->eps);
        rope_rotate(o, v, c0 + t);
      }
    // attention (source/transformer.c:1375-1422)
#pragma omp parallel
    {
      float* sc = xcalloc((c0 + T) * 4);
#pragma omp for collapse(2) schedule(static)
      for (size_t t = 0; t < T; t++)
        for (size_t h = 0; h < QH; h++) {
          const size_t k = h / G, len = c0 + t + 1;
          const float* qv = q + (t * QH + h) * HD;
          for (size_t s = 0; s < len; s++) {
            float d = 0.0f;
            for (size_t i = 0; i < HD; i++) d += qv[i] * kc[(k * ctx + s) * HD + i];
            sc[s] = d / sqrtf((float)HD);
          }
          float mx = sc[0];
          for (size_t s = 1; s < len; s++) mx = sc[s] > mx ? sc[s] : mx;
          float sum = 0.0f;
          for (size_t s = 0; s < len; s++) {
            sc[s] = expf(sc[s] - mx);
            sum += sc[s];
          }
          for (size_t s = 0; s < len; s++) sc[s] /= sum;
          float* out = att + (t * QH + h) * HD;
          for (size_t i = 0; i < HD; i++) out[i] = 0.0f;
          for (size_t s = 0; s < len; s++)
            for (size_t i = 0; i < HD; i++) out[i] += sc[s] * vc[(k * ctx + s) * HD + i];
        }
      free(sc);
    }
    project(T, QH * HD, att, QH * HD, y->o, D, x, D, 1);
    for (size_t t = 0; t < T; t++) rmsnorm(D, xn + t * D, x + t * D, y->ffn_norm, o->eps);
    if (o->E) {
      moe_ffn(o, y, T, xn, x);
    } else {
      project(T, D, xn, D, y->gate, F, fc, F, 0);
      project(T, D, xn, D, y->up, F, up, F, 0);
      for (size_t i = 0; i < T * F; i++) {
        fc[i] *= (1.0f / (1.0f + expf(-fc[i])));
        fc[i] *= up[i];
      }
      project(T, F, fc, F, y->down, D, x, D, 1);
    }
  }
  if (n) {
    for (size_t t = T - n; t < T; t++) rmsnorm(D, xn + t * D, x + t * D, o->out_norm, o->eps);
    project(n, D, xn + (T - n) * D, D, o->out, o->V, logits, o->V, 0);
  }
  free(x);
  free(xn);
  free(q);
  free(kv);
  free(att);
  free(fc);
  free(up);
  o->cached += T;
}

// Same contract as transformer_predict (source/transformer.c:1607-1727).
void oracle_predict(oracle_t* o, size_t T, const int* tok, size_t n,
                    float* logits) {
  if (!o || !tok || !logits || T == 0 || n == 0) return;
  if (T + o->cached > (size_t)o->ctx) die("context length exhausted");
  if (n > T) n = T;
  const size_t ls = T - n;
  o->min_router_gap = INFINITY;
  for (size_t t = 0; t < T; t += ORACLE_CHUNK) {
    size_t Tc = T - t < ORACLE_CHUNK ? T - t : ORACLE_CHUNK;
    size_t lo = t > ls ? t : ls;
    size_t rows = (t + Tc > lo) ? t + Tc - lo : 0;
    predict_chunk(o, Tc, tok + t, rows, logits + (lo - ls) * (size_t)o->V);
  }
}

void oracle_free(oracle_t* o) {
  if (!o) return;
  free(o->emb);
  if (!o->tied) free(o->out);
  free(o->out_norm);
  for (int l = 0; l < o->L; l++) {
    olayer_t* y = &o->layer[l];
    void* ps[] = {y->attn_norm, y->q, y->k, y->v, y->o, y->qn, y->kn,
                  y->ffn_norm, y->gate, y->up, y->down, y->router, y->gate_c,
                  y->gate_s, y->up_c, y->up_s, y->down_c, y->down_s};
    for (size_t i = 0; i < sizeof(ps) / sizeof(ps[0]); i++) free(ps[i]);
  }
  free(o->layer);
  free(o->kc);
  free(o->vc);
  free(o->rope);
  free(o);
}
