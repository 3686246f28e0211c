// Persistent decode megakernel for dense models (see mega.h).
//
// One CTA per SM (cooperative launch, so all CTAs are co-resident), 8
// warps. A decode step is a fixed sequence of phases; each phase splits its
// work over the CTAs:
//   per layer  QKV     x -> RMSNorm -> Wqkv rows                 -> qkv
//              ATTN    per (kv head, split): q/k RMSNorm + RoPE, K/V append
//                      at `pos`, scores / softmax / P.V -> split record;
//                      the last split of a kv head merges       -> att
//              O       att -> Wo rows, residual add             -> x
//              GU      x -> RMSNorm -> gate/up row pairs, SwiGLU -> h
//              DOWN    h -> Wd rows, residual add               -> x
//   LM head    x -> RMSNorm -> vocab rows (+ per-CTA argmax)     -> am
//   argmax     every CTA reduces the per-CTA partials           -> token
//
// Hand-off without barriers. Every phase output above is a flagged vector:
// element i is one 64-bit word (epoch << 32 | float bits), written with a
// single relaxed store. A consumer loads the words it needs and re-loads
// those whose epoch is not yet the step's, so waiting and fetching the data
// are the same L2 round trip. Each (layer, phase) has its own vector and
// step s of a launch uses epoch `epoch + s`, so a word is rewritten only in
// the next step, after every CTA has published its LM-head partial of this
// step (which it does after all of its reads of the step). Data that is not
// flagged (the K/V cache rows, the attention split records) is written
// before a __threadfence() and read after one.
//
// Weight streaming. Each weight phase gives CTA c a contiguous slice of row
// pairs, so a CTA's weights for the whole launch form a fixed list of
// contiguous byte ranges ("chunks", at most one shared-memory buffer each).
// kRing buffers per CTA: thread 0 issues the cp.async.bulk copy (into its
// own CTA's buffer only) of chunk g+kRing as soon as chunk g has been consumed, with
// completion on the buffer's mbarrier. Weights never depend on activations,
// so copies run ahead across phase and layer boundaries while a CTA waits
// for its inputs. Attention CTAs prefetch their K/V rows into L2 during the
// QKV phase.
//
// Every wait is bounded (2 s): a timeout sets *err, later waits return at
// once, the kernel runs to its end and the host reports the error. All
// issued copies are consumed (waited on) before the kernel ends.
//
// Math per element is the same as the multi-kernel path (kernels.cu) and
// the reference (source/transformer.c:1186-1602).
#include "common.cuh"
#include "kernels.h"
#include "mega.h"

namespace sg {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kPosPerPass = kWarps * 8;  // cache rows per CTA pass
constexpr int kMaxSplits = 64;
constexpr int kTpMaxWorld = 8;
constexpr unsigned long long kTimeoutNs = 2000000000ULL;
constexpr size_t kSmemBudget = 220 * 1024;  // dynamic shared memory per CTA

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Global -> this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, unsigned bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Flagged vectors
// ---------------------------------------------------------------------------
typedef unsigned long long u64;

__device__ __forceinline__ void ll_store(u64* p, float v, unsigned e) {
  const u64 w = ((u64)e << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64 ll_load(const u64* p) {
  u64 w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// System scope: words another GPU writes into this GPU's memory (or this
// GPU writes into a peer's) over NVLink.
__device__ __forceinline__ void ll_store_sys(u64* p, float v, unsigned e) {
  const u64 w = ((u64)e << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64 ll_load_sys(const u64* p) {
  u64 w;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ bool ll_ready(u64 w, unsigned e) { return (unsigned)(w >> 32) == e; }
__device__ __forceinline__ float ll_value(u64 w) { return __uint_as_float((unsigned)w); }

// Bounded spinning: false once the wait has run out (error flag set) or the
// error flag is already set.
struct Spin {
  unsigned long long t0 = 0;
  unsigned n = 0;
};
__device__ __forceinline__ bool spin_on(const MegaArgs& a, Spin& s) {
  if ((++s.n & 15) != 0) return true;
  if (*(volatile int*)a.err) return false;
  const unsigned long long t = now_ns();
  if (s.t0 == 0) s.t0 = t;
  if (t - s.t0 > kTimeoutNs) {
    atomicExch(a.err, 1);
    return false;
  }
  return true;
}

// Loads the flagged words src[k] for the N slots k = k0 + u * kstride
// (slots with k >= K are skipped) and waits until all carry epoch e; the
// values land in v[]. All loads of a round are issued before any is tested.
template <int N, bool SYS = false>
__device__ __forceinline__ void ll_gather(const MegaArgs& a, const u64* src, int k0, int kstride,
                                          int K, unsigned e, float* v) {
  u64 w[N];
#pragma unroll
  for (int u = 0; u < N; u++) {
    const int k = k0 + u * kstride;
    w[u] = (k < K) ? (SYS ? ll_load_sys(src + k) : ll_load(src + k)) : ((u64)e << 32);
  }
  unsigned pending = 0;
#pragma unroll
  for (int u = 0; u < N; u++)
    if (!ll_ready(w[u], e)) pending |= 1u << u;
  Spin sp;
  while (pending) {
    if (!spin_on(a, sp)) break;
#pragma unroll
    for (int u = 0; u < N; u++)
      if (pending & (1u << u))
        w[u] = SYS ? ll_load_sys(src + k0 + u * kstride) : ll_load(src + k0 + u * kstride);
#pragma unroll
    for (int u = 0; u < N; u++)
      if ((pending & (1u << u)) && ll_ready(w[u], e)) pending &= ~(1u << u);
  }
#pragma unroll
  for (int u = 0; u < N; u++) v[u] = ll_value(w[u]);
}

// Trace record per (phase, CTA): [stage start, inputs complete, staged,
// first chunk ready, consumed] (%globaltimer ns), then the phase's total ns
// spent waiting for weight buffers and computing on them (thread 0 writes
// them).
constexpr int kTraceWidth = kMegaTraceWidth;
enum {
  MARK_BEGIN = 0,
  MARK_INPUTS = 1,
  MARK_STAGED = 2,
  MARK_READY = 3,
  MARK_CONSUMED = 4,
  SUM_WAIT = 5,
  SUM_COMPUTE = 6
};

__device__ __forceinline__ void trace_put(const MegaArgs& a, int ph, int slot,
                                          unsigned long long v) {
  if (a.trace && ph < a.trace_phases && threadIdx.x == 0)
    a.trace[((size_t)ph * gridDim.x + blockIdx.x) * kTraceWidth + slot] = v;
}

__device__ __forceinline__ void trace_mark(const MegaArgs& a, int ph, int slot) {
  if (a.trace && ph < a.trace_phases && threadIdx.x == 0)
    a.trace[((size_t)ph * gridDim.x + blockIdx.x) * kTraceWidth + slot] = now_ns();
}

// ---------------------------------------------------------------------------
// Weight phases and the per-CTA chunk schedule
// ---------------------------------------------------------------------------
enum WKind { W_QKV = 0, W_O = 1, W_GU = 2, W_DOWN = 3, W_LM = 4 };

struct Phase {
  const uint16_t* W;
  int K;       // row length (elements)
  int pairs;   // total row pairs of the phase
  int kind;
};

// Per-layer weight pointers, copied to shared memory at kernel start so that
// no global load sits on the phase-to-phase critical path.
constexpr int kMaxLayers = 96;
__shared__ MegaLayer s_layers[kMaxLayers];

// Weight phase `wp` of a step: 4 per layer (QKV, O, GU, DOWN), then LM.
__device__ __forceinline__ Phase weight_phase(const MegaArgs& a, int wp) {
  Phase p;
  if (wp == 4 * a.L) {
    p.W = a.out_w;
    p.K = a.D;
    p.pairs = a.Vl / 2;
    p.kind = W_LM;
    return p;
  }
  const MegaLayer& ly = s_layers[wp >> 2];
  p.kind = wp & 3;
  switch (p.kind) {
    case W_QKV:
      p.W = ly.wqkv;
      p.K = a.D;
      p.pairs = a.QKVl / 2;
      break;
    case W_O:
      p.W = ly.wo;
      p.K = a.QHl * a.HD;
      p.pairs = a.D / 2;
      break;
    case W_GU:
      p.W = ly.wgu;
      p.K = a.D;
      p.pairs = a.Fl;
      break;
    default:
      p.W = ly.wd;
      p.K = a.Fl;
      p.pairs = a.D / 2;
      break;
  }
  return p;
}

// One chunk: row pairs [p0, p1) over columns [k0, k1) (either whole rows,
// several pairs; or one pair and a column segment when a pair does not fit a
// buffer).
struct Chunk {
  int p0, p1, k0, k1;
  bool last_seg;  // the chunk completes its pair(s)
};

struct Slice {
  int pb, pe;     // pairs [pb, pe) of this CTA
  int ppc;        // pairs per chunk (whole rows), 0 when rows are split
  int kseg;       // columns per segment when rows are split
  int spp;        // segments per pair
  int nchunks;
};

__device__ __forceinline__ Slice cta_slice(const Phase& ph, int buf_bytes) {
  Slice s;
  const long long np = ph.pairs;
  s.pb = (int)(np * blockIdx.x / gridDim.x);
  s.pe = (int)(np * (blockIdx.x + 1) / gridDim.x);
  const int n = s.pe - s.pb;
  const int pair_bytes = 4 * ph.K;
  if (pair_bytes <= buf_bytes) {
    s.ppc = buf_bytes / pair_bytes;
    s.kseg = ph.K;
    s.spp = 1;
    s.nchunks = (n + s.ppc - 1) / s.ppc;
  } else {
    s.ppc = 0;
    s.kseg = (buf_bytes / 4) / 256 * 256;
    s.spp = (ph.K + s.kseg - 1) / s.kseg;
    s.nchunks = n * s.spp;
  }
  return s;
}

__device__ __forceinline__ Chunk slice_chunk(const Slice& s, const Phase& ph, int ci) {
  Chunk c;
  if (s.ppc) {
    c.p0 = s.pb + ci * s.ppc;
    c.p1 = min(c.p0 + s.ppc, s.pe);
    c.k0 = 0;
    c.k1 = ph.K;
    c.last_seg = true;
  } else {
    const int pair = s.pb + ci / s.spp, seg = ci % s.spp;
    c.p0 = pair;
    c.p1 = pair + 1;
    c.k0 = seg * s.kseg;
    c.k1 = min(c.k0 + s.kseg, ph.K);
    c.last_seg = (seg == s.spp - 1);
  }
  return c;
}

// Copy-issue cursor (thread 0 only): walks the same chunk sequence as the
// consumers, kRing chunks ahead.
struct Cursor {
  int step, wp, ci;
};

// This CTA's slice of each weight-phase kind (QKV, O, GU, DOWN, LM); every
// layer has the same shapes, so they are computed once per launch.
__shared__ Slice s_slices[5];

__device__ void cursor_skip_empty(const MegaArgs& a, Cursor& c) {
  while (c.step < a.steps) {
    const int kind = (c.wp == 4 * a.L) ? W_LM : (c.wp & 3);
    if (c.ci < s_slices[kind].nchunks) return;
    c.ci = 0;
    if (++c.wp > 4 * a.L) {
      c.wp = 0;
      c.step++;
    }
  }
}

__device__ void cursor_issue(const MegaArgs& a, Cursor& c, char* buf, uint64_t* bar) {
  cursor_skip_empty(a, c);
  if (c.step >= a.steps) return;
  const Phase ph = weight_phase(a, c.wp);
  const Slice& s = s_slices[ph.kind];
  const Chunk ch = slice_chunk(s, ph, c.ci);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (s.ppc) {
    const unsigned bytes = (unsigned)(ch.p1 - ch.p0) * 4u * (unsigned)ph.K;
    mbar_expect_tx(bar, bytes);
    bulk_copy(buf, ph.W + (size_t)2 * ch.p0 * ph.K, bytes, bar);
  } else {
    const unsigned seg = (unsigned)(ch.k1 - ch.k0) * 2u;
    mbar_expect_tx(bar, 2 * seg);
    const uint16_t* r0 = ph.W + (size_t)2 * ch.p0 * ph.K + ch.k0;
    bulk_copy(buf, r0, seg, bar);
    bulk_copy(buf + seg, r0 + ph.K, seg, bar);
  }
  c.ci++;
}

// Bounded wait on a buffer's mbarrier phase.
__device__ void wait_buffer(const MegaArgs& a, uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return;
  const unsigned long long t0 = now_ns();
  unsigned spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 63) == 0) {
      if (*(volatile int*)a.err) return;
      if (now_ns() - t0 > kTimeoutNs) {
        atomicExch(a.err, 2);
        return;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Activation staging
// ---------------------------------------------------------------------------
__device__ __forceinline__ int split_index(int k, int K) {
  return (((k >> 2) & 1) * (K >> 1)) + ((k >> 3) << 2) + (k & 3);
}

// Largest K an RMSNorm staging keeps in registers (K = embedding_dim), read
// in rounds of kNormBatch words per thread.
constexpr int kNormBatch = 8;
constexpr int kNormRegs = 32;

// xs (split layout) = rmsnorm(x) * nw from the flagged vector src (epoch e);
// the raw values also go to xraw[K]. Every thread owns k = tid + u * 256.
__device__ void stage_norm_ll(const MegaArgs& a, const u64* src, unsigned e, const uint16_t* nw,
                              int K, float* xs, float* xraw, float* red, int ph) {
  const int tid = threadIdx.x;
  float v[kNormRegs], g[kNormRegs];
  float ss = 0.f;
  // The gains do not depend on the inputs: their loads go out first.
#pragma unroll
  for (int u = 0; u < kNormRegs; u++) {
    const int k = tid + u * kThreads;
    g[u] = (k < K) ? bf16_to_f32(__ldg(nw + k)) : 0.f;
  }
#pragma unroll
  for (int b = 0; b < kNormRegs; b += kNormBatch) {
    if (b * kThreads < K) {
      ll_gather<kNormBatch>(a, src, tid + b * kThreads, kThreads, K, e, v + b);
    } else {
#pragma unroll
      for (int u = 0; u < kNormBatch; u++) v[b + u] = 0.f;
    }
  }
  trace_mark(a, ph, MARK_INPUTS);
#pragma unroll
  for (int u = 0; u < kNormRegs; u++) {
    const int k = tid + u * kThreads;
    if (k >= K) v[u] = 0.f;
    ss += v[u] * v[u];
  }
  ss = block_sum(ss, red);
  ss /= (float)K;
  const float inv = 1.0f / sqrtf(ss + a.eps);
#pragma unroll
  for (int u = 0; u < kNormRegs; u++) {
    const int k = tid + u * kThreads;
    if (k < K) {
      xs[split_index(k, K)] = (v[u] * inv) * g[u];
      xraw[k] = v[u];
    }
  }
  __syncthreads();
}

// xs (split layout) = the flagged vector src (epoch e), K floats.
__device__ void stage_plain_ll(const MegaArgs& a, const u64* src, unsigned e, int K, float* xs,
                               int ph) {
  const int tid = threadIdx.x;
  constexpr int B = 16;
  for (int base = tid; base < K; base += B * kThreads) {
    float v[B];
    ll_gather<B>(a, src, base, kThreads, K, e, v);
#pragma unroll
    for (int u = 0; u < B; u++) {
      const int k = base + u * kThreads;
      if (k < K) xs[split_index(k, K)] = v[u];
    }
  }
  trace_mark(a, ph, MARK_INPUTS);
  __syncthreads();
}

// Layer-0 input: the embedding row of `token` (xraw) and its RMSNorm (xs).
__device__ void stage_embedding(const MegaArgs& a, int token, const uint16_t* nw, float* xs,
                                float* xraw, float* red) {
  const int tid = threadIdx.x, K = a.D;
  const uint16_t* row = a.emb + (size_t)token * K;
  float v[kNormRegs], g[kNormRegs];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < kNormRegs; u++) {
    const int k = tid + u * kThreads;
    v[u] = (k < K) ? bf16_to_f32(__ldg(row + k)) : 0.f;
    g[u] = (k < K) ? bf16_to_f32(__ldg(nw + k)) : 0.f;
  }
#pragma unroll
  for (int u = 0; u < kNormRegs; u++) ss += v[u] * v[u];
  ss = block_sum(ss, red);
  ss /= (float)K;
  const float inv = 1.0f / sqrtf(ss + a.eps);
#pragma unroll
  for (int u = 0; u < kNormRegs; u++) {
    const int k = tid + u * kThreads;
    if (k < K) {
      xs[split_index(k, K)] = (v[u] * inv) * g[u];
      xraw[k] = v[u];
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Consuming one weight phase
// ---------------------------------------------------------------------------
constexpr int kRing = 4;  // weight buffers per CTA

struct Ring {
  char* base;      // buffer b starts at base + b * buf_bytes
  uint64_t* bar;   // [kRing] in shared memory
  int buf_bytes;
  unsigned g;      // chunks consumed so far
  Cursor cur;      // thread 0: next chunk to issue
};

// Where a phase's outputs go.
struct Out {
  u64* dst;            // flagged vector of the phase (null for the LM head)
  const float* xraw;   // residual input (O, DOWN)
  unsigned e;
  size_t part;         // tensor parallel (O, DOWN): word offset of this rank's
                       // partial rows in every rank's xpart vector
};

__device__ __forceinline__ void pair_epilogue(const MegaArgs& a, const Out& o, int kind, int pair,
                                              float y0, float y1, float& bv, int& bi) {
  const int r0 = 2 * pair;
  switch (kind) {
    case W_QKV:
      ll_store(o.dst + r0, y0, o.e);
      ll_store(o.dst + r0 + 1, y1, o.e);
      break;
    case W_O:
    case W_DOWN:
      if (a.world > 1) {
        // This rank's partial sums go to every rank; the owner of the rows
        // adds them up in rank order (tp_reduce_rows).
        for (int p = 0; p < a.world; p++) {
          ll_store_sys(a.ll_peer[p] + o.part + r0, y0, o.e);
          ll_store_sys(a.ll_peer[p] + o.part + r0 + 1, y1, o.e);
        }
      } else {
        ll_store(o.dst + r0, o.xraw[r0] + y0, o.e);
        ll_store(o.dst + r0 + 1, o.xraw[r0 + 1] + y1, o.e);
      }
      break;
    case W_GU:
      ll_store(o.dst + pair, swiglu(y0, y1), o.e);
      break;
    default:
      if (a.write_logits) {
        a.logits[r0] = y0;
        a.logits[r0 + 1] = y1;
      }
      if (y0 > bv || (y0 == bv && r0 < bi)) {
        bv = y0;
        bi = r0;
      }
      if (y1 > bv || (y1 == bv && r0 + 1 < bi)) {
        bv = y1;
        bi = r0 + 1;
      }
      break;
  }
}

// Consumes every chunk of weight phase `wp` with activations in xs (split
// layout, K floats). For the LM head, (bv, bi) track the warp's argmax.
__device__ void consume_phase(const MegaArgs& a, Ring& r, int wp, const float* xs, const Out& o,
                              float* red, float& bv, int& bi, int ph) {
  trace_mark(a, ph, MARK_STAGED);
  const Phase phs = weight_phase(a, wp);
  const Slice s = s_slices[phs.kind];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = phs.K;
  const float4* lo4 = reinterpret_cast<const float4*>(xs);
  const float4* hi4 = lo4 + (K >> 3);
  float acc0 = 0.f, acc1 = 0.f;  // split rows: running sums (thread 0)
  const bool tr = a.trace != nullptr;
  unsigned long long t_wait = 0, t_comp = 0, t0 = 0;
  for (int ci = 0; ci < s.nchunks; ci++) {
    const int b = r.g % kRing;
    if (tr) t0 = now_ns();
    wait_buffer(a, r.bar + b, (r.g / kRing) & 1);
    if (tr) {
      const unsigned long long t1 = now_ns();
      t_wait += t1 - t0;
      t0 = t1;
    }
    if (ci == 0) trace_mark(a, ph, MARK_READY);
    const Chunk c = slice_chunk(s, phs, ci);
    const uint16_t* wb = reinterpret_cast<const uint16_t*>(r.base + (size_t)b * r.buf_bytes);
    if (s.ppc && c.p1 - c.p0 < kWarps) {
      // Fewer pairs than warps: wpp warps share each pair along K, the
      // partial sums meet in shared memory, lane 0 of warp i finishes pair i.
      const int P = c.p1 - c.p0;
      const int wpp = kWarps / P;
      const int pi = warp / wpp, part = warp % wpp;
      float a0 = 0.f, a1 = 0.f;
      if (pi < P) {
        const uint16_t* w0 = wb + (size_t)pi * 2 * K;
        const uint16_t* w1 = w0 + K;
        float s0[8], s1[8];
#pragma unroll
        for (int i = 0; i < 8; i++) s0[i] = s1[i] = 0.f;
#pragma unroll 4
        for (int k = part * 256 + lane * 8; k < K; k += wpp * 256) {
          const uint4 v0 = *reinterpret_cast<const uint4*>(w0 + k);
          const uint4 v1 = *reinterpret_cast<const uint4*>(w1 + k);
          const float4 xa = lo4[k >> 3], xb = hi4[k >> 3];
          acc8(v0, xa, xb, s0);
          acc8(v1, xa, xb, s1);
        }
        a0 = ((s0[0] + s0[1]) + (s0[2] + s0[3])) + ((s0[4] + s0[5]) + (s0[6] + s0[7]));
        a1 = ((s1[0] + s1[1]) + (s1[2] + s1[3])) + ((s1[4] + s1[5]) + (s1[6] + s1[7]));
        a0 = warp_sum(a0);
        a1 = warp_sum(a1);
      }
      if (lane == 0) {
        red[warp] = a0;
        red[kWarps + warp] = a1;
      }
      __syncthreads();
      if (lane == 0 && warp < P) {
        float y0 = 0.f, y1 = 0.f;
        for (int q = 0; q < wpp; q++) {
          y0 += red[warp * wpp + q];
          y1 += red[kWarps + warp * wpp + q];
        }
        pair_epilogue(a, o, phs.kind, c.p0 + warp, y0, y1, bv, bi);
      }
    } else if (s.ppc) {
      for (int p = c.p0 + warp; p < c.p1; p += kWarps) {
        const uint16_t* w0 = wb + (size_t)(p - c.p0) * 2 * K;
        const uint16_t* w1 = w0 + K;
        // One accumulator per element slot: no FMA dependency chain longer
        // than K / 256.
        float s0[8], s1[8];
#pragma unroll
        for (int i = 0; i < 8; i++) s0[i] = s1[i] = 0.f;
#pragma unroll 4
        for (int k = lane * 8; k < K; k += 256) {
          const uint4 v0 = *reinterpret_cast<const uint4*>(w0 + k);
          const uint4 v1 = *reinterpret_cast<const uint4*>(w1 + k);
          const float4 xa = lo4[k >> 3], xb = hi4[k >> 3];
          acc8(v0, xa, xb, s0);
          acc8(v1, xa, xb, s1);
        }
        float a0 = ((s0[0] + s0[1]) + (s0[2] + s0[3])) + ((s0[4] + s0[5]) + (s0[6] + s0[7]));
        float a1 = ((s1[0] + s1[1]) + (s1[2] + s1[3])) + ((s1[4] + s1[5]) + (s1[6] + s1[7]));
        a0 = warp_sum(a0);
        a1 = warp_sum(a1);
        if (lane == 0) pair_epilogue(a, o, phs.kind, p, a0, a1, bv, bi);
      }
    } else {
      const int seg = c.k1 - c.k0;
      const uint16_t* w0 = wb;
      const uint16_t* w1 = wb + seg;
      float s0[8], s1[8];
#pragma unroll
      for (int i = 0; i < 8; i++) s0[i] = s1[i] = 0.f;
#pragma unroll 4
      for (int k = warp * 256 + lane * 8; k < seg; k += kWarps * 256) {
        const uint4 v0 = *reinterpret_cast<const uint4*>(w0 + k);
        const uint4 v1 = *reinterpret_cast<const uint4*>(w1 + k);
        const int kk = c.k0 + k;
        const float4 xa = lo4[kk >> 3], xb = hi4[kk >> 3];
        acc8(v0, xa, xb, s0);
        acc8(v1, xa, xb, s1);
      }
      float a0 = ((s0[0] + s0[1]) + (s0[2] + s0[3])) + ((s0[4] + s0[5]) + (s0[6] + s0[7]));
      float a1 = ((s1[0] + s1[1]) + (s1[2] + s1[3])) + ((s1[4] + s1[5]) + (s1[6] + s1[7]));
      a0 = warp_sum(a0);
      a1 = warp_sum(a1);
      if (lane == 0) {
        red[warp] = a0;
        red[kWarps + warp] = a1;
      }
      __syncthreads();
      if (tid == 0) {
        for (int w = 0; w < kWarps; w++) {
          acc0 += red[w];
          acc1 += red[kWarps + w];
        }
        if (c.last_seg) {
          pair_epilogue(a, o, phs.kind, c.p0, acc0, acc1, bv, bi);
          acc0 = acc1 = 0.f;
        }
      }
    }
    __syncthreads();  // buffer b fully read
    if (tid == 0) cursor_issue(a, r.cur, r.base + (size_t)b * r.buf_bytes, r.bar + b);
    if (tr) t_comp += now_ns() - t0;
    r.g++;
  }
  trace_mark(a, ph, MARK_CONSUMED);
  trace_put(a, ph, SUM_WAIT, t_wait);
  trace_put(a, ph, SUM_COMPUTE, t_comp);
}

// Tensor parallelism: rows [r0, r1) of the residual (this CTA's rows of the
// o_proj / down phase) = xraw + the sum over ranks, in rank order, of the
// partial rows every rank pushed into this rank's xpart vector at `part0`
// (rank 0's slot; rank p's at part0 + p * D). Same inputs and order on
// every rank, so every rank's residual is bit-identical.
__device__ void tp_reduce_rows(const MegaArgs& a, const float* xraw, size_t part0, u64* dst,
                               int r0, int r1, unsigned e) {
  for (int r = r0 + threadIdx.x; r < r1; r += kThreads) {
    float v[kTpMaxWorld];
    ll_gather<kTpMaxWorld, true>(a, a.ll + part0, r, a.D, a.world * a.D, e, v);
    float s = v[0];
    for (int p = 1; p < a.world; p++) s += v[p];
    ll_store(dst + r, xraw[r] + s, e);
  }
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------
// The per-lane factors head_norm_rope needs for position `pos` (rope table
// entries and norm gains), loaded before the head's values are waited for.
template <int HD>
struct HeadFactors {
  float ca[HD / 32], cb[HD / 32], g[HD / 32];
};

template <int HD>
__device__ __forceinline__ void load_head_factors(const MegaArgs& a, const uint16_t* nw, int pos,
                                                  HeadFactors<HD>& f) {
  constexpr int V = HD / 32;
  const int lane = threadIdx.x & 31;
  const float* cs = a.rope + (size_t)pos * HD;
  const int off = a.pair_offset;
#pragma unroll
  for (int j = 0; j < V; j++) {
    const int i = lane + 32 * j;
    const bool first = (a.pair_stride == 1) ? (i < a.pair_bound) : ((i & 1) == 0);
    const int base = first ? i : i - off;
    f.ca[j] = __ldg(cs + base);
    f.cb[j] = __ldg(cs + base + off);
    f.g[j] = nw ? bf16_to_f32(__ldg(nw + i)) : 1.f;
  }
}

// One warp: out[i] = RoPE(RMSNorm(v) * nw) for a head of HD values held as
// V per lane (i = lane + 32 j) (source/transformer.c:1293-1323); without a
// norm (has_norm false) the values are rotated as they are. `scratch` holds
// HD floats private to the warp.
template <int HD>
__device__ void head_norm_rope(const MegaArgs& a, float* v, bool has_norm,
                               const HeadFactors<HD>& f, float* scratch, float* out) {
  constexpr int V = HD / 32;
  const int lane = threadIdx.x & 31;
  if (has_norm) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < V; j++) ss += v[j] * v[j];
    ss = warp_sum(ss);
    ss /= (float)HD;
    const float inv = 1.0f / sqrtf(ss + a.eps);
#pragma unroll
    for (int j = 0; j < V; j++) v[j] = (v[j] * inv) * f.g[j];
  }
#pragma unroll
  for (int j = 0; j < V; j++) scratch[lane + 32 * j] = v[j];
  __syncwarp();
  const int off = a.pair_offset;
#pragma unroll
  for (int j = 0; j < V; j++) {
    const int i = lane + 32 * j;
    const bool first = (a.pair_stride == 1) ? (i < a.pair_bound) : ((i & 1) == 0);
    float o;
    if (first) {
      o = scratch[i] * f.ca[j] - scratch[i + off] * f.cb[j];
    } else {
      const int hh = i - off;
      o = scratch[hh] * f.cb[j] + scratch[i] * f.ca[j];
    }
    out[i] = o;
  }
  __syncwarp();
}

// L2 prefetch of the cache rows [s_begin, min(s_end, pos)) of this CTA's
// attention items (rows below `pos` are final).
template <int HD>
__device__ void prefetch_kv(const MegaArgs& a, int l, int pos) {
  if (threadIdx.x != 0) return;
  const int items = a.KHl * a.nsplit;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int kh = it % a.KHl, sp = it / a.KHl;
    const int s0 = sp * a.split_len;
    const int s1 = min(s0 + a.split_len, pos);
    if (s1 <= s0) continue;
    const size_t off = ((size_t)l * a.KHl + kh) * a.ctx * HD + (size_t)s0 * HD;
    const uint32_t bytes = (uint32_t)(s1 - s0) * HD * 4;
    prefetch_l2(a.kc + off, bytes);
    prefetch_l2(a.vc + off, bytes);
  }
}

// L2 prefetch of the small per-layer vectors of layer `l` (norm gains), or
// of the final norm when l == L: they are evicted between decode steps by
// the weight stream, and every CTA reads them on a phase's critical path.
__device__ void prefetch_gains(const MegaArgs& a, int l) {
  if (threadIdx.x != 32) return;
  if (l >= a.L) {
    prefetch_l2(a.out_norm, (uint32_t)a.D * 2);
    return;
  }
  const MegaLayer& ly = s_layers[l];
  prefetch_l2(ly.attn_norm, (uint32_t)a.D * 2);
  prefetch_l2(ly.ffn_norm, (uint32_t)a.D * 2);
  if (ly.q_norm) prefetch_l2(ly.q_norm, (uint32_t)a.HD * 2);
  if (ly.k_norm) prefetch_l2(ly.k_norm, (uint32_t)a.HD * 2);
}

template <int HD, int G>
constexpr int attn_floats() {
  // qs [G][HD], wm/wl [kWarps][G], wacc [kWarps][G][HD], merge weights
  // [G][kMaxSplits], denominators [G], last-CTA flag.
  return G * HD + 2 * kWarps * G + kWarps * G * HD + G * kMaxSplits + G + 4;
}

// One attention item: kv head kh, cache split sp, at position pos. Its q,
// k and v come from the flagged qkv vector of layer l (epoch e). The split
// holding `pos` appends this step's k and v to the cache. The split record
// [m, l, -, -, acc[HD]] of each of the G query heads goes to attn_partial;
// the last split of the kv head to finish (ticket) merges the records and
// publishes the heads' attention output in the flagged att vector.
template <int HD, int G>
__device__ void attn_item(const MegaArgs& a, const MegaLayer& ly, int l, int kh, int sp,
                          int pos, unsigned e, float* sm, int ph) {
  constexpr int V = HD / 32;
  constexpr int QF = HD / 16;
  float* qs = sm;                      // [G][HD]
  float* wm = qs + G * HD;             // [kWarps][G]
  float* wl = wm + kWarps * G;         // [kWarps][G]
  float* wacc = wl + kWarps * G;       // [kWarps][G][HD]
  float* cw = wacc + kWarps * G * HD;  // [G][kMaxSplits]
  float* Ls = cw + G * kMaxSplits;     // [G]
  int* is_last = reinterpret_cast<int*>(Ls + G);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t layer_off = (size_t)l * a.KHl * a.ctx * HD;
  float* kb = a.kc + layer_off + (size_t)kh * a.ctx * HD;
  float* vb = a.vc + layer_off + (size_t)kh * a.ctx * HD;
  const int s_begin = sp * a.split_len;
  const int s_end = min(s_begin + a.split_len, pos + 1);
  const u64* qkv = a.ll + a.llo.qkv + (size_t)l * a.QKVl;

  // The cache rows below `pos` were written in earlier steps (made visible
  // by the fence at the top of the step).
  if (warp < G) {
    HeadFactors<HD> f;
    load_head_factors<HD>(a, ly.q_norm, pos, f);
    float v[V];
    ll_gather<V>(a, qkv + (size_t)(kh * G + warp) * HD, lane, 32, HD, e, v);
    head_norm_rope<HD>(a, v, ly.q_norm != nullptr, f, wacc + (size_t)warp * HD, qs + warp * HD);
  }
  if (warp == kWarps - 1 && pos >= s_begin && pos < s_begin + a.split_len) {
    HeadFactors<HD> f;
    load_head_factors<HD>(a, ly.k_norm, pos, f);
    float v[V], vv[V];
    ll_gather<V>(a, qkv + (size_t)(a.QHl + kh) * HD, lane, 32, HD, e, v);
    ll_gather<V>(a, qkv + (size_t)(a.QHl + a.KHl + kh) * HD, lane, 32, HD, e, vv);
    head_norm_rope<HD>(a, v, ly.k_norm != nullptr, f, wacc + (size_t)warp * HD,
                       kb + (size_t)pos * HD);
#pragma unroll
    for (int j = 0; j < V; j++) vb[(size_t)pos * HD + lane + 32 * j] = vv[j];
  }
  __syncthreads();
  trace_mark(a, ph, MARK_INPUTS);

  float m[G], lsum[G], acc[G][V];
#pragma unroll
  for (int g = 0; g < G; g++) {
    m[g] = -INFINITY;
    lsum[g] = 0.f;
#pragma unroll
    for (int v = 0; v < V; v++) acc[g][v] = 0.f;
  }
  const int j = lane >> 2, qd = lane & 3;
  const float div = sqrtf((float)HD);
  for (int base = s_begin + warp * 8; base < s_end; base += kPosPerPass) {
    const int s = base + j;
    const bool valid = s < s_end;
    float d[G];
#pragma unroll
    for (int g = 0; g < G; g++) d[g] = 0.f;
    float4 kv[QF];
    if (valid) {
      const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)s * HD);
#pragma unroll
      for (int i = 0; i < QF; i++) kv[i] = __ldcg(kr + qd + 4 * i);
    }
    float vv[8][V];
#pragma unroll
    for (int jj = 0; jj < 8; jj++) {
      const int sj = base + jj;
#pragma unroll
      for (int v = 0; v < V; v++)
        vv[jj][v] = (sj < s_end) ? __ldcg(vb + (size_t)sj * HD + lane * V + v) : 0.f;
    }
    if (valid) {
#pragma unroll
      for (int i = 0; i < QF; i++) {
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float4 q4 = *reinterpret_cast<const float4*>(&qs[g * HD + (qd + 4 * i) * 4]);
          d[g] = fmaf(q4.x, kv[i].x, d[g]);
          d[g] = fmaf(q4.y, kv[i].y, d[g]);
          d[g] = fmaf(q4.z, kv[i].z, d[g]);
          d[g] = fmaf(q4.w, kv[i].w, d[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
      float dd = d[g];
      dd += __shfl_xor_sync(0xFFFFFFFFu, dd, 1);
      dd += __shfl_xor_sync(0xFFFFFFFFu, dd, 2);
      const float sc = valid ? dd / div : -INFINITY;
      float mx = sc;
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
      const float mn = fmaxf(m[g], mx);
      const float corr = expf(m[g] - mn);
      const float p = valid ? expf(sc - mn) : 0.f;
      float ps = (qd == 0) ? p : 0.f;
      ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 4);
      ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 8);
      ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 16);
      lsum[g] = lsum[g] * corr + ps;
#pragma unroll
      for (int v = 0; v < V; v++) acc[g][v] *= corr;
#pragma unroll
      for (int jj = 0; jj < 8; jj++) {
        const float pj = __shfl_sync(0xFFFFFFFFu, p, jj * 4);
#pragma unroll
        for (int v = 0; v < V; v++) acc[g][v] = fmaf(pj, vv[jj][v], acc[g][v]);
      }
      m[g] = mn;
    }
  }
  __syncthreads();  // the q/k warps' scratch use of wacc is over
#pragma unroll
  for (int g = 0; g < G; g++) {
    if (lane == 0) {
      wm[warp * G + g] = m[g];
      wl[warp * G + g] = lsum[g];
    }
#pragma unroll
    for (int v = 0; v < V; v++) wacc[((size_t)warp * G + g) * HD + lane * V + v] = acc[g][v];
  }
  __syncthreads();
  const int nsplit = a.nsplit;
  float* part = a.attn_partial + (size_t)l * a.QHl * nsplit * (HD + 4);
  for (int ei = tid; ei < G * HD; ei += kThreads) {
    const int g = ei / HD, dd = ei % HD;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; w++) M = fmaxf(M, wm[w * G + g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < kWarps; w++) {
        const float mw = wm[w * G + g];
        if (mw == -INFINITY) continue;
        const float c = expf(mw - M);
        L += wl[w * G + g] * c;
        A += wacc[((size_t)w * G + g) * HD + dd] * c;
      }
    }
    // Split record: [m, l, -, -, acc[HD]] (16-byte aligned acc).
    float* P = part + ((size_t)(kh * G + g) * nsplit + sp) * (HD + 4);
    if (dd == 0) {
      P[0] = M;
      P[1] = L;
    }
    P[4 + dd] = A;
  }
  __threadfence();
  __syncthreads();
  trace_mark(a, ph, MARK_STAGED);
  if (tid == 0) {
    int* ticket = a.attn_ticket + (size_t)l * a.KHl + kh;
    *is_last = (atomicAdd(ticket, 1) == nsplit - 1);
    if (*is_last) *ticket = 0;  // its next use is in a later step
  }
  __syncthreads();
  if (!*is_last) return;
  __threadfence();
  // Merge: att = sum_j c_j acc_j / sum_j c_j l_j, c_j = exp(m_j - max m);
  // splits without positions have m = -inf.
  for (int g = warp; g < G; g += kWarps) {
    const float* P0 = part + (size_t)(kh * G + g) * nsplit * (HD + 4);
    float mloc = -INFINITY;
    for (int jx = lane; jx < nsplit; jx += 32)
      mloc = fmaxf(mloc, __ldcg(P0 + (size_t)jx * (HD + 4)));
    const float M = warp_max(mloc);
    float ls = 0.f;
    for (int jx = lane; jx < nsplit; jx += 32) {
      const float mj = __ldcg(P0 + (size_t)jx * (HD + 4));
      const float c = (mj == -INFINITY) ? 0.f : expf(mj - M);
      cw[g * kMaxSplits + jx] = c;
      ls += c * __ldcg(P0 + (size_t)jx * (HD + 4) + 1);
    }
    ls = warp_sum(ls);
    if (lane == 0) Ls[g] = ls;
  }
  __syncthreads();
  u64* att = a.ll + a.llo.att + (size_t)l * a.QHl * HD;
  for (int ei = tid; ei < G * HD; ei += kThreads) {
    const int g = ei / HD, dd = ei % HD;
    const float* P0 = part + (size_t)(kh * G + g) * nsplit * (HD + 4) + 4 + dd;
    float A = 0.f;
    for (int j0 = 0; j0 < nsplit; j0 += 8) {
      float pv[8];  // the loads of a batch go out together
#pragma unroll
      for (int u = 0; u < 8; u++)
        pv[u] = (j0 + u < nsplit) ? __ldcg(P0 + (size_t)(j0 + u) * (HD + 4)) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (j0 + u < nsplit) A = fmaf(cw[g * kMaxSplits + j0 + u], pv[u], A);
    }
    ll_store(att + (size_t)(kh * G + g) * HD + dd, A / Ls[g], e);
  }
  __syncthreads();
  trace_mark(a, ph, MARK_READY);
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int HD, int G>
__global__ void __launch_bounds__(kThreads, 1)
    k_mega_decode(const __grid_constant__ MegaArgs a, int buf_bytes) {
  extern __shared__ __align__(128) char dyn[];
  __shared__ float red[32];
  __shared__ float cbest_v[kWarps];
  __shared__ int cbest_i[kWarps];
  __shared__ __align__(8) uint64_t ring_bar[kRing];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  Ring r;
  r.base = dyn;
  r.bar = ring_bar;
  r.buf_bytes = buf_bytes;
  r.g = 0;
  r.cur = {0, 0, 0};
  float* xraw = reinterpret_cast<float*>(dyn + (size_t)kRing * buf_bytes);  // [D]
  float* xs = xraw + ((a.D + 31) / 32) * 32;  // matvec input / attention scratch
  for (int i = threadIdx.x; i < a.L; i += kThreads) s_layers[i] = a.layers[i];
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRing; i++) mbar_init(&ring_bar[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x < 5) {
    // Layer 0's phases stand for every layer (same shapes).
    const int wp = (threadIdx.x == W_LM) ? 4 * a.L : threadIdx.x;
    s_slices[threadIdx.x] = cta_slice(weight_phase(a, wp), buf_bytes);
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < kRing; i++) cursor_issue(a, r.cur, dyn + (size_t)i * buf_bytes, &ring_bar[i]);
  int ph = 0;  // phase counter (trace only)
  int pos = __ldcg(a.pos);
  int token = __ldcg(a.tok);
  int step = __ldcg(a.step);
  const int QD = a.QHl * a.HD;
  const int attn_items = a.KHl * a.nsplit;
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  u64* am = a.ll + a.llo.am;
  const int nam = a.world * (int)gridDim.x;  // argmax partials of all ranks

  for (int s = 0; s < a.steps; s++) {
    const unsigned e = a.epoch + (unsigned)s;
    for (int l = 0; l < a.L; l++) {
      const MegaLayer& ly = s_layers[l];
      u64* x_o = a.ll + a.llo.x + (size_t)l * 2 * a.D;  // after o_proj
      u64* x_d = x_o + a.D;                              // after down
      // QKV
      trace_mark(a, ph, MARK_BEGIN);
      prefetch_kv<HD>(a, l, pos);
      prefetch_gains(a, l + 1);
      if (l == 0)
        stage_embedding(a, token, ly.attn_norm, xs, xraw, red);
      else
        stage_norm_ll(a, x_o - 2 * (size_t)a.D + a.D, e, ly.attn_norm, a.D, xs, xraw, red, ph);
      consume_phase(a, r, 4 * l + W_QKV, xs,
                    Out{a.ll + a.llo.qkv + (size_t)l * a.QKVl, nullptr, e}, red, bv, bi, ph);
      ph++;
      // ATTN
      trace_mark(a, ph, MARK_BEGIN);
      for (int it = blockIdx.x; it < attn_items; it += gridDim.x)
        attn_item<HD, G>(a, ly, l, it % a.KHl, it / a.KHl, pos, e, xs, ph);
      ph++;
      // O + residual
      trace_mark(a, ph, MARK_BEGIN);
      stage_plain_ll(a, a.ll + a.llo.att + (size_t)l * QD, e, QD, xs, ph);
      {
        const size_t part0 = a.llo.xpart + (size_t)(l * 2 + 0) * a.world * a.D;
        consume_phase(a, r, 4 * l + W_O, xs, Out{x_o, xraw, e, part0 + (size_t)a.rank * a.D},
                      red, bv, bi, ph);
        if (a.world > 1)
          tp_reduce_rows(a, xraw, part0, x_o, 2 * s_slices[W_O].pb, 2 * s_slices[W_O].pe, e);
      }
      ph++;
      // gate/up + SwiGLU
      trace_mark(a, ph, MARK_BEGIN);
      stage_norm_ll(a, x_o, e, ly.ffn_norm, a.D, xs, xraw, red, ph);
      consume_phase(a, r, 4 * l + W_GU, xs, Out{a.ll + a.llo.h + (size_t)l * a.Fl, nullptr, e},
                    red, bv, bi, ph);
      ph++;
      // down + residual
      trace_mark(a, ph, MARK_BEGIN);
      stage_plain_ll(a, a.ll + a.llo.h + (size_t)l * a.Fl, e, a.Fl, xs, ph);
      {
        const size_t part0 = a.llo.xpart + (size_t)(l * 2 + 1) * a.world * a.D;
        consume_phase(a, r, 4 * l + W_DOWN, xs, Out{x_d, xraw, e, part0 + (size_t)a.rank * a.D},
                      red, bv, bi, ph);
        if (a.world > 1)
          tp_reduce_rows(a, xraw, part0, x_d, 2 * s_slices[W_DOWN].pb, 2 * s_slices[W_DOWN].pe,
                         e);
      }
      ph++;
    }
    // LM head with per-CTA argmax
    trace_mark(a, ph, MARK_BEGIN);
    prefetch_gains(a, 0);  // next step's layer 0
    stage_norm_ll(a, a.ll + a.llo.x + (size_t)(a.L - 1) * 2 * a.D + a.D, e, a.out_norm, a.D, xs,
                  xraw, red, ph);
    bv = -INFINITY;
    bi = 0x7FFFFFFF;
    consume_phase(a, r, 4 * a.L, xs, Out{nullptr, nullptr, e}, red, bv, bi, ph);
    if (lane == 0) {
      cbest_v[warp] = bv;
      cbest_i[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = cbest_v[0];
      int i = cbest_i[0];
      for (int w = 1; w < kWarps; w++) {
        if (cbest_v[w] > v || (cbest_v[w] == v && cbest_i[w] < i)) {
          v = cbest_v[w];
          i = cbest_i[w];
        }
      }
      // Global vocabulary index: this rank's rows start at rank * Vl.
      const int gi = (i == 0x7FFFFFFF) ? i : a.rank * a.Vl + i;
      const int slot = a.rank * gridDim.x + blockIdx.x;
      if (a.world > 1) {
        for (int p = 0; p < a.world; p++) {
          ll_store_sys(a.ll_peer[p] + a.llo.am + slot, v, e);
          ll_store_sys(a.ll_peer[p] + a.llo.am + nam + slot, __int_as_float(gi), e);
        }
      } else {
        ll_store(am + slot, v, e);
        ll_store(am + nam + slot, __int_as_float(gi), e);
      }
    }
    ph++;
    // Every CTA reduces the published partials (of every rank) itself.
    if (warp == 0) {
      float v = -INFINITY;
      int i = 0x7FFFFFFF;
      for (int b0 = 0; b0 < nam; b0 += 32 * 4) {
        float vb[4], ib[4];
        ll_gather<4, true>(a, am, b0 + lane, 32, nam, e, vb);
        ll_gather<4, true>(a, am + nam, b0 + lane, 32, nam, e, ib);
#pragma unroll
        for (int u = 0; u < 4; u++) {
          if (b0 + lane + 32 * u >= nam) continue;
          const int ii = __float_as_int(ib[u]);
          if (vb[u] > v || (vb[u] == v && ii < i)) {
            v = vb[u];
            i = ii;
          }
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        const int i2 = __shfl_xor_sync(0xFFFFFFFFu, i, o);
        if (v2 > v || (v2 == v && i2 < i)) {
          v = v2;
          i = i2;
        }
      }
      if (lane == 0) cbest_i[0] = (i == 0x7FFFFFFF) ? 0 : i;
    }
    __syncthreads();
    token = cbest_i[0];
    // Every CTA has published its partial after writing this step's K/V
    // rows (and a fence): the next step's attention reads them after this
    // one.
    __threadfence();
    if (blockIdx.x == 0 && threadIdx.x == 0 && step >= 0 && step < a.gen_len)
      a.gen[step] = token;
    step++;
    pos++;
    __syncthreads();
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *a.tok = token;
    *a.pos = pos;
    *a.step = step;
  }
}

template <int HD, int G>
void* kernel_ptr() {
  return (void*)k_mega_decode<HD, G>;
}

void* select(int HD, int G) {
#define SG_SEL(h, g) \
  if (HD == h && G == g) return kernel_ptr<h, g>();
  SG_SEL(32, 1) SG_SEL(32, 2) SG_SEL(32, 4) SG_SEL(32, 8)
  SG_SEL(64, 1) SG_SEL(64, 2) SG_SEL(64, 4) SG_SEL(64, 8)
  SG_SEL(128, 1) SG_SEL(128, 2) SG_SEL(128, 4) SG_SEL(128, 8)
#undef SG_SEL
  return nullptr;
}

size_t select_attn_floats(int HD, int G) {
#define SG_SEL(h, g) \
  if (HD == h && G == g) return (size_t)attn_floats<h, g>();
  SG_SEL(32, 1) SG_SEL(32, 2) SG_SEL(32, 4) SG_SEL(32, 8)
  SG_SEL(64, 1) SG_SEL(64, 2) SG_SEL(64, 4) SG_SEL(64, 8)
  SG_SEL(128, 1) SG_SEL(128, 2) SG_SEL(128, 4) SG_SEL(128, 8)
#undef SG_SEL
  return 0;
}

// Activation region, rounded to 128 bytes: the residual copy xraw [D]
// (rounded to 32 floats), then the matvec input or the attention scratch.
size_t act_bytes(int D, int QD, int Fl, int HD, int G) {
  size_t k = (size_t)std::max(D, std::max(QD, Fl));
  k = std::max(k, select_attn_floats(HD, G));
  k += (size_t)(D + 31) / 32 * 32;
  return (k * sizeof(float) + 127) / 128 * 128;
}

}  // namespace

MegaFlagged mega_flagged_layout(int D, int QKVl, int QD, int Fl, int L, int grid, int world) {
  MegaFlagged f;
  f.x = 0;
  f.qkv = f.x + (size_t)L * 2 * D;
  f.att = f.qkv + (size_t)L * QKVl;
  f.h = f.att + (size_t)L * QD;
  f.xpart = f.h + (size_t)L * Fl;
  f.am = f.xpart + (world > 1 ? (size_t)L * 2 * world * D : 0);
  f.total = f.am + 2 * (size_t)world * grid;
  return f;
}

// Ring buffers take what the activations leave of the budget.
size_t mega_smem_bytes(int D, int QD, int Fl, int HD, int G) {
  if (D > kNormRegs * kThreads) return 0;
  const size_t act = act_bytes(D, QD, Fl, HD, G);
  if (act + (size_t)kRing * 8 * 1024 > kSmemBudget) return 0;
  size_t buf = (kSmemBudget - act) / kRing / 1024 * 1024;
  return (size_t)kRing * buf + act;
}

static int buffer_bytes(size_t smem, int D, int QD, int Fl, int HD, int G) {
  return (int)((smem - act_bytes(D, QD, Fl, HD, G)) / kRing);
}

void mega_configure(size_t smem) {
  for (int hd : {32, 64, 128})
    for (int g : {1, 2, 4, 8})
      SG_CUDA(cudaFuncSetAttribute(select(hd, g), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)std::max(smem, (size_t)48 * 1024)));
}

int mega_grid(size_t smem, int HD, int G) {
  void* k = select(HD, G);
  if (!k || smem == 0) return 0;
  int per_sm = 0;
  SG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem));
  if (per_sm < 1) return 0;
  int dev, sms;
  SG_CUDA(cudaGetDevice(&dev));
  SG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return sms;
}

void mega_split(int ctx, int KHl, int grid, int* nsplit, int* split_len) {
  int target = (grid + KHl - 1) / KHl;
  if (target > kMaxSplits) target = kMaxSplits;
  if (target < 1) target = 1;
  int len = (ctx + target - 1) / target;
  len = (len + kPosPerPass - 1) / kPosPerPass * kPosPerPass;
  *split_len = len;
  *nsplit = (ctx + len - 1) / len;
}

void mega_decode(const MegaArgs& a, int grid, size_t smem, cudaStream_t s) {
  void* k = select(a.HD, a.G);
  if (!k) SG_DIE("megakernel: unsupported head_dim / group");
  if (a.nsplit > kMaxSplits) SG_DIE("megakernel: too many attention splits");
  if (a.L > kMaxLayers) SG_DIE("megakernel: too many layers");
  int buf = buffer_bytes(smem, a.D, a.QHl * a.HD, a.Fl, a.HD, a.G);
  if (buf < 8 * 1024 || buf % 16) SG_DIE("megakernel: weight buffers too small");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {(void*)&a, (void*)&buf};
  SG_CUDA(cudaLaunchKernelExC(&cfg, k, args));
}

}  // namespace sg
