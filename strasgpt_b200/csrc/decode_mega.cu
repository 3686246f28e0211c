// Persistent decode megakernel (see mega.h), for dense models and, as a
// compile-time variant (MOE), for mixtures of MXFP4 experts.
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
//   (MOE: GU, DOWN are ROUTER  x -> RMSNorm -> router rows   -> logits,
//              every CTA picks the top-k experts from the logits;
//              EGU     gate/up rows of the chosen experts, SwiGLU -> h[k]
//              EDOWN   down rows of the chosen experts, weighted in
//                      choice order, residual add               -> x)
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
// chunks (up to 64 rows by a column range, one shared-memory buffer each).
// A ninth warp is the producer: it walks that list and, for each of the
// ring buffers, waits until the consumers have released the buffer (empty
// mbarrier), then copies the chunk's rows into it with one cp.async.bulk per
// row (into its own CTA's buffer only; MXFP4 expert chunks: a few copies
// of contiguous runs), completion counted on the buffer's full mbarrier.
// The weight copies are marked evict-first in L2, so that the stream does
// not push out the kernel's instructions, flagged vectors and K/V rows. Rows sit kPad bytes further apart than in memory, so the
// eight rows of a tensor-core fragment fall into different banks. Weights
// never depend on activations, so copies run ahead across phase and layer
// boundaries while the consumers wait for their inputs. Attention CTAs
// prefetch their K/V rows into L2 during the QKV phase.
//
// Dot products on the tensor cores. The activation x is staged in shared
// memory as bf16 parts x = hi + mid + lo (each the bf16 rounding of what
// the previous parts leave), which reproduces fp32 x to about 2^-24. One
// mma.sync m16n8k16 multiplies A = sixteen weight rows (ldmatrix from the
// padded buffer) by B = the parts (columns 0..2 of 8) over 16 columns; the
// fp32 accumulator columns are summed at the end. Each of the eight
// consumer warps takes every eighth 32-column block of the chunk for all of
// its rows, and the warps' partial sums meet in shared memory. MXFP4 rows
// go through the same fragments: e2m1 codes converted to f16 in registers,
// the activation as two f16 parts with a scale per 32-column block
// (mx_chunk_dot).
//
// Every wait is bounded (MegaArgs::wait_ns, 2 s by default): a timeout sets
// *err, later waits return at once, the kernel runs to its end and the host
// reports the error. The producer waits (bounded) for the completion of its
// last copies before it exits.
//
// Math per element is the same as the multi-kernel path (kernels.cu) and
// the reference (source/transformer.c:1186-1602).
#include "common.cuh"
#include "kernels.h"
#include "mega.h"

namespace sg {
namespace {

#ifndef SG_MEGA_WARPS
#define SG_MEGA_WARPS 8
#endif
constexpr int kWarps = SG_MEGA_WARPS;       // consumer warps
constexpr int kThreads = 32 * kWarps;       // consumer threads
constexpr int kBlockThreads = kThreads + 32;  // + the producer warp
constexpr int kPosPerPass = kWarps * 8;  // cache rows per CTA pass
constexpr int kMaxChunkRows = 64;        // rows per MXFP4 weight chunk (4 fragments)
constexpr int kMaxDenseRows = 48;        // rows per bf16 weight chunk (3 fragments)
constexpr int kPad = 16;                 // extra bytes per row in a buffer
constexpr int kMaxRing = 4;              // weight buffers per CTA (at most)
constexpr int kMaxSplits = 64;
constexpr int kTpMaxWorld = 8;

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

// The same for weight rows, which are read once per step: marked
// evict-first in L2, so that the weight stream (GBs per step) does not push
// out what the kernel reuses (its own instructions, the flagged vectors,
// the K/V rows).
__device__ __forceinline__ void bulk_copy_stream(void* dst, const void* src, unsigned bytes,
                                                 uint64_t* bar) {
  asm volatile(
      "{\n"
      " .reg .b64 pol;\n"
      " createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n"
      " cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], pol;\n"
      "}" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Barrier of the consumer warps only (the producer warp never joins it).
__device__ __forceinline__ void csync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
}

// Four 8x8 bf16 matrices; lane i gives the address of row i % 8 of matrix
// i / 8 and receives, from each matrix, the pair (row i / 4, cols 2 (i % 4)).
// For matrices (rows 0-7, cols 0-7), (rows 8-15, cols 0-7), (rows 0-7,
// cols 8-15), (rows 8-15, cols 8-15) of a 16x16 tile these are the A
// fragments of m16n8k16. The registers come back by value: an array whose
// address is taken can end up in local memory, which with the shared-memory
// carveout at its maximum is served by L2.
__device__ __forceinline__ uint4 ldsm4(uint32_t addr) {
  uint4 r;
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(addr));
  return r;
}

// d += A (16x16 bf16, row-major fragments a.x..a.w) * B (16x8 bf16, b0/b1),
// fp32 accumulators (rows g, g + 8; columns 2c, 2c + 1 of lane 4g + c).
// (Register operands only, so not volatile: the compiler may interleave
// the steps of independent fragments.)
__device__ __forceinline__ void mma4(float4& d, uint4 a, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d.x), "+f"(d.y), "+f"(d.z), "+f"(d.w)
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
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
  if (t - s.t0 > a.wait_ns) {
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
// spent waiting for weight buffers, on its chunks (wait excluded), on warp
// 0's dot products, and on the cross-warp sums and epilogues (thread 0
// writes them).
constexpr int kTraceWidth = kMegaTraceWidth;
enum {
  MARK_BEGIN = 0,
  MARK_INPUTS = 1,
  MARK_STAGED = 2,
  MARK_READY = 3,
  MARK_CONSUMED = 4,
  SUM_WAIT = 5,
  SUM_COMPUTE = 6,
  SUM_DOT = 7,
  SUM_REDUCE = 8,
  MARK_NORMED = 9,
  MARK_SCALED = 10,
  MARK_SYNCED = 11,
  MARK_GAINS = 12
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
enum WKind {
  W_QKV = 0,
  W_O = 1,
  W_GU = 2,
  W_DOWN = 3,
  W_LM = 4,
  W_ROUTER = 5,  // MoE: router rows (bf16)
  W_EGU = 6,     // MoE: gate/up rows of the selected experts (MXFP4)
  W_EDOWN = 7    // MoE: down rows of the selected experts (MXFP4)
};
constexpr int kKinds = 8;
constexpr int kMaxTopk = 8;

struct Phase {
  const uint16_t* W;  // bf16 rows (null for the MXFP4 expert phases)
  int K;       // row length (elements)
  int pairs;   // total row pairs of the phase
  int kind;
};

// Per-layer weight pointers, copied to shared memory at kernel start so that
// no global load sits on the phase-to-phase critical path.
constexpr int kMaxLayers = 96;
// It sits at the end of the dynamic region (a.layers_off), sized by the
// model's layer count.
extern __shared__ __align__(128) char s_dyn[];
__device__ __forceinline__ MegaLayer* layer_table(const MegaArgs& a) {
  return reinterpret_cast<MegaLayer*>(s_dyn + a.layers_off);
}

// Weight phases per layer: dense QKV, O, GU, DOWN; mixture of experts QKV,
// O, ROUTER, EGU, EDOWN. The LM head follows the last layer. MOE (a.moe) is
// a template parameter of the kernel, so that the dense kernel carries no
// expert code.
template <bool MOE>
__device__ __forceinline__ int phases_per_layer(const MegaArgs&) { return MOE ? 5 : 4; }

template <bool MOE>
__device__ __forceinline__ int phase_kind(const MegaArgs& a, int wp) {
  const int P = phases_per_layer<MOE>(a);
  if (wp == P * a.L) return W_LM;
  const int i = wp % P;
  if (!MOE || i < 2) return i;
  return i == 2 ? W_ROUTER : (i == 3 ? W_EGU : W_EDOWN);
}

// MXFP4 rows in a buffer: the codes (K / 2 bytes) then the scales (K / 32
// bytes, rounded up to 16).
__device__ __host__ __forceinline__ int mx_scale_bytes(int K) { return (K / 32 + 15) / 16 * 16; }
__device__ __host__ __forceinline__ int mx_row_bytes(int K) { return K / 2 + mx_scale_bytes(K); }

// MXFP4 expert inputs in shared memory ("xm"): per vector of K values two
// f16 arrays hi, mid with x * 2^s = hi + mid (hi the f16 rounding of
// x * 2^s, mid that of what it leaves), s a power-of-two exponent per
// 32-column block that puts the block's largest magnitude in [2^14, 2^15).
// Array p of vector j starts at byte (2 j + p) * mx_x_vbytes(K) (64 mod 128,
// so that the two arrays' 64-byte pieces of a block share no bank); after
// all arrays, the inverse block scales 2^-s, floats [vectors][K / 32].
__device__ __host__ __forceinline__ int mx_x_vbytes(int K) { return (2 * K + 127) / 128 * 128 + 64; }
__device__ __host__ __forceinline__ int mx_x_bytes(int nvec, int K) {
  return nvec * (2 * mx_x_vbytes(K) + K / 32 * 4);
}
// Floats of the xm region of a mixture of experts (none for a dense model):
// the normalised x [D] (gate/up input), later the selected experts' SwiGLU
// outputs [topk][Fe] (down input).
__device__ __host__ __forceinline__ int moe_xf_floats(int D, int topk, int Fe) {
  if (!topk) return 0;
  const int b = mx_x_bytes(1, D) > mx_x_bytes(topk, Fe) ? mx_x_bytes(1, D) : mx_x_bytes(topk, Fe);
  return (b / 4 + 31) / 32 * 32;
}

// 2^(e - 127) for an e8m0 scale byte (e = 0: 2^-127, a denormal).
__device__ __forceinline__ float mx_scale(uint32_t e) {
  return e == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(e << 23);
}

__device__ __forceinline__ uint16_t f16_rn(float f) {
  uint16_t h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f));
  return h;
}
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}

// Stores v (element k of vector j of an xm region for K columns) as its two
// f16 parts, m being the largest magnitude of k's 32-column block.
__device__ __forceinline__ void xm_store(uint8_t* xm, int K, int nvec, int j, int k, float v,
                                         float m) {
  int sh = 0;
  if (m > 0.f) {
    const int ex = (int)((__float_as_uint(m) >> 23) & 0xFF) - 127;
    sh = min(max(14 - ex, -126), 126);
  }
  const float xs = v * __uint_as_float((uint32_t)(sh + 127) << 23);
  const uint16_t hi = f16_rn(xs);
  const uint16_t mid = f16_rn(xs - f16_to_f32(hi));
  const int vb = mx_x_vbytes(K);
  reinterpret_cast<uint16_t*>(xm + (size_t)(2 * j) * vb)[k] = hi;
  reinterpret_cast<uint16_t*>(xm + (size_t)(2 * j + 1) * vb)[k] = mid;
  if ((threadIdx.x & 31) == 0)
    reinterpret_cast<float*>(xm + (size_t)nvec * 2 * vb)[j * (K / 32) + k / 32] =
        __uint_as_float((uint32_t)(127 - sh) << 23);
}

// xm_store of v[u] at k = k0 + u * kThreads (u < N) by the 32 lanes of a warp
// together, each k one column of a 32-column block (lane 0 at the block's
// first column; blocks at or past K are skipped). The N block maxima are
// reduced side by side, so the shuffle latency is paid once per batch.
template <int N>
__device__ __forceinline__ void xm_put_batch(uint8_t* xm, int K, int nvec, int j, int k0,
                                             const float* v) {
  float m[N];
#pragma unroll
  for (int u = 0; u < N; u++) m[u] = fabsf(v[u]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int u = 0; u < N; u++) m[u] = fmaxf(m[u], __shfl_xor_sync(0xFFFFFFFFu, m[u], o));
#pragma unroll
  for (int u = 0; u < N; u++) {
    const int k = k0 + u * kThreads;
    if (k - (k & 31) < K) xm_store(xm, K, nvec, j, k, v[u], m[u]);
  }
}

// Weight phase `wp` of a step.
template <bool MOE>
__device__ __forceinline__ Phase weight_phase(const MegaArgs& a, int wp) {
  Phase p;
  p.kind = phase_kind<MOE>(a, wp);
  if (p.kind == W_LM) {
    p.W = a.out_w;
    p.K = a.D;
    p.pairs = a.Vl / 2;
    return p;
  }
  const MegaLayer& ly = layer_table(a)[wp / phases_per_layer<MOE>(a)];
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
    case W_DOWN:
      p.W = ly.wd;
      p.K = a.Fl;
      p.pairs = a.D / 2;
      break;
    case W_ROUTER:
      p.W = ly.router;
      p.K = a.D;
      p.pairs = a.E / 2;
      break;
    case W_EGU:  // pair (slot j, f): gate row f and up row f of expert j
      p.W = nullptr;
      p.K = a.D;
      p.pairs = a.topk * a.Fe;
      break;
    default:  // W_EDOWN: output rows, one chunk per selected expert
      p.W = nullptr;
      p.K = a.Fe;
      p.pairs = a.D / 2;
      break;
  }
  return p;
}

// One chunk: rows [r0, r1) of the phase's matrix over columns [k0, k1): up
// to kMaxChunkRows rows, whole when they fit a buffer, else a column segment
// (a row group then spans several chunks). For W_EDOWN the segments are the
// selected experts (seg = slot).
struct Chunk {
  int r0, r1, k0, k1, seg;
  bool first_seg, last_seg;
};

struct Slice {
  int rb, re;     // rows [rb, re) of this CTA (whole row pairs)
  int rows;       // rows per chunk (even, at most kMaxChunkRows)
  int kseg;       // columns per chunk (a multiple of 256, or K)
  int spp;        // chunks per row group
  int nchunks;
};

__device__ __forceinline__ int row_stride(int cols) { return 2 * cols + kPad; }

// EGU chunk ci of a slice: pairs [p0, p0 + np), at most rows / 2 pairs and
// never across a selected-expert boundary (a multiple of Fe), so that each
// chunk's gate and up rows are contiguous runs of one expert.
__device__ __forceinline__ void egu_chunk(int pb, int pe, int R, int Fe, int ci, int& p0,
                                          int& np) {
  int p = pb;
  for (int i = 0;; i++) {
    const int n = min(R, min(pe, (p / Fe + 1) * Fe) - p);
    if (i == ci || p + n >= pe) {
      p0 = p;
      np = n;
      return;
    }
    p += n;
  }
}

__device__ __forceinline__ Slice cta_slice(const Phase& ph, int buf_bytes, int topk, int Fe) {
  Slice s;
  const long long np = ph.pairs;
  s.rb = 2 * (int)(np * blockIdx.x / gridDim.x);
  s.re = 2 * (int)(np * (blockIdx.x + 1) / gridDim.x);
  const int n = s.re - s.rb;
  const bool mx = ph.kind == W_EGU || ph.kind == W_EDOWN;
  const int want = min(mx ? kMaxChunkRows : kMaxDenseRows, max(n, 2));
  if (mx) {
    // Whole MXFP4 rows; the down rows once per selected expert; gate/up
    // chunks end at expert boundaries.
    s.rows = max(2, min(want, (buf_bytes / mx_row_bytes(ph.K)) & ~1));
    s.kseg = ph.K;
    s.spp = (ph.kind == W_EDOWN) ? topk : 1;
    if (ph.kind == W_EDOWN) {
      s.nchunks = ((n + s.rows - 1) / s.rows) * s.spp;
    } else {
      s.nchunks = 0;
      for (int p = s.rb / 2; p < s.re / 2; s.nchunks++)
        p += min(s.rows / 2, min(s.re / 2, (p / Fe + 1) * Fe) - p);
    }
    return s;
  }
  // Whole rows, as many as the slice has up to kMaxChunkRows and what a
  // buffer holds, when that is at least 16 rows (or the whole slice); else
  // row segments of kSegCols columns (each row segment is one bulk copy:
  // long segments keep the copy count per byte low), as many rows as a
  // buffer holds, the columns split into equal segments (multiples of 256).
  constexpr int kSegCols = 1024;
  const int whole = min(want, (buf_bytes / row_stride(ph.K)) & ~1);
  if (whole >= min(16, want)) {
    s.rows = whole;
    s.kseg = ph.K;
    s.spp = 1;
  } else {
    const int kmax = min(kSegCols, ph.K);
    s.rows = max(2, min(want, (buf_bytes / row_stride(kmax)) & ~1));
    s.spp = (ph.K + kmax - 1) / kmax;
    s.kseg = ((ph.K + s.spp - 1) / s.spp + 255) / 256 * 256;
  }
  s.nchunks = ((n + s.rows - 1) / s.rows) * s.spp;
  return s;
}

__device__ __forceinline__ Chunk slice_chunk(const Slice& s, const Phase& ph, int ci) {
  Chunk c;
  const int grp = ci / s.spp, seg = ci % s.spp;
  c.r0 = s.rb + grp * s.rows;
  c.r1 = min(c.r0 + s.rows, s.re);
  c.seg = seg;
  if (ph.kind == W_EDOWN) {
    c.k0 = 0;
    c.k1 = ph.K;
  } else {
    c.k0 = seg * s.kseg;
    c.k1 = min(c.k0 + s.kseg, ph.K);
  }
  c.first_seg = (seg == 0);
  c.last_seg = (seg == s.spp - 1);
  return c;
}

// Position in the producer's walk over the chunks of the launch.
struct Cursor {
  int step, wp, ci;
};

// This CTA's slice of each weight-phase kind; every layer has the same
// shapes, so they are computed once per launch.
__shared__ Slice s_slices[kKinds];

template <bool MOE>
__device__ void cursor_skip_empty(const MegaArgs& a, Cursor& c) {
  const int last = phases_per_layer<MOE>(a) * a.L;
  while (c.step < a.steps) {
    if (c.ci < s_slices[phase_kind<MOE>(a, c.wp)].nchunks) return;
    c.ci = 0;
    if (++c.wp > last) {
      c.wp = 0;
      c.step++;
    }
  }
}

// Bounded wait on an mbarrier phase; with `stop_on_err` it also returns as
// soon as the error flag is set. True when the phase completed. The error
// flag (global memory, one L2 round trip) is read only while waiting.
__device__ bool wait_bar(const MegaArgs& a, uint64_t* bar, unsigned parity,
                         bool stop_on_err = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  unsigned spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 63) == 0) {
      if (stop_on_err && *(volatile int*)a.err) return false;
      if (now_ns() - t0 > a.wait_ns) {
        atomicExch(a.err, 2);
        return false;
      }
    }
  }
  return true;
}

// The producer warp: copies every chunk of the launch, in the consumers'
// order, into the ring. Chunk g goes to buffer g % nbuf once the consumer
// warps have released that buffer's previous chunk (empty[b]); its rows land
// row_stride(k1 - k0) bytes apart. Stops issuing once the error flag is set;
// before returning it waits (bounded) until its copies have landed.
__device__ void expert_select(const MegaArgs& a, int l, unsigned e, int* sel, float* w);

__device__ __forceinline__ bool expert_owned(const MegaArgs& a, int ex) {
  return ex >= a.e_begin && ex < a.e_end;
}

// The producer's copy of the expert choice of the layer being streamed.
__shared__ int s_psel[kMaxTopk];

// An MXFP4 expert chunk in a buffer: the codes of its rows back to back,
// then their scales (rows of mx_scale_bytes). EGU chunk of np pairs (slot j,
// outputs f0 .. f0 + np): gate codes, up codes, gate scales, up scales;
// EDOWN chunk (slot ch.seg, output rows r0 .. r1): codes, scales. Each run
// is contiguous in memory, one bulk copy; experts this rank does not own
// are not copied.
__device__ void produce_mx(const MegaArgs& a, const Phase& ph, const Slice& sl, const Chunk& ch,
                           int ci, int l, char* buf, uint64_t* bar) {
  const int lane = threadIdx.x & 31;
  const int cb = ph.K / 2, sb = mx_scale_bytes(ph.K);
  const MegaLayer& ly = layer_table(a)[l];
  if (ph.kind == W_EGU) {
    int p0, np;
    egu_chunk(sl.rb / 2, sl.re / 2, sl.rows / 2, a.Fe, ci, p0, np);
    const int j = p0 / a.Fe, f0 = p0 % a.Fe;
    const bool own = expert_owned(a, s_psel[j]);
    if (lane == 0) {
      mbar_expect_tx(bar, own ? (unsigned)(2 * np * (cb + sb)) : 0u);
      if (own) {
        const size_t row = (size_t)(s_psel[j] - a.e_begin) * a.Fe + f0;
        bulk_copy_stream(buf, ly.gate_c + row * cb, (unsigned)(np * cb), bar);
        bulk_copy_stream(buf + (size_t)np * cb, ly.up_c + row * cb, (unsigned)(np * cb), bar);
        bulk_copy_stream(buf + (size_t)2 * np * cb, ly.gate_s + row * sb, (unsigned)(np * sb), bar);
        bulk_copy_stream(buf + (size_t)2 * np * cb + (size_t)np * sb, ly.up_s + row * sb,
                  (unsigned)(np * sb), bar);
      }
    }
  } else {
    const int nr = ch.r1 - ch.r0, j = ch.seg;
    const bool own = expert_owned(a, s_psel[j]);
    if (lane == 0) {
      mbar_expect_tx(bar, own ? (unsigned)(nr * (cb + sb)) : 0u);
      if (own) {
        const size_t row = (size_t)(s_psel[j] - a.e_begin) * a.D + ch.r0;
        bulk_copy_stream(buf, ly.down_c + row * cb, (unsigned)(nr * cb), bar);
        bulk_copy_stream(buf + (size_t)nr * cb, ly.down_s + row * sb, (unsigned)(nr * sb), bar);
      }
    }
  }
  __syncwarp();
}

template <bool MOE>
__device__ void produce(const MegaArgs& a, char* base, int buf_bytes, int nbuf, uint64_t* full,
                        uint64_t* empty) {
  const int lane = threadIdx.x & 31;
  Cursor c = {0, 0, 0};
  unsigned g = 0;
  int psel_key = -1;  // (step, layer) of s_psel
  for (;;) {
    cursor_skip_empty<MOE>(a, c);
    if (c.step >= a.steps) break;
    const int b = (int)(g % nbuf);
    if (g >= (unsigned)nbuf) {
      // Only a wait that ran out (or saw the error flag) stops the
      // producer: no global load per chunk.
      int ok = 1;
      if (lane == 0) ok = wait_bar(a, empty + b, (g / nbuf - 1) & 1) ? 1 : 0;
      if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) break;
    }
    const Phase ph = weight_phase<MOE>(a, c.wp);
    const Chunk ch = slice_chunk(s_slices[ph.kind], ph, c.ci);
    char* buf = base + (size_t)b * buf_bytes;
    if constexpr (MOE) {
      if (ph.kind == W_EGU || ph.kind == W_EDOWN) {
        // The expert rows depend on this step's router output of the layer.
        const int l = c.wp / phases_per_layer<MOE>(a);
        if (psel_key != c.step * a.L + l) {
          expert_select(a, l, a.epoch + (unsigned)c.step, s_psel, nullptr);
          psel_key = c.step * a.L + l;
          if (*(volatile int*)a.err) break;  // the choice may be incomplete
        }
        produce_mx(a, ph, s_slices[ph.kind], ch, c.ci, l, buf, full + b);
        c.ci++;
        g++;
        continue;
      }
    }
    const int nr = ch.r1 - ch.r0, w = ch.k1 - ch.k0;
    const int stride = row_stride(w);
    if (lane == 0) mbar_expect_tx(full + b, (unsigned)(nr * w * 2));
    __syncwarp();
    const uint16_t* src = ph.W + (size_t)ch.r0 * ph.K + ch.k0;
    for (int r = lane; r < nr; r += 32)
      bulk_copy_stream(buf + (size_t)r * stride, src + (size_t)r * ph.K, (unsigned)(w * 2), full + b);
    c.ci++;
    g++;
  }
  // The last use of each buffer: its copy has landed (or the wait ran out).
  if (lane == 0)
    for (unsigned i = (g > (unsigned)nbuf ? g - nbuf : 0); i < g; i++)
      wait_bar(a, full + i % nbuf, (i / nbuf) & 1, false);
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Activation staging
// ---------------------------------------------------------------------------
// The matvec input lives in shared memory as `parts` bf16 arrays (hi, mid,
// lo), part p at element p * (K + 32). Inside an array, each block of 32
// columns holds, for c = 0..3, the 16 bytes lane c of a warp feeds to two
// m16n8k16 steps: words (2c, 2c + 8) of the block's first 16 columns, then
// of its last 16 (a word = two consecutive columns).
__device__ __forceinline__ int xq_pos(int k) {
  const int kk = k & 31;
  const int step = kk >> 4, ks = kk & 15;
  return (k & ~31) + ((ks & 7) >> 1) * 8 + (step * 2 + (ks >> 3)) * 2 + (ks & 1);
}

__device__ __forceinline__ int xq_stride(int K) { return K + 32; }

// Round to nearest even, fp32 -> bf16 bits (finite inputs).
__device__ __forceinline__ uint16_t bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ void xq_put(uint16_t* xq, int K, int parts, int k, float v) {
  const int pos = xq_pos(k), ps = xq_stride(K);
  const uint16_t p0 = bf16_rne(v);
  const float r1 = v - bf16_to_f32(p0);
  const uint16_t p1 = bf16_rne(r1);
  xq[pos] = p0;
  xq[ps + pos] = p1;
  if (parts > 2) xq[2 * ps + pos] = bf16_rne(r1 - bf16_to_f32(p1));
}

// Sum over the consumer threads (warp sums, then the warps' in order).
__device__ __forceinline__ float cta_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  csync();
  if (lane == 0) red[warp] = v;
  csync();
  float t = (lane < kWarps) ? red[lane] : 0.f;
  return warp_sum(t);
}

// Largest K an RMSNorm staging handles (K = embedding_dim), read in rounds
// of kNormBatch flagged words per thread.
constexpr int kNormBatch = 16;
constexpr int kNormMaxK = 8192;

// RMSNorm gains in shared memory: one bf16 vector of D, refilled by a bulk
// copy (consumer thread 0) as soon as a norm staging is done with it, with
// the gains of the next norm (after the attention norm the FFN norm, after
// the FFN norm the next layer's attention norm or the final norm), two
// phases or more before they are needed, so that no gain load sits on a
// phase's critical path. Every consumer thread counts the fills; thread 0
// issues them.
struct Gains {
  uint16_t* buf;
  uint64_t* bar;   // in shared memory
  unsigned n;      // fills issued so far
};

__device__ __forceinline__ void gains_fill(Gains& gs, const uint16_t* src, int D) {
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(gs.bar, (unsigned)D * 2u);
    bulk_copy(gs.buf, src, (unsigned)D * 2u, gs.bar);
  }
  gs.n++;
}

__device__ __forceinline__ const uint16_t* gains_ready(const MegaArgs& a, Gains& gs) {
  wait_bar(a, gs.bar, (gs.n - 1) & 1);
  return gs.buf;
}

// xq = rmsnorm(x) * gains from the flagged vector src (epoch e); the raw
// values also go to xraw[K] (and the normalised ones to the xm region, as
// vector 0, when set). Thread t owns k = t + u * kThreads. The loops are kept short: this code
// runs once per phase, from a cold instruction cache.
__device__ void stage_norm_ll(const MegaArgs& a, const u64* src, unsigned e, Gains& gs,
                              int K, uint16_t* xq, int parts, float* xraw, float* red, int ph,
                              uint8_t* xm = nullptr) {
  const int tid = threadIdx.x;
  float ss = 0.f;
  for (int b = 0; b * kThreads < K; b += kNormBatch) {
    float v[kNormBatch];
    ll_gather<kNormBatch>(a, src, tid + b * kThreads, kThreads, K, e, v);
#pragma unroll
    for (int u = 0; u < kNormBatch; u++) {
      const int k = tid + (b + u) * kThreads;
      if (k < K) {
        xraw[k] = v[u];
        ss += v[u] * v[u];
      }
    }
  }
  trace_mark(a, ph, MARK_INPUTS);
  ss = cta_sum(ss, red);
  trace_mark(a, ph, MARK_NORMED);
  ss /= (float)K;
  const float inv = 1.0f / sqrtf(ss + a.eps);
  const uint16_t* g = gains_ready(a, gs);
  trace_mark(a, ph, MARK_GAINS);
  if (xm) {
    // Also the MXFP4 expert input (K is then a multiple of 32: a warp's
    // lanes hold one block), in batches of four blocks.
    for (int k0 = tid; k0 - tid < K; k0 += 4 * kThreads) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int k = k0 + u * kThreads;
        v[u] = 0.f;
        if (k < K) {
          v[u] = (xraw[k] * inv) * bf16_to_f32(g[k]);
          xq_put(xq, K, parts, k, v[u]);
        }
      }
      xm_put_batch<4>(xm, K, 1, 0, k0, v);
    }
  } else {
    // Four elements per iteration, their loads first (independent chains).
    for (int k0 = tid; k0 < K; k0 += 4 * kThreads) {
      float xv[4], gv[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int k = k0 + u * kThreads;
        xv[u] = k < K ? xraw[k] : 0.f;
        gv[u] = k < K ? bf16_to_f32(g[k]) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int k = k0 + u * kThreads;
        if (k < K) xq_put(xq, K, parts, k, (xv[u] * inv) * gv[u]);
      }
    }
  }
  trace_mark(a, ph, MARK_SCALED);
  csync();
  trace_mark(a, ph, MARK_SYNCED);
}

// xq = the flagged vector src (epoch e), K floats.
__device__ void stage_plain_ll(const MegaArgs& a, const u64* src, unsigned e, int K, uint16_t* xq,
                               int parts, int ph) {
  const int tid = threadIdx.x;
  constexpr int B = 16;
  for (int base = tid; base < K; base += B * kThreads) {
    float v[B];
    ll_gather<B>(a, src, base, kThreads, K, e, v);
#pragma unroll
    for (int u = 0; u < B; u++) {
      const int k = base + u * kThreads;
      if (k < K) xq_put(xq, K, parts, k, v[u]);
    }
  }
  trace_mark(a, ph, MARK_INPUTS);
  csync();
}

// Layer-0 input: the embedding row of `token` (xraw) and its RMSNorm (xq)
// with the gains in shared memory.
__device__ void stage_embedding(const MegaArgs& a, int token, Gains& gs, uint16_t* xq,
                                int parts, float* xraw, float* red) {
  const int tid = threadIdx.x, K = a.D;
  const uint16_t* row = a.emb + (size_t)token * K;
  float ss = 0.f;
  for (int b = 0; b * kThreads < K; b += kNormBatch) {
    float v[kNormBatch];
#pragma unroll
    for (int u = 0; u < kNormBatch; u++) {
      const int k = tid + (b + u) * kThreads;
      v[u] = (k < K) ? bf16_to_f32(__ldg(row + k)) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kNormBatch; u++) {
      const int k = tid + (b + u) * kThreads;
      if (k < K) {
        xraw[k] = v[u];
        ss += v[u] * v[u];
      }
    }
  }
  ss = cta_sum(ss, red);
  ss /= (float)K;
  const float inv = 1.0f / sqrtf(ss + a.eps);
  const uint16_t* g = gains_ready(a, gs);
  for (int k = tid; k < K; k += kThreads)
    xq_put(xq, K, parts, k, (xraw[k] * inv) * bf16_to_f32(g[k]));
  csync();
}

// ---------------------------------------------------------------------------
// Consuming one weight phase
// ---------------------------------------------------------------------------
// The ring lives at fixed shared-memory places (the buffers at the start of
// the dynamic region, a.buf_bytes apart; the barriers and the per-warp row
// sums in file-scope arrays) and its geometry in the kernel arguments, so
// that the chunk loops keep only two counters in registers.
__shared__ __align__(8) uint64_t s_full[kMaxRing];   // the chunk in buffer b has landed
__shared__ __align__(8) uint64_t s_empty[kMaxRing];  // the consumer warps are done with it
__shared__ __align__(16) float s_mvred[2 * kWarps * kMaxChunkRows];  // per-warp row sums
__shared__ unsigned long long s_tsum[4];  // trace: wait, dot, reduce sums; last mark

struct Ring {
  unsigned g;      // chunks consumed so far
  unsigned nred;   // cross-warp reductions so far (selects the row-sum half)
  int b;           // buffer of chunk g (g mod nbuf)
  unsigned par;    // phase parity of that buffer's barriers ((g / nbuf) & 1)
};

// The next chunk of the ring (without a division per chunk).
__device__ __forceinline__ void ring_next(Ring& r, const MegaArgs& a) {
  r.g++;
  if (++r.b == a.nbuf) {
    r.b = 0;
    r.par ^= 1u;
  }
}

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
    case W_ROUTER:
      ll_store(o.dst + r0, y0, o.e);
      ll_store(o.dst + r0 + 1, y1, o.e);
      break;
    case W_O:
    case W_DOWN:
    case W_EDOWN:
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

// Consumes every chunk of weight phase `wp` with the activation parts in xq
// (K columns). Warp w multiplies 32-column blocks w, w + 8, ... of a chunk
// for all of the chunk's 16-row groups and keeps its row sums in shared
// memory (added up over the column segments of a row group); after the last
// segment the warps' sums meet and thread t finishes row pair t. For the LM
// head, (bv, bi) track the thread's argmax.
template <bool MOE, int KIND>
__device__ void consume_phase(const MegaArgs& a, Ring& r, int wp, const uint16_t* xq, int parts,
                              const Out& o, float& bv, int& bi, int ph) {
  trace_mark(a, ph, MARK_STAGED);
  const Phase phs = weight_phase<MOE>(a, wp);
  const Slice s = s_slices[KIND];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int xps = xq_stride(phs.K) / 8;  // uint4 per activation part
  const uint4* xq4 = reinterpret_cast<const uint4*>(xq);
  const bool tr = a.trace != nullptr;
  // Trace sums (thread 0 only) in shared memory: no registers held across
  // the chunk loop when tracing is off.
  const bool tr0 = tr && tid == 0;
  if (tr0) s_tsum[0] = s_tsum[1] = s_tsum[2] = 0;
  // The chunk's row group and column segment, advanced per chunk (the order
  // of slice_chunk, without its divisions), and the warp's row sums of the
  // current row group, kept in registers across its column segments.
  int grp = 0, segi = 0;
  float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0, acc2 = acc0;
  for (int ci = 0; ci < s.nchunks; ci++) {
    const int b = r.b;
    if (tr0) s_tsum[3] = now_ns();
    wait_bar(a, s_full + b, r.par);
    if (tr) {
      const unsigned long long t1 = now_ns();
      if (tr0) {
        s_tsum[0] += t1 - s_tsum[3];
        s_tsum[3] = t1;
      }
    }
    if (ci == 0) trace_mark(a, ph, MARK_READY);
    Chunk ch;
    ch.r0 = s.rb + grp * s.rows;
    ch.r1 = min(ch.r0 + s.rows, s.re);
    ch.seg = segi;
    ch.k0 = segi * s.kseg;
    ch.k1 = min(ch.k0 + s.kseg, phs.K);
    ch.first_seg = segi == 0;
    ch.last_seg = segi == s.spp - 1;
    if (++segi == s.spp) {
      segi = 0;
      grp++;
    }
    const int nr = ch.r1 - ch.r0;
    const int stride = row_stride(ch.k1 - ch.k0);
    const int nkb = (ch.k1 - ch.k0) >> 5;
    // Folded chunk (at most 8 whole rows): fragment rows 8..15 are the same
    // rows over the second half of the columns, and B carries the parts of
    // both halves (columns p and parts + p), so each warp walks half as many
    // 32-column blocks.
    const bool fold = nr <= 8 && ch.first_seg && ch.last_seg && (nkb & 1) == 0;
    const int nkw = fold ? nkb >> 1 : nkb;  // blocks walked
    const int ng = fold ? 1 : (nr + 15) >> 4;
    const int xhalf = fold && g >= parts;    // B column g: part g - parts, second half
    const bool has_x = g < (fold ? 2 * parts : parts);
    const uint4* xsrc = xq4 + (size_t)(g - xhalf * parts) * xps +
                        (size_t)(((ch.k0 >> 5) + xhalf * nkw) * 4 + c);
    // Folded chunks: one accumulator pair (named, by value).
    float4 facc0 = make_float4(0.f, 0.f, 0.f, 0.f), facc1 = facc0;
    // Lane address for ldmatrix: row (lane % 8) + 8 ((lane / 8) % 2) of a
    // 16-row group (rows past the chunk read its last row), 8 columns at
    // 8 (lane / 16) of the 16-column step.
    const uint32_t bbase = smem_addr(s_dyn + (size_t)b * a.buf_bytes) + (uint32_t)((lane >> 4) * 16);
    const int m = (lane & 7) + ((lane >> 3) & 1) * 8;  // fragment row of this lane's address
    const uint32_t lrow0 =
        fold ? bbase + (uint32_t)(min(m & 7, nr - 1) * stride + (m >> 3) * nkw * 64) : 0u;
    if (fold) {
      for (int kb = warp; kb < nkw; kb += kWarps) {
        uint4 xb = make_uint4(0u, 0u, 0u, 0u);
        if (has_x) xb = xsrc[(size_t)kb * 4];
        const uint4 m0 = ldsm4(lrow0 + (uint32_t)(kb * 64));
        const uint4 m1 = ldsm4(lrow0 + (uint32_t)(kb * 64 + 32));
        mma4(facc0, m0, xb.x, xb.y);
        mma4(facc1, m1, xb.z, xb.w);
      }
    }
    __syncwarp();
    // Column p of the accumulators holds part p's products: lane 4g has
    // parts 0, 1 and lane 4g + 1 part 2 of rows g and g + 8. The warp's row
    // sums go to its red row.
    float* red = s_mvred + (size_t)(r.nred & 1) * kWarps * kMaxChunkRows;
    float* wred = red + warp * kMaxChunkRows;
    if (fold) {
      if (lane == 0) mbar_arrive(s_empty + b);  // this warp is done with buffer b
      // Row g: columns 0..parts-1 of fragment row g (first half) plus
      // columns parts..2 parts-1 of fragment row g + 8 (second half).
      const float c0 = facc0.x + facc1.x, c1 = facc0.y + facc1.y;
      const float c2 = facc0.z + facc1.z, c3 = facc0.w + facc1.w;
      const float n1c0 = __shfl_down_sync(0xFFFFFFFFu, c0, 1);
      const float n1c1 = __shfl_down_sync(0xFFFFFFFFu, c1, 1);
      const float n1c3 = __shfl_down_sync(0xFFFFFFFFu, c3, 1);
      const float n1c2 = __shfl_down_sync(0xFFFFFFFFu, c2, 1);
      const float n2c2 = __shfl_down_sync(0xFFFFFFFFu, c2, 2);
      const float n2c3 = __shfl_down_sync(0xFFFFFFFFu, c3, 2);
      if (c == 0) {
        // parts == 3: first half = C[g][0..2], second = C[g+8][3..5];
        // parts == 2: first half = C[g][0..1], second = C[g+8][2..3].
        const float v = (parts == 3) ? ((c0 + c1) + n1c0) + (n1c3 + (n2c2 + n2c3))
                                     : (c0 + c1) + (n1c2 + n1c3);
        (void)n1c1;
        wred[g] = v;
      }
    } else {
      // The chunk's 16-row groups (at most three: 48 rows) per 32-column
      // block: each block's fragment loads issued before its MMAs (one
      // accumulator chain per group), so that the ldmatrix and MMA latencies
      // overlap.
      {
        const bool two = ng > 1;    // ng <= 3: dense chunks have at most 48 rows
        const bool three = ng > 2;  // (a third group mostly for a slice's last rows)
        const uint32_t l0 = bbase + (uint32_t)(min(m, nr - 1) * stride);
        const uint32_t l1 = bbase + (uint32_t)(min(16 + m, nr - 1) * stride);
        const uint32_t l2 = bbase + (uint32_t)(min(32 + m, nr - 1) * stride);
        // One accumulator per 16-row group (both k16 steps of a block add
        // into it, and so do the later column segments of the chunk's rows),
        // fragments as values; the first two groups always (with one group,
        // the second reads the chunk's last row again and is discarded), so
        // the common loop has no branches and no arrays.
        if (ch.first_seg) acc0 = acc1 = acc2 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
        for (int kb = warp; kb < nkw; kb += kWarps) {
          uint4 x0 = make_uint4(0u, 0u, 0u, 0u);
          if (has_x) x0 = xsrc[(size_t)kb * 4];
          const uint32_t o0 = (uint32_t)(kb * 64);
          const uint4 f00 = ldsm4(l0 + o0), f01 = ldsm4(l0 + o0 + 32);
          const uint4 f10 = ldsm4(l1 + o0), f11 = ldsm4(l1 + o0 + 32);
          mma4(acc0, f00, x0.x, x0.y);
          mma4(acc1, f10, x0.x, x0.y);
          mma4(acc0, f01, x0.z, x0.w);
          mma4(acc1, f11, x0.z, x0.w);
          if (three) {
            const uint4 f20 = ldsm4(l2 + o0), f21 = ldsm4(l2 + o0 + 32);
            mma4(acc2, f20, x0.x, x0.y);
            mma4(acc2, f21, x0.z, x0.w);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty + b);  // done with buffer b
        // After the row group's last column segment: the warp's row sums.
#pragma unroll
        for (int q = 0; q < 3; q++) {
          if (!ch.last_seg || (q == 1 && !two) || (q == 2 && !three)) break;
          const float4 aq = q == 2 ? acc2 : (q ? acc1 : acc0);
          const float lo0 = __shfl_down_sync(0xFFFFFFFFu, aq.x, 1);
          const float lo2 = __shfl_down_sync(0xFFFFFFFFu, aq.z, 1);
          if (c == 0) {
            const int rr = q * 16 + g;
            wred[rr] = (aq.x + aq.y) + lo0;
            wred[rr + 8] = (aq.z + aq.w) + lo2;
          }
        }
      }
    }
    if (tr) {
      const unsigned long long t1 = now_ns();
      if (tr0) {
        s_tsum[1] += t1 - s_tsum[3];
        s_tsum[3] = t1;
      }
    }
    if (ch.last_seg) {
      r.nred++;
      csync();
      if (tid < (nr >> 1)) {
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
          y0 += red[w * kMaxChunkRows + 2 * tid];
          y1 += red[w * kMaxChunkRows + 2 * tid + 1];
        }
        pair_epilogue(a, o, KIND, (ch.r0 >> 1) + tid, y0, y1, bv, bi);
      }
      if (tr0) s_tsum[2] += now_ns() - s_tsum[3];
    }
    ring_next(r, a);
  }
  trace_mark(a, ph, MARK_CONSUMED);
  if (tr0) {
    trace_put(a, ph, SUM_WAIT, s_tsum[0]);
    trace_put(a, ph, SUM_COMPUTE, s_tsum[1] + s_tsum[2]);
    trace_put(a, ph, SUM_DOT, s_tsum[1]);
    trace_put(a, ph, SUM_REDUCE, s_tsum[2]);
  }
}

// ---------------------------------------------------------------------------
// Mixture of experts
// ---------------------------------------------------------------------------
// Expert choice for layer l from its router logits (flagged vector rl,
// epoch e), as the per-op router (kernels.cu moe_topk): topk rounds of the
// warp argmax (ties -> lower index), then the softmax over the chosen
// logits in choice order. One warp; lanes s < topk write sel[s] and, when
// w is set, w[s]; the warp is synchronised on return.
__device__ void expert_select(const MegaArgs& a, int l, unsigned e, int* sel, float* w) {
  const int lane = threadIdx.x & 31;
  float v[4];  // E <= 128
  ll_gather<4>(a, a.ll + a.llo.rl + (size_t)l * a.E, lane, 32, a.E, e, v);
#pragma unroll
  for (int u = 0; u < 4; u++)
    if (lane + 32 * u >= a.E) v[u] = -INFINITY;
  // Round s's winner stays in lane s (registers only: arrays indexed by
  // the runtime round would live in local memory, one L2 round trip per
  // access).
  float mine = -INFINITY;
  int mine_i = 0;
  for (int s = 0; s < a.topk; s++) {
    float best = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int ex = lane + 32 * u;
      if (ex < a.E && (v[u] > best || (v[u] == best && ex < bi))) {
        best = v[u];
        bi = ex;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xFFFFFFFFu, best, o);
      const int i2 = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (v2 > best || (v2 == best && i2 < bi)) {
        best = v2;
        bi = i2;
      }
    }
    if (lane == s) {
      mine = best;
      mine_i = bi;
    }
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (lane + 32 * u == bi) v[u] = -INFINITY;
  }
  // Softmax over the chosen logits, the sum taken in choice order (every
  // lane takes part in every shuffle).
  const float mx = __shfl_sync(0xFFFFFFFFu, mine, 0);
  const float ex = lane < a.topk ? expf(mine - mx) : 0.f;
  float sum = 0.f;
  for (int s = 0; s < a.topk; s++) sum += __shfl_sync(0xFFFFFFFFu, ex, s);
  if (lane < a.topk) {
    sel[lane] = mine_i;
    if (w) w[lane] = ex / sum;
  }
  __syncwarp();
}

// Four e2m1 pairs (the bytes of w, low byte first) as f16x2 words, the low
// nibble of a byte in the low half (exact: every e2m1 value is an f16).
__device__ __forceinline__ uint4 e2m1x8_to_f16v(uint32_t w) {
  uint4 h;
  asm("{\n"
      " .reg .b8 b0, b1, b2, b3;\n"
      " mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      " cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      " cvt.rn.f16x2.e2m1x2 %3, b3;\n"
      "}"
      : "=r"(h.x), "=r"(h.y), "=r"(h.z), "=r"(h.w)
      : "r"(w));
  return h;
}
// d += A (16x16 f16) * B (16x8 f16), fp32 accumulators; fragments as mma4.
__device__ __forceinline__ void mma_f16v(float4& d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d.x), "+f"(d.y), "+f"(d.z), "+f"(d.w)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One MXFP4 chunk on the tensor cores: rows [0, nr) (at most kMaxChunkRows;
// codes at buf + i cb, scale bytes at buf + nr cb + i sb) times vector j of
// the xm region (K columns). The products of a 32-column block are exact
// in f16 x f16 -> fp32: lane 4g + c holds, from ldmatrix, the 32-bit code
// word c (columns 8c .. 8c + 7) of rows g and g + 8 of a block, and those
// eight columns are the lane's k slots of the block's two m16n8k16 steps;
// B column n is x part min(n, 1) over the same columns (one 16-byte load).
// Each block's accumulators are scaled by (weight block scale) x (x block
// scale) into the row sums. Warp w walks block pairs w, w + 8, ... for every
// 16-row group; lane 4g stores (first) or adds wgt x its row sums to
// wred[row].
__device__ __forceinline__ void mx_chunk_dot(const uint8_t* buf, int nr, int K, int cb, int sb,
                                             const uint8_t* xm, int nvec, int j, float wgt,
                                             bool first, float* wred) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int nb = K >> 5, npair = (nb + 1) >> 1, ng = (nr + 15) >> 4;
  const int vb = mx_x_vbytes(K);
  const uint8_t* xp = xm + (size_t)(2 * j + min(g, 1)) * vb + c * 16;
  const float* xsi = reinterpret_cast<const float*>(xm + (size_t)nvec * 2 * vb) + j * nb;
  const uint8_t* scl = buf + (size_t)nr * cb;
  // ldmatrix lane address: row (lane % 8) + 8 ((lane / 8) % 2) of group q
  // (rows past the chunk read its last row), block + lane / 16.
  const uint32_t bbase = smem_addr(buf) + (uint32_t)((lane >> 4) * 16);
  const int m = (lane & 7) + ((lane >> 3) & 1) * 8;
  // Named float4 accumulators and by-value fragments: arrays written under
  // runtime conditions end up in local memory (served by L2 here).
  float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f), acc1 = acc0, acc2 = acc0, acc3 = acc0;
  // One 16-row group q of block pair kp: codes by ldmatrix, e2m1 -> f16 in
  // registers, two MMA pairs, scaled into the group's accumulator.
  auto group = [&](int q, int kp, int b0, bool two, uint4 x0, uint4 x1, float xs0, float xs1,
                   float4& acc) {
    const uint4 w = ldsm4(bbase + (uint32_t)(min(q * 16 + m, nr - 1) * cb + kp * 32));
    const uint32_t sg =
        *reinterpret_cast<const uint16_t*>(scl + min(q * 16 + g, nr - 1) * sb + b0);
    const uint32_t s8 =
        *reinterpret_cast<const uint16_t*>(scl + min(q * 16 + g + 8, nr - 1) * sb + b0);
    uint4 hg = e2m1x8_to_f16v(w.x), h8 = e2m1x8_to_f16v(w.y);
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    mma_f16v(t, hg.x, h8.x, hg.y, h8.y, x0.x, x0.y);
    mma_f16v(t, hg.z, h8.z, hg.w, h8.w, x0.z, x0.w);
    float fg = mx_scale(sg & 0xFF) * xs0, f8 = mx_scale(s8 & 0xFF) * xs0;
    acc.x = fmaf(t.x, fg, acc.x);
    acc.y = fmaf(t.y, fg, acc.y);
    acc.z = fmaf(t.z, f8, acc.z);
    acc.w = fmaf(t.w, f8, acc.w);
    if (two) {
      float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
      hg = e2m1x8_to_f16v(w.z);
      h8 = e2m1x8_to_f16v(w.w);
      mma_f16v(u, hg.x, h8.x, hg.y, h8.y, x1.x, x1.y);
      mma_f16v(u, hg.z, h8.z, hg.w, h8.w, x1.z, x1.w);
      fg = mx_scale(sg >> 8) * xs1;
      f8 = mx_scale(s8 >> 8) * xs1;
      acc.x = fmaf(u.x, fg, acc.x);
      acc.y = fmaf(u.y, fg, acc.y);
      acc.z = fmaf(u.z, f8, acc.z);
      acc.w = fmaf(u.w, f8, acc.w);
    }
  };
  for (int kp = warp; kp < npair; kp += kWarps) {
    const int b0 = 2 * kp;
    const bool two = b0 + 1 < nb;
    const uint4 x0 = *reinterpret_cast<const uint4*>(xp + (size_t)b0 * 64);
    const uint4 x1 = two ? *reinterpret_cast<const uint4*>(xp + (size_t)(b0 + 1) * 64) : x0;
    const float xs0 = xsi[b0], xs1 = two ? xsi[b0 + 1] : 0.f;
    group(0, kp, b0, two, x0, x1, xs0, xs1, acc0);
    if (ng > 1) group(1, kp, b0, two, x0, x1, xs0, xs1, acc1);
    if (ng > 2) group(2, kp, b0, two, x0, x1, xs0, xs1, acc2);
    if (ng > 3) group(3, kp, b0, two, x0, x1, xs0, xs1, acc3);
  }
  // Lane 4g: columns 0 and 1 (parts hi and mid) of rows g and g + 8.
  if (c == 0) {
    auto put = [&](int q, float4 a4) {
      const int r0 = q * 16 + g, r8 = r0 + 8;
      if (r0 < nr) wred[r0] = (first ? 0.f : wred[r0]) + wgt * (a4.x + a4.y);
      if (r8 < nr) wred[r8] = (first ? 0.f : wred[r8]) + wgt * (a4.z + a4.w);
    };
    put(0, acc0);
    put(1, acc1);
    put(2, acc2);
    put(3, acc3);
  }
}

// Gate/up of the selected experts, one chunk of np (gate, up) row pairs of
// expert sel[j] at a time (2 np rows: gate rows then up rows); after each
// chunk the warps' row sums meet and thread i publishes swiglu(gate_i . x,
// up_i . x) in the flagged vector hm (experts this rank does not own:
// nothing). x is vector 0 of the xm region.
__device__ void consume_mx_gu(const MegaArgs& a, Ring& r, int l, const uint8_t* xm,
                              const int* sel, unsigned e, int ph) {
  trace_mark(a, ph, MARK_STAGED);
  const Slice s = s_slices[W_EGU];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cb = a.D / 2, sb = mx_scale_bytes(a.D);
  u64* hm = a.ll + a.llo.hm + (size_t)l * a.topk * a.Fe;
  const bool tr = a.trace != nullptr;
  unsigned long long t_wait = 0, t0 = 0;
  for (int ci = 0; ci < s.nchunks; ci++) {
    const int b = r.b;
    if (tr) t0 = now_ns();
    wait_bar(a, s_full + b, r.par);
    if (tr) t_wait += now_ns() - t0;
    if (ci == 0) trace_mark(a, ph, MARK_READY);
    int p0, np;
    egu_chunk(s.rb / 2, s.re / 2, s.rows / 2, a.Fe, ci, p0, np);
    const int j = p0 / a.Fe, f0 = p0 % a.Fe;
    const bool own = expert_owned(a, sel[j]);
    float* red = s_mvred + (size_t)(r.nred & 1) * kWarps * kMaxChunkRows;
    if (own)
      mx_chunk_dot(reinterpret_cast<const uint8_t*>(s_dyn + (size_t)b * a.buf_bytes), 2 * np,
                   a.D, cb, sb, xm, 1, 0, 1.f, true, red + warp * kMaxChunkRows);
    __syncwarp();
    if (lane == 0) mbar_arrive(s_empty + b);
    if (own) {
      r.nred++;
      csync();
      if (tid < np) {
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
          gs += red[w * kMaxChunkRows + tid];
          us += red[w * kMaxChunkRows + np + tid];
        }
        ll_store(hm + (size_t)j * a.Fe + f0 + tid, swiglu(gs, us), e);
      }
    }
    ring_next(r, a);
  }
  csync();  // the xm region (the normalised x) is read no more
  trace_mark(a, ph, MARK_CONSUMED);
  trace_put(a, ph, SUM_WAIT, t_wait);
}

// xm vectors j < topk = the selected experts' SwiGLU outputs (flagged
// vector hm, epoch e), for the experts this rank owns.
__device__ void stage_moe_h(const MegaArgs& a, int l, unsigned e, const int* sel, uint8_t* xm,
                            int ph) {
  constexpr int B = 16;
  for (int j = 0; j < a.topk; j++) {
    if (!expert_owned(a, sel[j])) continue;
    const u64* src = a.ll + a.llo.hm + ((size_t)l * a.topk + j) * a.Fe;
    for (int base = threadIdx.x; base - (int)threadIdx.x < a.Fe; base += B * kThreads) {
      float v[B];
      ll_gather<B>(a, src, base, kThreads, a.Fe, e, v);
      // A warp's 32 lanes hold one 32-column block (Fe is a multiple of 32).
#pragma unroll
      for (int u = 0; u < B; u++)
        if (base + u * kThreads >= a.Fe) v[u] = 0.f;
      xm_put_batch<B>(xm, a.Fe, a.topk, j, base, v);
    }
  }
  trace_mark(a, ph, MARK_INPUTS);
  csync();
}

// Down rows of the selected experts: one chunk per (row group, expert j);
// the warps add w_j (down_j[row] . h_j) to their row sums in choice order;
// after the last expert, thread t finishes row pair t (residual add, or the
// tensor-parallel push).
__device__ void consume_mx_down(const MegaArgs& a, Ring& r, const uint8_t* xm, const int* sel,
                                const float* selw, const Out& o, float& bv, int& bi, int ph) {
  trace_mark(a, ph, MARK_STAGED);
  const Slice s = s_slices[W_EDOWN];
  const Phase phs = {nullptr, a.Fe, a.D / 2, W_EDOWN};
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cb = a.Fe / 2, sb = mx_scale_bytes(a.Fe);
  const bool tr = a.trace != nullptr;
  unsigned long long t_wait = 0, t0 = 0;
  for (int ci = 0; ci < s.nchunks; ci++) {
    const int b = r.b;
    if (tr) t0 = now_ns();
    wait_bar(a, s_full + b, r.par);
    if (tr) t_wait += now_ns() - t0;
    if (ci == 0) trace_mark(a, ph, MARK_READY);
    const Chunk ch = slice_chunk(s, phs, ci);
    const int nr = ch.r1 - ch.r0, j = ch.seg;
    float* red = s_mvred + (size_t)(r.nred & 1) * kWarps * kMaxChunkRows;
    float* wred = red + warp * kMaxChunkRows;
    if (expert_owned(a, sel[j])) {
      mx_chunk_dot(reinterpret_cast<const uint8_t*>(s_dyn + (size_t)b * a.buf_bytes), nr, a.Fe,
                   cb, sb, xm, a.topk, j, selw[j], ch.first_seg, wred);
    } else if (ch.first_seg && lane == 0) {
      for (int i = 0; i < nr; i++) wred[i] = 0.f;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(s_empty + b);
    if (ch.last_seg) {
      r.nred++;
      csync();
      if (tid < (nr >> 1)) {
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
          y0 += red[w * kMaxChunkRows + 2 * tid];
          y1 += red[w * kMaxChunkRows + 2 * tid + 1];
        }
        pair_epilogue(a, o, W_EDOWN, (ch.r0 >> 1) + tid, y0, y1, bv, bi);
      }
    }
    ring_next(r, a);
  }
  trace_mark(a, ph, MARK_CONSUMED);
  trace_put(a, ph, SUM_WAIT, t_wait);
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
#pragma unroll
    for (int p = 1; p < kTpMaxWorld; p++)
      if (p < a.world) s += v[p];
    ll_store(dst + r, xraw[r] + s, e);
  }
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------
// Lane `lane`'s V values of one cache row (elements lane * V .. + V - 1),
// one vector load from L2.
template <int V>
__device__ __forceinline__ void load_vrow(const float* row, int lane, float* out) {
  if constexpr (V == 4) {
    const float4 t = __ldcg(reinterpret_cast<const float4*>(row) + lane);
    out[0] = t.x;
    out[1] = t.y;
    out[2] = t.z;
    out[3] = t.w;
  } else if constexpr (V == 2) {
    const float2 t = __ldcg(reinterpret_cast<const float2*>(row) + lane);
    out[0] = t.x;
    out[1] = t.y;
  } else {
    out[0] = __ldcg(row + lane);
  }
}

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

// L2 prefetch of the q/k norm gains of layer `l` (l < L): the attention
// CTAs read them on the phase's critical path.
__device__ void prefetch_gains(const MegaArgs& a, int l) {
  if (threadIdx.x != 32 || l >= a.L) return;
  const MegaLayer& ly = layer_table(a)[l];
  if (ly.q_norm) prefetch_l2(ly.q_norm, (uint32_t)a.HD * 2);
  if (ly.k_norm) prefetch_l2(ly.k_norm, (uint32_t)a.HD * 2);
}

template <int HD, int G>
constexpr int attn_floats() {
  // qs [G][HD], wm/wl [kWarps][G], wacc [kWarps][G][HD].
  return G * HD + 2 * kWarps * G + kWarps * G * HD;
}

// One attention item: kv head kh, cache split sp, at position pos. Its q,
// k and v come from the flagged qkv vector of layer l (epoch e). The split
// holding `pos` appends this step's k and v to the cache. The split record
// [m, l, acc[HD]] of each of the G query heads goes out as flagged words
// (rec vector); merge_item or merge_slice combines the records.
template <int HD, int G>
__device__ void attn_item(const MegaArgs& a, const MegaLayer& ly, int l, int kh, int sp,
                          int pos, unsigned e, float* sm, int ph) {
  constexpr int V = HD / 32;
  constexpr int QF = HD / 16;
  float* qs = sm;                      // [G][HD]
  float* wm = qs + G * HD;             // [kWarps][G]
  float* wl = wm + kWarps * G;         // [kWarps][G]
  float* wacc = wl + kWarps * G;       // [kWarps][G][HD]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t layer_off = (size_t)l * a.KHl * a.ctx * HD;
  float* kb = a.kc + layer_off + (size_t)kh * a.ctx * HD;
  float* vb = a.vc + layer_off + (size_t)kh * a.ctx * HD;
  const int s_begin = sp * a.split_len;
  const int s_end = min(s_begin + a.split_len, pos + 1);
  const u64* qkv = a.ll + a.llo.qkv + (size_t)l * a.QKVl;

  // The cache rows below `pos` were written in earlier steps (made visible
  // by the fence at the top of the step): the K rows of the warp's first 8
  // positions go into registers before the wait for this step's q, k and v.
  const int j = lane >> 2, qd = lane & 3;
  const int base0 = s_begin + warp * 8;
  float4 kv[QF];
  {
    const int s = base0 + j;
    if (s < pos) {
      const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)s * HD);
#pragma unroll
      for (int i = 0; i < QF; i++) kv[i] = __ldcg(kr + qd + 4 * i);
    }
  }
  for (int gq = warp; gq < G; gq += kWarps) {
    HeadFactors<HD> f;
    load_head_factors<HD>(a, ly.q_norm, pos, f);
    float v[V];
    ll_gather<V>(a, qkv + (size_t)(kh * G + gq) * HD, lane, 32, HD, e, v);
    head_norm_rope<HD>(a, v, ly.q_norm != nullptr, f, wacc + (size_t)gq * HD, qs + gq * HD);
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
  csync();
  trace_mark(a, ph, MARK_INPUTS);

  float m[G], lsum[G], acc[G][V];
#pragma unroll
  for (int g = 0; g < G; g++) {
    m[g] = -INFINITY;
    lsum[g] = 0.f;
#pragma unroll
    for (int v = 0; v < V; v++) acc[g][v] = 0.f;
  }
  const float div = sqrtf((float)HD);
  for (int base = base0; base < s_end; base += kPosPerPass) {
    const int s = base + j;
    const bool valid = s < s_end;
    float d[G];
#pragma unroll
    for (int g = 0; g < G; g++) d[g] = 0.f;
    // K rows not loaded yet: all of them after the first pass, the row at
    // `pos` (appended above) in the first.
    const int lo = (base == base0) ? pos : base;
    if (valid && s >= lo) {
      const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)s * HD);
#pragma unroll
      for (int i = 0; i < QF; i++) kv[i] = __ldcg(kr + qd + 4 * i);
    }
    float vv[8][V];
#pragma unroll
    for (int jj = 0; jj < 8; jj++) {
      const int sj = base + jj;
      if (sj < s_end) {
        load_vrow<V>(vb + (size_t)sj * HD, lane, vv[jj]);
      } else {
#pragma unroll
        for (int v = 0; v < V; v++) vv[jj][v] = 0.f;
      }
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
  trace_mark(a, ph, MARK_NORMED);  // attention: scores and P.V done
  csync();  // the q/k warps' scratch use of wacc is over
#pragma unroll
  for (int g = 0; g < G; g++) {
    if (lane == 0) {
      wm[warp * G + g] = m[g];
      wl[warp * G + g] = lsum[g];
    }
#pragma unroll
    for (int v = 0; v < V; v++) wacc[((size_t)warp * G + g) * HD + lane * V + v] = acc[g][v];
  }
  csync();
  // Per query head g and warp w the factor exp(m_w - M) (M the CTA's
  // maximum), once per CTA (qs is free now), then the records.
  float* cw = qs;  // [G][kWarps]
  if (tid < G * kWarps) {
    const int g = tid / kWarps, w = tid % kWarps;
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < kWarps; w2++) M = fmaxf(M, wm[w2 * G + g]);
    const float mw = wm[w * G + g];
    cw[g * kWarps + w] = (mw == -INFINITY) ? 0.f : expf(mw - M);
  }
  csync();
  // The split record of each query head, as flagged words.
  u64* rec = a.ll + a.llo.rec + (((size_t)l * a.KHl + kh) * a.nsplit + sp) * G * (HD + 2);
  for (int ei = tid; ei < G * HD; ei += kThreads) {
    const int g = ei / HD, dd = ei % HD;
    float A = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; w++)
      A = fmaf(cw[g * kWarps + w], wacc[((size_t)w * G + g) * HD + dd], A);
    u64* R = rec + (size_t)g * (HD + 2);
    if (dd == 0) {
      float M = -INFINITY, L = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) {
        M = fmaxf(M, wm[w * G + g]);
        L = fmaf(cw[g * kWarps + w], wl[w * G + g], L);
      }
      ll_store(R, M, e);
      ll_store(R + 1, L, e);
    }
    ll_store(R + 2 + dd, A, e);
  }
  trace_mark(a, ph, MARK_SCALED);  // attention: split record written
  csync();  // the scratch (qs, wm, wl, wacc) is free for the next item
  trace_mark(a, ph, MARK_STAGED);
}

// Waits for the flagged words m, l and acc[dd] of `count` split records
// (at most N) starting at base, `stride` words apart, and returns their
// values; all loads of a round go out together.
template <int N>
__device__ __forceinline__ void ll_gather_rec(const MegaArgs& a, const u64* base, int stride,
                                              int count, int dd, unsigned e, float* m, float* l,
                                              float* acc) {
  u64 w[3 * N];
#pragma unroll
  for (int u = 0; u < N; u++) {
    const u64* R = base + (size_t)u * stride;
    const bool in = u < count;
    w[3 * u] = in ? ll_load(R) : ((u64)e << 32 | __float_as_uint(-INFINITY));
    w[3 * u + 1] = in ? ll_load(R + 1) : ((u64)e << 32);
    w[3 * u + 2] = in ? ll_load(R + 2 + dd) : ((u64)e << 32);
  }
  unsigned long long pending = 0;
#pragma unroll
  for (int i = 0; i < 3 * N; i++)
    if (!ll_ready(w[i], e)) pending |= 1ull << i;
  Spin sp;
  while (pending) {
    if (!spin_on(a, sp)) break;
#pragma unroll
    for (int u = 0; u < N; u++) {
      const u64* R = base + (size_t)u * stride;
      if (pending & (1ull << (3 * u))) w[3 * u] = ll_load(R);
      if (pending & (1ull << (3 * u + 1))) w[3 * u + 1] = ll_load(R + 1);
      if (pending & (1ull << (3 * u + 2))) w[3 * u + 2] = ll_load(R + 2 + dd);
    }
#pragma unroll
    for (int i = 0; i < 3 * N; i++)
      if ((pending & (1ull << i)) && ll_ready(w[i], e)) pending &= ~(1ull << i);
  }
#pragma unroll
  for (int u = 0; u < N; u++) {
    m[u] = ll_value(w[3 * u]);
    l[u] = ll_value(w[3 * u + 1]);
    acc[u] = ll_value(w[3 * u + 2]);
  }
}

// The attention output of kv head kh (its G query heads) at position pos,
// merged by one CTA (the layout when many CTAs have no attention item: one
// of them per kv head merges, and the others do not poll):
// att = sum_j c_j acc_j / sum_j c_j l_j over the splits holding positions
// (c_j = exp(m_j - max m); splits of the kv head with positions <= pos).
// Each thread merges one output element and waits for the words of up to
// kMergeBatch splits at once; later batches rescale the running sums.
template <int HD, int G>
__device__ void merge_item(const MegaArgs& a, int l, int kh, int pos, unsigned e) {
  constexpr int kMergeBatch = 12;
  const int nact = min(a.nsplit, pos / a.split_len + 1);
  const int stride = G * (HD + 2);
  const u64* rec0 = a.ll + a.llo.rec + ((size_t)l * a.KHl + kh) * a.nsplit * stride;
  u64* att = a.ll + a.llo.att + (size_t)l * a.QHl * HD;
  for (int ei = threadIdx.x; ei < G * HD; ei += kThreads) {
    const int g = ei / HD, dd = ei % HD;
    float M = -INFINITY, Ls = 0.f, A = 0.f;
    for (int j0 = 0; j0 < nact; j0 += kMergeBatch) {
      float mj[kMergeBatch], lj[kMergeBatch], aj[kMergeBatch];
      ll_gather_rec<kMergeBatch>(a, rec0 + (size_t)j0 * stride + (size_t)g * (HD + 2), stride,
                                 nact - j0, dd, e, mj, lj, aj);
      float Mb = M;
#pragma unroll
      for (int u = 0; u < kMergeBatch; u++) Mb = fmaxf(Mb, mj[u]);
      if (Mb == -INFINITY) continue;
      if (M != -INFINITY && M != Mb) {
        const float r = expf(M - Mb);
        Ls *= r;
        A *= r;
      }
      M = Mb;
#pragma unroll
      for (int u = 0; u < kMergeBatch; u++) {
        if (mj[u] == -INFINITY) continue;
        const float c = expf(mj[u] - M);
        Ls += c * lj[u];
        A = fmaf(c, aj[u], A);
      }
    }
    ll_store(att + (size_t)(kh * G + g) * HD + dd, A / Ls, e);
  }
}

// The attention outputs att[e] for e in merge CTA mb's share of the QHl * HD
// outputs (nmerge CTAs take equal slices): att = sum_j c_j acc_j /
// sum_j c_j l_j over the splits j holding positions <= pos (c_j =
// exp(m_j - max m)). S threads share an element, each folding every S-th
// split with one round of loads (up to kMergeLoads splits per thread); the
// S partial (m, l, acc) meet in shared memory (`sm`, 3 * kThreads floats),
// where one thread per element finishes it.
template <int HD, int G>
__device__ void merge_slice(const MegaArgs& a, int l, int pos, unsigned e, float* sm, int mb,
                            int nmerge) {
  constexpr int kMergeLoads = 6;
  const int QD = a.QHl * HD;
  const int e0 = (int)((long long)QD * mb / nmerge);
  const int e1 = (int)((long long)QD * (mb + 1) / nmerge);
  const int n = e1 - e0;
  if (n <= 0) return;
  const int nact = min(a.nsplit, pos / a.split_len + 1);
  const int S = max(1, min(kThreads / n, nact));
  const int stride = G * (HD + 2);
  const int tid = threadIdx.x;
  const int el = tid / S, sub = tid % S;
  float M = -INFINITY, Ls = 0.f, A = 0.f;
  if (el < n) {
    const int ei = e0 + el;
    const int kh = ei / (G * HD), g = (ei / HD) % G, dd = ei % HD;
    const u64* R0 = a.ll + a.llo.rec + ((size_t)l * a.KHl + kh) * a.nsplit * stride +
                    (size_t)g * (HD + 2);
    for (int j0 = sub; j0 < nact; j0 += S * kMergeLoads) {
      float mj[kMergeLoads], lj[kMergeLoads], aj[kMergeLoads];
      const int cnt = min(kMergeLoads, (nact - j0 + S - 1) / S);
      ll_gather_rec<kMergeLoads>(a, R0 + (size_t)j0 * stride, S * stride, cnt, dd, e, mj, lj, aj);
#pragma unroll
      for (int u = 0; u < kMergeLoads; u++) {
        if (u >= cnt || mj[u] == -INFINITY) continue;
        const float Mn = fmaxf(M, mj[u]);
        const float r = (M == -INFINITY) ? 0.f : expf(M - Mn);
        const float c = expf(mj[u] - Mn);
        Ls = fmaf(Ls, r, c * lj[u]);
        A = fmaf(A, r, c * aj[u]);
        M = Mn;
      }
    }
  }
  sm[tid] = M;
  sm[kThreads + tid] = Ls;
  sm[2 * kThreads + tid] = A;
  csync();
  if (tid < n) {
    float Mt = -INFINITY;
    for (int s2 = 0; s2 < S; s2++) Mt = fmaxf(Mt, sm[tid * S + s2]);
    float Lt = 0.f, At = 0.f;
    for (int s2 = 0; s2 < S; s2++) {
      const float ms = sm[tid * S + s2];
      if (ms == -INFINITY) continue;
      const float c = expf(ms - Mt);
      Lt = fmaf(c, sm[kThreads + tid * S + s2], Lt);
      At = fmaf(c, sm[2 * kThreads + tid * S + s2], At);
    }
    u64* att = a.ll + a.llo.att + (size_t)l * QD;
    ll_store(att + e0 + tid, At / Lt, e);
  }
  csync();  // sm is free again
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int HD, int G, bool MOE>
__global__ void __launch_bounds__(kBlockThreads, 1)
    k_mega_decode(const __grid_constant__ MegaArgs a) {
  char* dyn = s_dyn;
  const int buf_bytes = a.buf_bytes, nbuf = a.nbuf, parts = a.parts;
  __shared__ float red[32];
  __shared__ float cbest_v[kWarps];
  __shared__ int cbest_i[kWarps];
  __shared__ __align__(8) uint64_t gain_bar[1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D32 = (a.D + 31) / 32 * 32;
  float* xraw = reinterpret_cast<float*>(dyn + (size_t)nbuf * buf_bytes);  // [D]
  uint16_t* gain_buf = reinterpret_cast<uint16_t*>(xraw + D32);              // [D]
  // MoE: the xm region (expert inputs as f16 parts: the normalised x, then
  // the selected experts' SwiGLU outputs [topk][Fe]).
  float* xf = reinterpret_cast<float*>(gain_buf + D32);
  uint8_t* xm = reinterpret_cast<uint8_t*>(xf);
  // Matvec input (bf16 parts) or attention scratch (floats).
  float* xs = xf + (MOE ? moe_xf_floats(a.D, a.topk, a.Fe) : 0);
  uint16_t* xq = reinterpret_cast<uint16_t*>(xs);
  __shared__ int s_csel[kMaxTopk];
  __shared__ float s_cselw[kMaxTopk];
  for (int i = threadIdx.x; i < a.L; i += kBlockThreads) layer_table(a)[i] = a.layers[i];
  if (threadIdx.x == 0) {
    for (int i = 0; i < nbuf; i++) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kWarps);
    }
    mbar_init(&gain_bar[0], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x < kKinds) {
    // Layer 0's phases stand for every layer (same shapes); kinds the model
    // does not have get no chunks.
    const int k = threadIdx.x, P = phases_per_layer<MOE>(a);
    int wp = -1;
    if (k == W_LM)
      wp = P * a.L;
    else if (k == W_QKV || k == W_O)
      wp = k;
    else if (!MOE && (k == W_GU || k == W_DOWN))
      wp = k;
    else if (MOE && k >= W_ROUTER)
      wp = k - W_ROUTER + 2;
    if (wp >= 0) {
      s_slices[k] = cta_slice(weight_phase<MOE>(a, wp), buf_bytes, a.topk, a.Fe);
    } else {
      Slice z = {0, 0, 2, 0, 1, 0};
      s_slices[k] = z;
    }
  }
  __syncthreads();
  if (warp == kWarps) {
    produce<MOE>(a, dyn, buf_bytes, nbuf, s_full, s_empty);
    return;
  }
  Ring r;
  r.g = 0;
  r.nred = 0;
  r.b = 0;
  r.par = 0;
  Gains gs;
  gs.buf = gain_buf;
  gs.bar = gain_bar;
  gs.n = 0;
  gains_fill(gs, layer_table(a)[0].attn_norm, a.D);
  int ph = 0;  // phase counter (trace only)
  int pos = __ldcg(a.pos);
  int token = __ldcg(a.tok);
  int step = __ldcg(a.step);
  const int QD = a.QHl * a.HD;
  const int P = phases_per_layer<MOE>(a);
  const int attn_items = a.KHl * a.nsplit;
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  u64* am = a.ll + a.llo.am;
  const int nam = a.world * (int)gridDim.x;  // argmax partials of all ranks

  prefetch_kv<HD>(a, 0, pos);
  for (int s = 0; s < a.steps; s++) {
    const unsigned e = a.epoch + (unsigned)s;
    for (int l = 0; l < a.L; l++) {
      const MegaLayer& ly = layer_table(a)[l];
      u64* x_o = a.ll + a.llo.x + (size_t)l * 2 * a.D;  // after o_proj
      u64* x_d = x_o + a.D;                              // after down
      // QKV
      trace_mark(a, ph, MARK_BEGIN);
      // The next layer's cache rows, a layer ahead of their use (this
      // layer's were requested during the previous one).
      if (l + 1 < a.L)
        prefetch_kv<HD>(a, l + 1, pos);
      else if (s + 1 < a.steps)
        prefetch_kv<HD>(a, 0, pos + 1);
      prefetch_gains(a, l + 1);
      if (l == 0)
        stage_embedding(a, token, gs, xq, parts, xraw, red);
      else
        stage_norm_ll(a, x_o - 2 * (size_t)a.D + a.D, e, gs, a.D, xq, parts, xraw, red, ph);
      gains_fill(gs, ly.ffn_norm, a.D);
      consume_phase<MOE, W_QKV>(a, r, P * l + 0, xq, parts,
                    Out{a.ll + a.llo.qkv + (size_t)l * a.QKVl, nullptr, e}, bv, bi, ph);
      ph++;
      // ATTN
      trace_mark(a, ph, MARK_BEGIN);
      for (int it = blockIdx.x; it < attn_items; it += gridDim.x)
        attn_item<HD, G>(a, ly, l, it % a.KHl, it / a.KHl, pos, e, xs, ph);
      // The split records: when at least KHl CTAs have no attention item,
      // one such CTA per kv head merges them (few CTAs poll while the
      // items run); otherwise every CTA merges an equal slice of the
      // outputs once its own item is done.
      if ((int)gridDim.x - attn_items >= a.KHl) {
        for (int kh = 0; kh < a.KHl; kh++)
          if (attn_items + kh == (int)blockIdx.x) merge_item<HD, G>(a, l, kh, pos, e);
      } else {
        merge_slice<HD, G>(a, l, pos, e, xs, (int)blockIdx.x, (int)gridDim.x);
      }
      trace_mark(a, ph, MARK_READY);
      ph++;
      // O + residual
      trace_mark(a, ph, MARK_BEGIN);
      stage_plain_ll(a, a.ll + a.llo.att + (size_t)l * QD, e, QD, xq, parts, ph);
      {
        const size_t part0 = a.llo.xpart + (size_t)(l * 2 + 0) * a.world * a.D;
        consume_phase<MOE, W_O>(a, r, P * l + 1, xq, parts,
                      Out{x_o, xraw, e, part0 + (size_t)a.rank * a.D}, bv, bi, ph);
        if (a.world > 1)
          tp_reduce_rows(a, xraw, part0, x_o, s_slices[W_O].rb, s_slices[W_O].re, e);
      }
      ph++;
      // FFN input: RMSNorm of x_o (for MoE also as f16 parts in xm)
      trace_mark(a, ph, MARK_BEGIN);
      stage_norm_ll(a, x_o, e, gs, a.D, xq, parts, xraw, red, ph, MOE ? xm : nullptr);
      gains_fill(gs, l + 1 < a.L ? layer_table(a)[l + 1].attn_norm : a.out_norm, a.D);
      const size_t part_d = a.llo.xpart + (size_t)(l * 2 + 1) * a.world * a.D;
      if constexpr (MOE) {
        // router logits, then every CTA picks the experts
        consume_phase<MOE, W_ROUTER>(a, r, P * l + 2, xq, parts,
                      Out{a.ll + a.llo.rl + (size_t)l * a.E, nullptr, e}, bv, bi, ph);
        if (warp == 0) expert_select(a, l, e, s_csel, s_cselw);
        csync();
        ph++;
        // gate/up + SwiGLU of the selected experts
        trace_mark(a, ph, MARK_BEGIN);
        consume_mx_gu(a, r, l, xm, s_csel, e, ph);
        ph++;
        // down of the selected experts, weighted sum + residual
        trace_mark(a, ph, MARK_BEGIN);
        stage_moe_h(a, l, e, s_csel, xm, ph);
        consume_mx_down(a, r, xm, s_csel, s_cselw,
                        Out{x_d, xraw, e, part_d + (size_t)a.rank * a.D}, bv, bi, ph);
        if (a.world > 1)
          tp_reduce_rows(a, xraw, part_d, x_d, s_slices[W_EDOWN].rb, s_slices[W_EDOWN].re, e);
        ph++;
      } else {
        // gate/up + SwiGLU
        consume_phase<MOE, W_GU>(a, r, P * l + 2, xq, parts,
                      Out{a.ll + a.llo.h + (size_t)l * a.Fl, nullptr, e}, bv, bi, ph);
        ph++;
        // down + residual
        trace_mark(a, ph, MARK_BEGIN);
        stage_plain_ll(a, a.ll + a.llo.h + (size_t)l * a.Fl, e, a.Fl, xq, parts, ph);
        consume_phase<MOE, W_DOWN>(a, r, P * l + 3, xq, parts,
                      Out{x_d, xraw, e, part_d + (size_t)a.rank * a.D}, bv, bi, ph);
        if (a.world > 1)
          tp_reduce_rows(a, xraw, part_d, x_d, s_slices[W_DOWN].rb, s_slices[W_DOWN].re, e);
        ph++;
      }
    }
    // LM head with per-CTA argmax
    trace_mark(a, ph, MARK_BEGIN);
    stage_norm_ll(a, a.ll + a.llo.x + (size_t)(a.L - 1) * 2 * a.D + a.D, e, gs, a.D, xq, parts,
                  xraw, red, ph);
    if (s + 1 < a.steps) gains_fill(gs, layer_table(a)[0].attn_norm, a.D);
    bv = -INFINITY;
    bi = 0x7FFFFFFF;
    consume_phase<MOE, W_LM>(a, r, P * a.L, xq, parts, Out{nullptr, nullptr, e}, bv, bi, ph);
    // Warp argmax (ties: lower index), then the warps' in order.
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int i2 = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (v2 > bv || (v2 == bv && i2 < bi)) {
        bv = v2;
        bi = i2;
      }
    }
    if (lane == 0) {
      cbest_v[warp] = bv;
      cbest_i[warp] = bi;
    }
    csync();
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
    csync();
    token = cbest_i[0];
    // Every CTA has published its partial after writing this step's K/V
    // rows (and a fence): the next step's attention reads them after this
    // one.
    __threadfence();
    if (blockIdx.x == 0 && threadIdx.x == 0 && step >= 0 && step < a.gen_len)
      a.gen[step] = token;
    step++;
    pos++;
    csync();
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *a.tok = token;
    *a.pos = pos;
    *a.step = step;
  }
}

template <int HD, int G>
void* kernel_ptr(bool moe) {
  return moe ? (void*)k_mega_decode<HD, G, true> : (void*)k_mega_decode<HD, G, false>;
}

void* select(int HD, int G, bool moe = false) {
#define SG_SEL(h, g) \
  if (HD == h && G == g) return kernel_ptr<h, g>(moe);
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
// (rounded to 32 floats), one bf16 gain vector [D] (same rounding), then
// the matvec input (`parts` bf16 arrays of K + 32 columns), the attention
// scratch or the attention merge's partials (3 floats per thread).

size_t act_core_bytes(int D, int QD, int Fl, int HD, int G, int parts, int xf_floats) {
  const size_t kmax = (size_t)std::max(D, std::max(QD, Fl));
  size_t bytes = std::max((size_t)parts * 2 * (kmax + 32), select_attn_floats(HD, G) * 4);
  bytes = std::max(bytes, (size_t)3 * kThreads * 4);  // the attention merge's partials
  bytes += (size_t)(D + 31) / 32 * 32 * (4 + 2);  // xraw, the gain vector
  bytes += (size_t)xf_floats * 4;
  return (bytes + 127) / 128 * 128;
}

// ... then the layer table (L entries).
size_t act_bytes(int D, int QD, int Fl, int HD, int G, int parts, int xf_floats, int L) {
  return act_core_bytes(D, QD, Fl, HD, G, parts, xf_floats) +
         ((size_t)L * sizeof(MegaLayer) + 127) / 128 * 128;
}

// Dynamic shared memory a CTA may take: the device's opt-in limit less the
// kernel's static shared memory, rounded down to 1 KB.
size_t smem_budget(int HD, int G) {
  static size_t cached[3][4] = {};
  const int hi = HD == 32 ? 0 : HD == 64 ? 1 : 2;
  const int gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
  if (!cached[hi][gi]) {
    cudaFuncAttributes fa, fm;
    SG_CUDA(cudaFuncGetAttributes(&fa, select(HD, G, false)));
    SG_CUDA(cudaFuncGetAttributes(&fm, select(HD, G, true)));
    fa.sharedSizeBytes = std::max(fa.sharedSizeBytes, fm.sharedSizeBytes);
    int dev = 0, optin = 0;
    SG_CUDA(cudaGetDevice(&dev));
    SG_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    const size_t lim = (size_t)optin > fa.sharedSizeBytes ? (size_t)optin - fa.sharedSizeBytes : 0;
    cached[hi][gi] = lim / 1024 * 1024;
  }
  return cached[hi][gi];
}

// Weight buffers of the ring (STRASGPT_MEGA_RING, 2..4; default 2).
int ring_count() {
  static int n = 0;
  if (!n) {
    const char* v = getenv("STRASGPT_MEGA_RING");
    n = v ? atoi(v) : 2;
    if (n < 2) n = 2;
    if (n > kMaxRing) n = kMaxRing;
  }
  return n;
}

// Three activation parts (fp32-faithful) when the weight ring keeps at
// least 112 KB; two (x to about 2^-17, as in the tensor-core prefill)
// otherwise, so that large models keep enough weight bytes in flight.
// STRASGPT_MEGA_PARTS=2 or 3 overrides the choice (when the ring still
// fits).
int act_parts(int D, int QD, int Fl, int HD, int G, int xf, int L) {
  const char* v = getenv("STRASGPT_MEGA_PARTS");
  if (v && (atoi(v) == 2 || atoi(v) == 3) &&
      act_bytes(D, QD, Fl, HD, G, atoi(v), xf, L) + (size_t)ring_count() * 16 * 1024 <=
          smem_budget(HD, G))
    return atoi(v);
  return act_bytes(D, QD, Fl, HD, G, 3, xf, L) + (size_t)112 * 1024 <= smem_budget(HD, G) ? 3
                                                                                           : 2;
}

// dst[r][0 .. src_bytes) = src[r][...], dst[r][src_bytes .. dst_bytes) = 0.
__global__ void k_pad_rows(const uint8_t* __restrict__ src, size_t rows, int src_bytes,
                           int dst_bytes, uint8_t* __restrict__ dst) {
  const size_t n = rows * (size_t)dst_bytes;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / dst_bytes;
    const int c = (int)(i % dst_bytes);
    dst[i] = c < src_bytes ? src[r * src_bytes + c] : 0;
  }
}

}  // namespace

void mega_pad_rows(const uint8_t* src, size_t rows, int src_bytes, int dst_bytes, uint8_t* dst,
                   cudaStream_t s) {
  if (rows == 0) return;
  const size_t n = rows * (size_t)dst_bytes;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 16);
  k_pad_rows<<<blocks, 256, 0, s>>>(src, rows, src_bytes, dst_bytes, dst);
  SG_CUDA(cudaGetLastError());
}

int mega_scale_row_bytes(int K) { return mx_scale_bytes(K); }

MegaFlagged mega_flagged_layout(int D, int QKVl, int QD, int Fl, int L, int grid, int world,
                                int nsplit, int HD, int E, int topk, int Fe) {
  MegaFlagged f;
  f.x = 0;
  f.qkv = f.x + (size_t)L * 2 * D;
  f.att = f.qkv + (size_t)L * QKVl;
  f.h = f.att + (size_t)L * QD;
  f.xpart = f.h + (size_t)L * Fl;
  f.am = f.xpart + (world > 1 ? (size_t)L * 2 * world * D : 0);
  f.rec = f.am + 2 * (size_t)world * grid;
  // QD / HD query heads, each with one record per split.
  f.rl = f.rec + (size_t)L * (QD / HD) * nsplit * (HD + 2);
  f.hm = f.rl + (size_t)L * E;
  f.total = f.hm + (size_t)L * topk * Fe;
  return f;
}

// Ring buffers take what the activations leave of the budget. Every row
// length (D, QD, Fl) must be a multiple of 32 columns.
size_t mega_smem_bytes(int D, int QD, int Fl, int HD, int G, int L, int topk, int Fe) {
  if (!select(HD, G)) return 0;
  if (D > kNormMaxK || L > kMaxLayers) return 0;
  if (D % 32 || QD % 32 || Fl % 32 || Fe % 32) return 0;
  const int xf = moe_xf_floats(D, topk, Fe);
  const size_t act = act_bytes(D, QD, Fl, HD, G, act_parts(D, QD, Fl, HD, G, xf, L), xf, L);
  const size_t budget = smem_budget(HD, G);
  const int nbuf = ring_count();
  if (act + (size_t)nbuf * 16 * 1024 > budget) return 0;
  size_t buf = (budget - act) / nbuf / 1024 * 1024;
  return (size_t)nbuf * buf + act;
}

static int buffer_bytes(size_t smem, int D, int QD, int Fl, int HD, int G, int xf, int L) {
  return (int)((smem - act_bytes(D, QD, Fl, HD, G, act_parts(D, QD, Fl, HD, G, xf, L), xf, L)) /
               ring_count());
}

void mega_configure(size_t smem) {
  for (int hd : {32, 64, 128})
    for (int g : {1, 2, 4, 8})
      for (bool moe : {false, true})
        SG_CUDA(cudaFuncSetAttribute(select(hd, g, moe),
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)std::max(smem, (size_t)48 * 1024)));
}

int mega_grid(size_t smem, int HD, int G) {
  void* k = select(HD, G);
  if (!k || smem == 0) return 0;
  for (bool moe : {false, true}) {
    int per_sm = 0;
    SG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, select(HD, G, moe),
                                                          kBlockThreads, smem));
    if (per_sm < 1) return 0;
  }
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
  void* k = select(a.HD, a.G, a.moe != 0);
  if (!k) SG_DIE("megakernel: unsupported head_dim / group");
  if (a.nsplit > kMaxSplits) SG_DIE("megakernel: too many attention splits");
  if (a.L > kMaxLayers) SG_DIE("megakernel: too many layers");
  const int xf = moe_xf_floats(a.D, a.moe ? a.topk : 0, a.Fe);
  int buf = buffer_bytes(smem, a.D, a.QHl * a.HD, a.Fl, a.HD, a.G, xf, a.L);
  if (buf < 16 * 1024 || buf % 1024) SG_DIE("megakernel: weight buffers too small");
  if (a.moe && (a.topk < 1 || a.topk > kMaxTopk || a.E > 128 || a.E % 2))
    SG_DIE("megakernel: unsupported expert count / top-k");
  if (a.moe && 2 * mx_row_bytes(std::max(a.D, a.Fe)) > buf)
    SG_DIE("megakernel: weight buffers too small for two expert rows");
  int parts = act_parts(a.D, a.QHl * a.HD, a.Fl, a.HD, a.G, xf, a.L);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kBlockThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int nbuf = ring_count();
  MegaArgs ak = a;
  ak.buf_bytes = buf;
  ak.nbuf = nbuf;
  ak.layers_off = (long long)nbuf * buf +
                  (long long)act_core_bytes(a.D, a.QHl * a.HD, a.Fl, a.HD, a.G, parts, xf);
  ak.parts = parts;
  void* args[] = {(void*)&ak};
  SG_CUDA(cudaLaunchKernelExC(&cfg, k, args));
}

}  // namespace sg
