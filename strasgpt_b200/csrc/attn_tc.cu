// Causal GQA attention of a prefill chunk on the tensor cores
// (source/transformer.c:1375-1422: s = q.k / sqrtf(HD) over positions
// [0, pos], max-subtracted expf softmax, att = sum p v).
//
// One CTA = one kv head and 64 rows, a row being one (query, q head of the
// group) pair (64 / G queries x G heads), so every K/V tile is shared by the
// whole group. Four warps, 16 rows each. The reference's operands are fp32;
// the tensor cores take bf16, so each operand is split as x = hi + lo
// (hi = bf16(x), lo = bf16(x - hi), about 17 significant bits, as in the
// tensor-core projections) and every product takes three mma.sync
// m16n8k16 (hi.hi + hi.lo + lo.hi) with fp32 accumulators:
//   S = Q K^T   Q fragments from shared memory (ldmatrix), K rows as the
//               col-major B operand (ldmatrix of [key][hd] tiles);
//   online softmax on the S accumulators (rows g and g + 8 of a lane);
//   O += P V    P re-packed from the S accumulators into A fragments, V as
//               the B operand (ldmatrix.trans of [key][hd] tiles).
// K/V tiles of kKeysTc keys are read from the fp32 cache, split and stored in
// shared memory with rows padded by 16 bytes (conflict-free ldmatrix).
#include "common.cuh"
#include "kernels.h"

#include <math.h>

namespace sg {
namespace {

constexpr int kRowsTc = 64;  // rows per CTA
constexpr int kKeysTc = 32;  // keys per tile (two CTAs fit on an SM)
constexpr int kKT8 = kKeysTc / 8;    // n8 tiles of S
constexpr int kKT16 = kKeysTc / 16;  // k16 steps of P.V

template <int HD>
struct TcAttn {
  static constexpr int LD = HD + 8;  // bf16 elements per shared-memory row
  // bf16 Q hi/lo, K hi/lo, V hi/lo, then the fp32 K and V rows of the next
  // tile (filled by cp.async while the current tile is multiplied).
  static constexpr size_t kBf16Bytes = (size_t)(2 * kRowsTc + 4 * kKeysTc) * LD * 2;
  static constexpr size_t kBytes = kBf16Bytes + (size_t)2 * kKeysTc * HD * 4;
};

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Two fp32 values -> their bf16 (round to nearest even) hi halves and the
// bf16 of what they leave (lo), each pair packed as one word, x0 in the low
// 16 bits (the hardware conversion cvt.rn.bf16x2.f32 puts its first source
// in the high half).
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
  const float r0 = x0 - __uint_as_float(hi << 16);
  const float r1 = x1 - __uint_as_float(hi & 0xFFFF0000u);
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r1), "f"(r0));
}

// Four fp32 values -> hi and lo halves as 8-byte stores.
__device__ __forceinline__ void store_split4(uint16_t* hi, uint16_t* lo, float4 v) {
  uint32_t h0, h1, l0, l1;
  split_pair(v.x, v.y, h0, l0);
  split_pair(v.z, v.w, h1, l1);
  *reinterpret_cast<uint2*>(hi) = make_uint2(h0, h1);
  *reinterpret_cast<uint2*>(lo) = make_uint2(l0, l1);
}

// 16-byte asynchronous copy global -> shared; src_bytes 0 fills zeros.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
__global__ void __launch_bounds__(128) k_attn_prefill_tc(AttnPrefillArgs a) {
  constexpr int LD = TcAttn<HD>::LD;
  constexpr int KS = HD / 16;  // k16 steps of q.k
  constexpr int NH = HD / 8;   // n8 tiles of the output
  extern __shared__ __align__(16) uint16_t sm[];
  uint16_t* Qh = sm;
  uint16_t* Ql = Qh + kRowsTc * LD;
  uint16_t* Kh = Ql + kRowsTc * LD;
  uint16_t* Kl = Kh + kKeysTc * LD;
  uint16_t* Vh = Kl + kKeysTc * LD;
  uint16_t* Vl = Vh + kKeysTc * LD;
  float* Kraw = reinterpret_cast<float*>(Vl + kKeysTc * LD);  // [kKeysTc][HD]
  float* Vraw = Kraw + kKeysTc * HD;
  const int kh = blockIdx.x, G = a.G, qt = kRowsTc / G, t0 = blockIdx.y * qt;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, c = lane & 3;
  constexpr int kVecPerThread = kKeysTc * (HD / 4) / 128;  // float4 per thread per tile
  pdl_trigger();
  pdl_wait();

  const int tl = min(t0 + qt, a.T) - 1;
  const int kend = a.pos0 + tl + 1;  // keys [0, kend) for this CTA
  const float* kbase = a.k_cache + (size_t)kh * a.ctx * HD;
  const float* vbase = a.v_cache + (size_t)kh * a.ctx * HD;
  // fp32 K and V rows [k0, k0 + kKeysTc) -> Kraw, Vraw (zeros past kend).
  auto fetch = [&](int k0) {
#pragma unroll
    for (int u = 0; u < kVecPerThread; u++) {
      const int i = tid + u * 128;
      const int key = i / (HD / 4), d4 = i % (HD / 4);
      const bool in = k0 + key < kend;
      const size_t off = in ? (size_t)(k0 + key) * HD + d4 * 4 : 0;
      cp_async16(Kraw + key * HD + d4 * 4, kbase + off, in ? 16 : 0);
      cp_async16(Vraw + key * HD + d4 * 4, vbase + off, in ? 16 : 0);
    }
    cp_async_commit();
  };
  fetch(0);

  // Q tile: row r = (query t0 + r / G, head r % G); all loads of a batch
  // go out before the values are split.
  const float4* q4 = reinterpret_cast<const float4*>(a.q);
  constexpr int kQBatch = 8;
  for (int i0 = tid; i0 < kRowsTc * (HD / 4); i0 += kQBatch * 128) {
    float4 v[kQBatch];
#pragma unroll
    for (int u = 0; u < kQBatch; u++) {
      const int i = i0 + u * 128;
      const int r = i / (HD / 4), d4 = i % (HD / 4);
      const int t = t0 + r / G, g = r % G;
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < kRowsTc * (HD / 4) && t < a.T)
        v[u] = q4[((size_t)(t * a.KHl + kh) * G + g) * (HD / 4) + d4];
    }
#pragma unroll
    for (int u = 0; u < kQBatch; u++) {
      const int i = i0 + u * 128;
      if (i < kRowsTc * (HD / 4)) {
        const int r = i / (HD / 4), d4 = i % (HD / 4);
        store_split4(Qh + r * LD + d4 * 4, Ql + r * LD + d4 * 4, v[u]);
      }
    }
  }

  // This lane's rows (g8 and g8 + 8 of the warp's 16) and their positions.
  const int rA = 16 * warp + g8, rB = rA + 8;
  const int tA = t0 + rA / G, tB = t0 + rB / G;
  const int posA = (tA < a.T) ? a.pos0 + tA : -1;  // -1: no keys
  const int posB = (tB < a.T) ? a.pos0 + tB : -1;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  float o[NH][4];
#pragma unroll
  for (int n = 0; n < NH; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const float div = sqrtf((float)HD);

  // ldmatrix lane addresses (element offsets within a tile):
  //  A (Q rows of this warp): row (lane % 16), column 8 (lane / 16);
  //  B (K, two n8 tiles): key (lane % 8) + 8 (lane / 16), column 8 ((lane / 8) % 2);
  //  B (V, transposed, two n8 tiles): key (lane % 8) + 8 ((lane / 8) % 2), column 8 (lane / 16).
  const int qoff = (16 * warp + (lane & 15)) * LD + (lane >> 4) * 8;
  const int koff = ((lane & 7) + (lane >> 4) * 8) * LD + ((lane >> 3) & 1) * 8;
  const int voff = ((lane & 7) + ((lane >> 3) & 1) * 8) * LD + (lane >> 4) * 8;

  for (int k0 = 0; k0 < kend; k0 += kKeysTc) {
    // This tile's fp32 rows have landed (each thread waits for its own
    // copies; the barrier makes all of them visible) and the previous
    // tile's bf16 K and V are consumed.
    cp_async_wait_all();
    __syncthreads();
#pragma unroll 4
    for (int u = 0; u < kVecPerThread; u++) {
      const int i = tid + u * 128;
      const int key = i / (HD / 4), d4 = i % (HD / 4);
      const float4 kv = *reinterpret_cast<const float4*>(Kraw + key * HD + d4 * 4);
      const float4 vv = *reinterpret_cast<const float4*>(Vraw + key * HD + d4 * 4);
      store_split4(Kh + key * LD + d4 * 4, Kl + key * LD + d4 * 4, kv);
      store_split4(Vh + key * LD + d4 * 4, Vl + key * LD + d4 * 4, vv);
    }
    __syncthreads();
    // The next tile's rows stream in while this one is multiplied.
    if (k0 + kKeysTc < kend) fetch(k0 + kKeysTc);

    // S = Q K^T: 16 rows x kKeysTc keys per warp (kKT8 n8 tiles).
    float s[kKT8][4];
#pragma unroll
    for (int n = 0; n < kKT8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
    // Per k16 step: every fragment first, then the three products of all
    // tiles in turn (kKT8 independent accumulation chains).
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
      uint32_t ah[4], al[4], bh[kKT16][4], bl[kKT16][4];
      ldsm4(saddr(Qh + qoff + ks * 16), ah);
      ldsm4(saddr(Ql + qoff + ks * 16), al);
#pragma unroll
      for (int n = 0; n < kKT16; n++) {
        ldsm4(saddr(Kh + koff + n * 16 * LD + ks * 16), bh[n]);
        ldsm4(saddr(Kl + koff + n * 16 * LD + ks * 16), bl[n]);
      }
#pragma unroll
      for (int n = 0; n < kKT16; n++) {
        mma(s[2 * n], ah, bh[n][0], bh[n][1]);
        mma(s[2 * n + 1], ah, bh[n][2], bh[n][3]);
      }
#pragma unroll
      for (int n = 0; n < kKT16; n++) {
        mma(s[2 * n], ah, bl[n][0], bl[n][1]);
        mma(s[2 * n + 1], ah, bl[n][2], bl[n][3]);
      }
#pragma unroll
      for (int n = 0; n < kKT16; n++) {
        mma(s[2 * n], al, bh[n][0], bh[n][1]);
        mma(s[2 * n + 1], al, bh[n][2], bh[n][3]);
      }
    }

    // Scale, causal mask, online softmax (rows A and B of this lane; the
    // four lanes of a row hold its kKeysTc keys).
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int n = 0; n < kKT8; n++) {
      const int key = k0 + n * 8 + 2 * c;
      s[n][0] = (key <= posA) ? s[n][0] / div : -INFINITY;
      s[n][1] = (key + 1 <= posA) ? s[n][1] / div : -INFINITY;
      s[n][2] = (key <= posB) ? s[n][2] / div : -INFINITY;
      s[n][3] = (key + 1 <= posB) ? s[n][3] / div : -INFINITY;
      mxA = fmaxf(mxA, fmaxf(s[n][0], s[n][1]));
      mxB = fmaxf(mxB, fmaxf(s[n][2], s[n][3]));
    }
    mxA = fmaxf(mxA, __shfl_xor_sync(0xFFFFFFFFu, mxA, 1));
    mxA = fmaxf(mxA, __shfl_xor_sync(0xFFFFFFFFu, mxA, 2));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xFFFFFFFFu, mxB, 1));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xFFFFFFFFu, mxB, 2));
    const float nA = fmaxf(mA, mxA), nB = fmaxf(mB, mxB);
    // A row with no key so far keeps m = -inf and contributes nothing.
    const float cA = (nA == -INFINITY) ? 1.f : expf(mA - nA);
    const float cB = (nB == -INFINITY) ? 1.f : expf(mB - nB);
    mA = nA;
    mB = nB;
    lA *= cA;
    lB *= cB;
#pragma unroll
    for (int n = 0; n < NH; n++) {
      o[n][0] *= cA;
      o[n][1] *= cA;
      o[n][2] *= cB;
      o[n][3] *= cB;
    }
#pragma unroll
    for (int n = 0; n < kKT8; n++) {
      s[n][0] = (s[n][0] == -INFINITY) ? 0.f : expf(s[n][0] - nA);
      s[n][1] = (s[n][1] == -INFINITY) ? 0.f : expf(s[n][1] - nA);
      s[n][2] = (s[n][2] == -INFINITY) ? 0.f : expf(s[n][2] - nB);
      s[n][3] = (s[n][3] == -INFINITY) ? 0.f : expf(s[n][3] - nB);
      lA += s[n][0] + s[n][1];
      lB += s[n][2] + s[n][3];
    }

    // O += P V: k16 step j = keys 16 j .. 16 j + 15 (S tiles 2j, 2j + 1).
#pragma unroll
    for (int j = 0; j < kKT16; j++) {
      uint32_t ph[4], pl[4];
      split_pair(s[2 * j][0], s[2 * j][1], ph[0], pl[0]);
      split_pair(s[2 * j][2], s[2 * j][3], ph[1], pl[1]);
      split_pair(s[2 * j + 1][0], s[2 * j + 1][1], ph[2], pl[2]);
      split_pair(s[2 * j + 1][2], s[2 * j + 1][3], ph[3], pl[3]);
      // Output tiles in groups of eight: fragments first, then the three
      // products of the group in turn.
#pragma unroll
      for (int n0 = 0; n0 < NH; n0 += 8) {
        constexpr int kPairs = (NH < 8 ? NH : 8) / 2;
        uint32_t bh[kPairs][4], bl[kPairs][4];
#pragma unroll
        for (int q = 0; q < kPairs; q++) {
          ldsm4t(saddr(Vh + voff + j * 16 * LD + (n0 + 2 * q) * 8), bh[q]);
          ldsm4t(saddr(Vl + voff + j * 16 * LD + (n0 + 2 * q) * 8), bl[q]);
        }
#pragma unroll
        for (int q = 0; q < kPairs; q++) {
          mma(o[n0 + 2 * q], ph, bh[q][0], bh[q][1]);
          mma(o[n0 + 2 * q + 1], ph, bh[q][2], bh[q][3]);
        }
#pragma unroll
        for (int q = 0; q < kPairs; q++) {
          mma(o[n0 + 2 * q], ph, bl[q][0], bl[q][1]);
          mma(o[n0 + 2 * q + 1], ph, bl[q][2], bl[q][3]);
        }
#pragma unroll
        for (int q = 0; q < kPairs; q++) {
          mma(o[n0 + 2 * q], pl, bh[q][0], bh[q][1]);
          mma(o[n0 + 2 * q + 1], pl, bh[q][2], bh[q][3]);
        }
      }
    }
  }

  // Row sums over the four lanes of a row, then att = O / l.
  lA += __shfl_xor_sync(0xFFFFFFFFu, lA, 1);
  lA += __shfl_xor_sync(0xFFFFFFFFu, lA, 2);
  lB += __shfl_xor_sync(0xFFFFFFFFu, lB, 1);
  lB += __shfl_xor_sync(0xFFFFFFFFu, lB, 2);
  const int gA = rA % G, gB = rB % G;
  if (tA < a.T) {
    float* out = a.att + ((size_t)(tA * a.KHl + kh) * G + gA) * HD;
#pragma unroll
    for (int n = 0; n < NH; n++)
      *reinterpret_cast<float2*>(out + n * 8 + 2 * c) = make_float2(o[n][0] / lA, o[n][1] / lA);
  }
  if (tB < a.T) {
    float* out = a.att + ((size_t)(tB * a.KHl + kh) * G + gB) * HD;
#pragma unroll
    for (int n = 0; n < NH; n++)
      *reinterpret_cast<float2*>(out + n * 8 + 2 * c) = make_float2(o[n][2] / lB, o[n][3] / lB);
  }
}

template <int HD>
void launch_hd(const AttnPrefillArgs& a, cudaStream_t s) {
  const int qt = kRowsTc / a.G;
  dim3 grid(a.KHl, (a.T + qt - 1) / qt);
  launch(k_attn_prefill_tc<HD>, grid, dim3(128), TcAttn<HD>::kBytes, s, a);
}

}  // namespace

bool attn_prefill_tc_supported(const AttnPrefillArgs& a) {
  return (a.HD == 32 || a.HD == 64 || a.HD == 128) && a.G >= 1 && a.G <= kRowsTc &&
         kRowsTc % a.G == 0;
}

void attn_prefill_tc(const AttnPrefillArgs& a, cudaStream_t s) {
  if (!attn_prefill_tc_supported(a)) SG_DIE("attn_prefill_tc: unsupported head_dim / group");
  if (a.HD == 128)
    launch_hd<128>(a, s);
  else if (a.HD == 64)
    launch_hd<64>(a, s);
  else
    launch_hd<32>(a, s);
}

void attn_prefill_tc_configure() {
  SG_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)TcAttn<32>::kBytes));
  SG_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)TcAttn<64>::kBytes));
  SG_CUDA(cudaFuncSetAttribute(k_attn_prefill_tc<128>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)TcAttn<128>::kBytes));
}

}  // namespace sg
