// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMA).
//
// C[t][r] (op)= sum_k A[t][k] W[r][k] for a chunk of T tokens, with fp32
// activations A and bf16 weights W, accumulated in fp32. The tensor cores
// take bf16 operands, so the activations are split on the way in:
// A = A_hi + A_lo with A_hi = bf16(A), A_lo = bf16(A - A_hi), which keeps
// about 16 bits of A (relative error <= 2^-17) while every product stays
// exact in fp32. Each 16-wide K step is one MMA of N = 2*BN: the A_hi and
// A_lo tiles are adjacent in shared memory and form a single operand, so
// the weight tile is read once; the epilogue adds the two accumulator
// halves.
//
// Tile: 128 weight rows (MMA M) x BN tokens (BN = 32, 64 or 128), K in
// steps of 64 (one 128-byte swizzle row). A ring of stages of
// {W, A_hi, A_lo} tiles filled by TMA with 128-byte swizzling; the fp32
// accumulators live in tensor memory (2*BN columns). The stage ring is
// bound by TMA latency, so the host picks BN to minimise waves x bytes per
// stage (few weight-row tiles: narrow token tiles and more CTAs; many: wide
// tiles and fewer bytes per MMA).
// Warp roles (6 warps): 0 TMA producer, 1 MMA issuer (one elected thread
// each), 2..5 epilogue (each reads the 32 TMEM lanes of its quarter with
// tcgen05.ld, applies STORE / ADD / SwiGLU and writes C coalesced along r).
// Launched with programmatic dependent launch: for weights no earlier kernel
// writes, the tiles of the first stages are requested before
// griddepcontrol.wait, i.e. while the kernel that produces the activations
// is still finishing.
// Every wait is bounded: a timeout sets *err and the CTA finishes without
// touching C further; the host reports the error.
#include "common.cuh"
#include "gemm_tc.h"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace sg {
namespace {

constexpr int BM = 128;  // weight rows per tile
constexpr int BK = 64;   // K per stage
constexpr int kWTileBytes = BM * BK * 2;  // 16 KB
// Two CTAs per SM (each with its own 2-4 stages and 2*BN TMEM columns,
// 512 in all for BN = 128): one CTA's epilogue and set-up overlap the
// other's main loop.
constexpr int kSmemBudget = 112 * 1024;
constexpr int kThreads = 192;
constexpr unsigned long long kTimeoutNs = 2000000000ULL;

template <int BN>
struct Cfg {
  static constexpr int kATileBytes = BN * BK * 2;
  static constexpr int kStageBytes = kWTileBytes + 2 * kATileBytes;
  static constexpr int kStagesFit = (kSmemBudget - 1024) / kStageBytes;
  static constexpr int STAGES = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 1024;  // + alignment slack
  // One MMA per 16-wide K step covers both activation halves: the A_hi and
  // A_lo tiles sit back to back in shared memory and form one operand of
  // 2*BN rows, so the weight tile is read once per step. Accumulator
  // columns [0, BN) hold W x A_hi, [BN, 2*BN) W x A_lo.
  static constexpr int kN = 2 * BN;
  // Instruction descriptor: bf16 x bf16 -> f32, both operands K-major,
  // N = 2*BN, M = 128.
  static constexpr uint32_t kIdesc = (1u << 4)                        // D: f32
                                     | (1u << 7) | (1u << 10)         // A, B: bf16
                                     | ((uint32_t)(kN >> 3) << 17)    // N
                                     | ((uint32_t)(BM >> 4) << 24);   // M
};

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait; false (and *err set) on timeout or when *err is already set.
__device__ bool mbar_wait(uint32_t bar, unsigned parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = now_ns();
  unsigned spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 63) == 0) {
      if (*(volatile int*)err) return false;
      if (now_ns() - t0 > kTimeoutNs) {
        atomicExch(err, 3);
        return false;
      }
    }
  }
  return true;
}

// 2D TMA tile load (x = inner element offset, a multiple of 64 -> 128-byte
// aligned; y = row offset; rows past the tensor read as zeros). Each load
// fills only the issuing CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand tile with 128-byte
// swizzling, 8-row swizzle atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);  // start address
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused here)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

template <int BN>
__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem),
      "l"(a), "l"(b), "r"(Cfg<BN>::kIdesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

struct TcParams {
  int T;       // tokens (rows of A and C)
  int N;       // weight rows
  int K;
  float* C;
  int ldc;
  int epi;     // EPI_STORE / EPI_ADD / EPI_SWIGLU (C has N/2 columns)
  int* err;
  int w_early; // 1: no earlier kernel writes W, its first tiles may load
               // before the dependency wait
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmAh,
              const __grid_constant__ CUtensorMap tmAl, const TcParams p) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], acc_bar;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = (saddr(smem_raw) + 1023u) & ~1023u;
  // Token tiles vary fastest: the CTAs resident at a time share a few
  // weight tiles (each read from HBM about once) and every token tile (the
  // activations stay in L2); weight tiles varying fastest re-read all
  // weights once per wave of token tiles.
  const int t0 = blockIdx.x * BN;  // tokens
  const int r0 = blockIdx.y * BM;  // weight rows
  const int nk = (p.K + BK - 1) / BK;  // the K tail reads zeros from TMA

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(saddr(&full_bar[s]), 1);
      mbar_init(saddr(&empty_bar[s]), 1);
    }
    mbar_init(saddr(&acc_bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(&tmem_slot)),
                 "r"(C::kN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // TMA producer (one thread). When no earlier kernel writes the weights
    // (w_early), the first stages' weight tiles go out before the
    // dependency wait.
    if (lane == 0) {
      const int pre = p.w_early ? (nk < STAGES ? nk : STAGES) : 0;
      for (int kb = 0; kb < pre; kb++) {
        const uint32_t fb = saddr(&full_bar[kb]);
        mbar_expect_tx(fb, C::kStageBytes);
        tma_load_2d(sbase + kb * C::kStageBytes, &tmW, kb * BK, r0, fb);
      }
      pdl_wait();
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % STAGES;
        const uint32_t st = sbase + s * C::kStageBytes;
        const uint32_t fb = saddr(&full_bar[s]);
        if (kb >= pre) {
          if (kb >= STAGES &&
              !mbar_wait(saddr(&empty_bar[s]), ((kb / STAGES) - 1) & 1, p.err))
            break;
          mbar_expect_tx(fb, C::kStageBytes);
          tma_load_2d(st, &tmW, kb * BK, r0, fb);
        }
        tma_load_2d(st + kWTileBytes, &tmAh, kb * BK, t0, fb);
        tma_load_2d(st + kWTileBytes + C::kATileBytes, &tmAl, kb * BK, t0, fb);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // MMA issuer (one thread)
    if (lane == 0) {
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % STAGES;
        if (!mbar_wait(saddr(&full_bar[s]), (kb / STAGES) & 1, p.err)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t st = sbase + s * C::kStageBytes;
#pragma unroll
        for (int k = 0; k < BK / 16; k++) {
          const uint64_t aw = sw128_desc(st + k * 32);
          const uint64_t bhl = sw128_desc(st + kWTileBytes + k * 32);  // A_hi rows, then A_lo
          mma_bf16<BN>(tmem, aw, bhl, (kb | k) != 0);
        }
        mma_commit(saddr(&empty_bar[s]));
      }
      mma_commit(saddr(&acc_bar));
    }
    __syncwarp();
  } else {
    // Epilogue: warp w owns TMEM lanes (w % 4) * 32 .. +31 = weight rows.
    const int q = warp & 3;
    pdl_wait();
    const bool ok = mbar_wait(saddr(&acc_bar), 0, p.err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok && !*(volatile int*)p.err) {
      const int r = r0 + q * 32 + lane;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        if (t0 + c0 >= p.T) break;  // warp-uniform
        float v[32], vl[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(BN + c0), vl);
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] += vl[j];
        if (p.epi == EPI_SWIGLU) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int t = t0 + c0 + j;
            const float up = __shfl_down_sync(0xFFFFFFFFu, v[j], 1);
            if (t < p.T && (r & 1) == 0 && r + 1 < p.N)
              p.C[(size_t)t * p.ldc + (r >> 1)] = swiglu(v[j], up);
          }
        } else {
          float* cb = p.C + (size_t)(t0 + c0) * p.ldc + r;
          const int nt = min(32, p.T - (t0 + c0));
          if (p.epi == EPI_ADD) {
            // The residual rows: all 32 loads issued before any store (one
            // read-modify-write at a time left each load's latency exposed).
#pragma unroll
            for (int j = 0; j < 32; j++)
              vl[j] = (j < nt && r < p.N) ? cb[(size_t)j * p.ldc] : 0.f;
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] += vl[j];
          }
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (j < nt && r < p.N) cb[(size_t)j * p.ldc] = v[j];
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kN)
                 : "memory");
  }
}

// fp32 -> (bf16 hi, bf16 lo) with hi = RNE(x), lo = RNE(x - hi).
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// Four consecutive activations per thread (K % 4 == 0 and ldx % 4 == 0 on
// this path), 8-byte stores of each half.
__global__ void k_split_hi_lo(const float* __restrict__ x, int ldx, int T, int K,
                              uint16_t* __restrict__ hi, uint16_t* __restrict__ lo) {
  pdl_trigger();
  pdl_wait();
  const int kq = K >> 2;
  const size_t n = (size_t)T * kq;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / kq, k = (i % kq) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + t * ldx + k);
    const float f[4] = {v.x, v.y, v.z, v.w};
    uint16_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      h[j] = f2bf(f[j]);
      l[j] = f2bf(f[j] - __uint_as_float((uint32_t)h[j] << 16));
    }
    const size_t o = t * K + k;
    *reinterpret_cast<uint2*>(hi + o) =
        make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
    *reinterpret_cast<uint2*>(lo + o) =
        make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    SG_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !ptr) SG_DIE("cuTensorMapEncodeTiled unavailable");
    fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  }
  return fn;
}

void encode(TcMap* m, const uint16_t* base, int rows, int K, int box_rows) {
  if (K % 8) SG_DIE("tensor-core GEMM: K must be a multiple of 8");
  if (rows <= 0) SG_DIE("tensor-core GEMM: empty matrix");
  if (((uintptr_t)base) % 16) SG_DIE("tensor-core GEMM: base must be 16-byte aligned");
  CUtensorMap* map = reinterpret_cast<CUtensorMap*>(m->bytes);
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)base, dims, strides,
                           box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) SG_DIE("cuTensorMapEncodeTiled failed");
  m->rows = rows;
  m->K = K;
  m->box_rows = box_rows;
}

constexpr int kWidths[3] = {32, 64, 128};

template <int BN>
void launch_bn(const TcMap& w, const TcAct& a, int wi, const TcParams& p, cudaStream_t s) {
  const int row_tiles = (w.rows + BM - 1) / BM;
  if (row_tiles > 65535) SG_DIE("tensor-core GEMM: too many weight rows");
  dim3 grid((p.T + BN - 1) / BN, row_tiles);
  launch(k_gemm_tc<BN>, grid, dim3(kThreads), (size_t)Cfg<BN>::kSmemBytes, s,
         *reinterpret_cast<const CUtensorMap*>(w.bytes),
         *reinterpret_cast<const CUtensorMap*>(a.hi[wi].bytes),
         *reinterpret_cast<const CUtensorMap*>(a.lo[wi].bytes), p);
}

}  // namespace

void tc_make_map(TcMap* m, const uint16_t* base, int rows, int K) { encode(m, base, rows, K, BM); }

void tc_make_act(TcAct* a, const uint16_t* hi, const uint16_t* lo, int rows, int K) {
  for (int i = 0; i < 3; i++) {
    encode(&a->hi[i], hi, rows, K, kWidths[i]);
    encode(&a->lo[i], lo, rows, K, kWidths[i]);
  }
  a->hi_base = hi;
  a->lo_base = lo;
}

void tc_split(const float* x, int ldx, int T, int K, uint16_t* hi, uint16_t* lo, cudaStream_t s) {
  if (K % 4 || ldx % 4 || ((uintptr_t)x) % 16)
    SG_DIE("tensor-core GEMM: activations need K and their row stride in multiples of 4");
  const size_t n = (size_t)T * (K / 4);
  int blocks = (int)((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  launch(k_split_hi_lo, dim3(blocks), dim3(256), 0, s, x, ldx, T, K, hi, lo);
}

// Resident CTAs of the current device: two per SM (kSmemBudget), the SM
// count read once per device.
int resident_ctas() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 2 * 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = 2 * n;
  }
  return cached[dev];
}

int tc_width(int rows, int T) {
  // Streaming-bound model: time ~ waves x bytes per stage; ties go to the
  // wider tile.
  const int rt = (rows + BM - 1) / BM;
  const long per_wave = resident_ctas();
  int best = 0;
  long best_cost = 0;
  for (int i = 2; i >= 0; i--) {
    const int bn = kWidths[i];
    const long ctas = (long)rt * ((T + bn - 1) / bn);
    const long waves = (ctas + per_wave - 1) / per_wave;
    const long cost = waves * (kWTileBytes + 2L * bn * BK * 2);
    if (best == 0 || cost < best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

void tc_gemm(const TcMap& w, const TcAct& a, int T, float* C, int ldc, Epilogue epi, int* err,
             cudaStream_t s, bool w_early) {
  if (w.K != a.hi[0].K) SG_DIE("tensor-core GEMM: K mismatch");
  if (T > a.hi[0].rows) SG_DIE("tensor-core GEMM: more tokens than the activation map holds");
  if (T <= 0) return;
  const TcParams p{T, w.rows, w.K, C, ldc, (int)epi, err, w_early ? 1 : 0};
  const int bn = tc_width(w.rows, T);
  if (bn == 128)
    launch_bn<128>(w, a, 2, p, s);
  else if (bn == 64)
    launch_bn<64>(w, a, 1, p, s);
  else
    launch_bn<32>(w, a, 0, p, s);
}

void tc_configure() {
  SG_CUDA(cudaFuncSetAttribute(k_gemm_tc<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg<32>::kSmemBytes));
  SG_CUDA(cudaFuncSetAttribute(k_gemm_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg<64>::kSmemBytes));
  SG_CUDA(cudaFuncSetAttribute(k_gemm_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg<128>::kSmemBytes));
}

}  // namespace sg
