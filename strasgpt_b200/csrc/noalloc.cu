// strasgpt_k_matvec_noalloc: the one-token projection of strasgpt_k_matvec,
// computed split-K, with its scratch in a fixed device array instead of
// memory the call allocates.
//
// Who needs it: a host engine that has already handed the GPU's free memory
// to its own pools (a KV-cache pool sized to fill HBM, a caching allocator
// that must account for every byte) cannot let a library call cudaMalloc
// behind its back, and a decode loop cannot afford cudaMalloc/cudaFree
// between steps either, since cudaFree waits for the whole device. This entry
// point lets such callers pass inputs and outputs they own and nothing else.
//
// Scratch: g_noalloc_scratch below, 4 MiB per device, reserved when the
// library's device code is loaded on a GPU and held until the process
// exits. Layout (floats): [0, 64) per-split sums of squares of x (RMSNorm),
// then [nsplit][weight rows] per-split partial dot products. Every float a
// call reads is written earlier in the same call, so nothing has to start
// at zero and nothing is cleared; the array keeps the last call's contents.
// All calls on a device share the array: calls whose kernels overlap on the
// GPU (two streams, or two host threads on different streams) race on it and
// must be serialised by the caller, e.g. by issuing them on one stream.
//
// Set-up: the first call on each device resolves the array's device address
// with cudaGetSymbolAddress while that device is current, and caches it.
// That first call on a device should therefore come before any stream
// capture on that device.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

extern "C" {
#include "strasgpt_kernels.h"
}

namespace {

constexpr int kScratchFloats = STRASGPT_NOALLOC_SCRATCH_BYTES / 4;
constexpr int kMaxSplits = 64;      // also the sums-of-squares slots
constexpr int kRowsPerCta = 8;      // one warp per weight row
constexpr int kCtasPerSm = 8;       // split-K target: this many CTAs per SM

// The scratch itself. In host code this name is only a stand-in for the
// symbol; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

// Partial dot products of weight rows with one K-slice of x (times the
// RMSNorm gain when NORM; the 1/rms factor is applied in the reduction).
template <bool NORM>
__global__ void __launch_bounds__(256)
    k_matvec_splitk(const float* __restrict__ x, const uint16_t* __restrict__ nw,
                    const uint16_t* __restrict__ W, int K, int wrows, int ks,
                    float* __restrict__ scratch) {
  __shared__ float red[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.y;
  const int k0 = split * ks;
  const int k1 = min(K, k0 + ks);
  if (NORM && blockIdx.x == 0) {
    float ss = 0.f;
    for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) ss = fmaf(x[k], x[k], ss);
    ss = sg::block_sum(ss, red);
    if (threadIdx.x == 0) scratch[split] = ss;
  }
  const int r = blockIdx.x * kRowsPerCta + warp;
  if (r >= wrows) return;
  const uint16_t* wr = W + (size_t)r * K;
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int k = k0 + lane * 8; k < k1; k += 256) {
    const uint4 w = sg::ldg_stream(wr + k);
    float4 a = *reinterpret_cast<const float4*>(x + k);
    float4 b = *reinterpret_cast<const float4*>(x + k + 4);
    if (NORM) {
      const uint4 g = *reinterpret_cast<const uint4*>(nw + k);
      a.x *= sg::bf16_lo(g.x); a.y *= sg::bf16_hi(g.x);
      a.z *= sg::bf16_lo(g.y); a.w *= sg::bf16_hi(g.y);
      b.x *= sg::bf16_lo(g.z); b.y *= sg::bf16_hi(g.z);
      b.z *= sg::bf16_lo(g.w); b.w *= sg::bf16_hi(g.w);
    }
    sg::acc8(w, a, b, s);
  }
  float t = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
  t = sg::warp_sum(t);
  if (lane == 0) scratch[kMaxSplits + (size_t)split * wrows + r] = t;
}

// Sum of the split partials, RMSNorm scale, epilogue: one thread per output.
template <bool NORM>
__global__ void __launch_bounds__(256)
    k_matvec_splitk_reduce(const float* __restrict__ scratch, int nsplit, int wrows, int K,
                           float eps, int epi, int rows, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  float scale = 1.f;
  if (NORM) {
    float ss = 0.f;
    for (int s = 0; s < nsplit; s++) ss += scratch[s];
    scale = 1.0f / sqrtf(ss / (float)K + eps);
  }
  const float* part = scratch + kMaxSplits;
  auto total = [&](int r) {
    float v = 0.f;
    for (int s = 0; s < nsplit; s++) v += part[(size_t)s * wrows + r];
    return v * scale;
  };
  if (epi == STRASGPT_EPI_SWIGLU) {
    const int gate = sg::gu_gate_row(i);
    out[i] = sg::swiglu(total(gate), total(gate + SG_GU_GROUP));
  }
  else if (epi == STRASGPT_EPI_ADD)
    out[i] += total(i);
  else
    out[i] = total(i);
}

std::mutex g_setup_mutex;
float* g_scratch_on_device[64];
int g_sms_on_device[64];

// Device address of g_noalloc_scratch on the current device, resolved once
// per device, and that device's SM count (which sizes the split).
float* scratch_on_current_device(int* sms) {
  int dev = 0;
  SG_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) SG_DIE("strasgpt_k_matvec_noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_on_device[dev]) {
    int n = 0;
    SG_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    g_sms_on_device[dev] = n > 0 ? n : 1;
    float* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      char m[256];
      snprintf(m, sizeof(m), "strasgpt_k_matvec_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
      SG_DIE(m);
    }
    g_scratch_on_device[dev] = ptr;
  }
  *sms = g_sms_on_device[dev];
  return g_scratch_on_device[dev];
}

int reject(const char* why) {
  fprintf(stderr, "[StrasGPT] Error: strasgpt_k_matvec_noalloc: %s\n", why);
  return -1;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

extern "C" int strasgpt_k_matvec_noalloc(const float* x, const uint16_t* norm_w, float eps,
                                         const uint16_t* w, int k, int rows, float* out,
                                         int epi, void* stream) {
  if (epi < STRASGPT_EPI_STORE || epi > STRASGPT_EPI_SWIGLU) return reject("unknown epilogue");
  if (k <= 0 || rows <= 0) return reject("empty shape");
  if (k % 8 != 0) return reject("k must be a multiple of 8");
  if (!x || !w || !out) return reject("null buffer");
  if (!aligned16(x) || !aligned16(w) || (norm_w && !aligned16(norm_w)))
    return reject("x, w and norm_w must be 16-byte aligned");
  if (epi == STRASGPT_EPI_SWIGLU && rows % SG_GU_GROUP != 0)
    return reject("SwiGLU rows must be a multiple of the gate/up group");
  const long long wrows = epi == STRASGPT_EPI_SWIGLU ? 2LL * rows : (long long)rows;
  if (wrows + kMaxSplits > kScratchFloats) {
    char m[200];
    snprintf(m, sizeof(m),
             "%lld weight rows exceed the %d-byte scratch (at most %d weight rows; "
             "use strasgpt_k_matvec)",
             wrows, STRASGPT_NOALLOC_SCRATCH_BYTES, kScratchFloats - kMaxSplits);
    return reject(m);
  }
  int sms = 1;
  float* scratch = scratch_on_current_device(&sms);
  const int row_blocks = (int)((wrows + kRowsPerCta - 1) / kRowsPerCta);
  int nsplit = (sms * kCtasPerSm + row_blocks - 1) / row_blocks;
  nsplit = std::min(nsplit, kMaxSplits);
  nsplit = std::min(nsplit, (k + 255) / 256);
  nsplit = std::min(nsplit, (int)((kScratchFloats - kMaxSplits) / wrows));
  nsplit = std::max(nsplit, 1);
  int ks = (k + nsplit - 1) / nsplit;
  ks = (ks + 7) & ~7;
  nsplit = (k + ks - 1) / ks;

  cudaStream_t s = (cudaStream_t)stream;
  const dim3 grid(row_blocks, nsplit);
  const int rgrid = (rows + 255) / 256;
  if (norm_w) {
    k_matvec_splitk<true><<<grid, 256, 0, s>>>(x, norm_w, w, k, (int)wrows, ks, scratch);
    k_matvec_splitk_reduce<true>
        <<<rgrid, 256, 0, s>>>(scratch, nsplit, (int)wrows, k, eps, epi, rows, out);
  } else {
    k_matvec_splitk<false><<<grid, 256, 0, s>>>(x, norm_w, w, k, (int)wrows, ks, scratch);
    k_matvec_splitk_reduce<false>
        <<<rgrid, 256, 0, s>>>(scratch, nsplit, (int)wrows, k, eps, epi, rows, out);
  }
  SG_CUDA(cudaGetLastError());
  return 0;
}
