// Shared device helpers for the strasgpt-b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#define SG_DIE(msg)                                                        \
  do {                                                                     \
    fprintf(stderr, "[StrasGPT] Error at %s:%d (%s): %s\n", __FILE__,      \
            __LINE__, __func__, msg);                                      \
    exit(EXIT_FAILURE);                                                    \
  } while (0)

#define SG_CUDA(call)                                                      \
  do {                                                                     \
    cudaError_t err_ = (call);                                             \
    if (err_ != cudaSuccess) {                                             \
      char m_[512];                                                        \
      snprintf(m_, sizeof(m_), "CUDA error %s: %s", #call,                 \
               cudaGetErrorString(err_));                                  \
      SG_DIE(m_);                                                          \
    }                                                                      \
  } while (0)

namespace sg {

// Bound (ns of %globaltimer) of the device-side waits on other CTAs or
// GPUs: STRASGPT_WAIT_LIMIT_MS when set (tests make waits run out quickly
// with it), else `default_ms`.
inline unsigned long long wait_limit_ns(unsigned long long default_ms) {
  const char* v = getenv("STRASGPT_WAIT_LIMIT_MS");
  const long long ms = (v && *v) ? atoll(v) : 0;
  return (ms > 0 ? (unsigned long long)ms : default_ms) * 1000000ull;
}

// bf16 stored as raw uint16_t everywhere: widening is a 16-bit shift
// (the reference's util_bf16_to_f32, include/util.h:33-39).
__device__ __forceinline__ float bf16_lo(uint32_t w) {
  return __uint_as_float(w << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t w) {
  return __uint_as_float(w & 0xFFFF0000u);
}
__device__ __forceinline__ float bf16_to_f32(uint16_t w) {
  return __uint_as_float(((uint32_t)w) << 16);
}

// 128-bit streaming load that bypasses L1 (weights are read once per step).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Bulk prefetch of [p, p + bytes) into L2 (bytes a multiple of 16, p
// 16-byte aligned). Only ever used on read-only weights.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes)
               : "memory");
}

// Programmatic dependent launch. Every kernel launched through sg::launch
// calls pdl_wait() before it reads anything an earlier kernel writes or
// writes anything an earlier kernel reads; only read-only weights are
// touched before it. pdl_trigger() lets the next kernel of the stream start
// its own prologue (weight prefetch) while this one runs.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Block-wide sum; every thread gets the result. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// Dot of 8 bf16 weights (one 16-byte vector) with 8 fp32 activations.
__device__ __forceinline__ float dot8(uint4 w, float4 a, float4 b, float acc) {
  acc = fmaf(bf16_lo(w.x), a.x, acc);
  acc = fmaf(bf16_hi(w.x), a.y, acc);
  acc = fmaf(bf16_lo(w.y), a.z, acc);
  acc = fmaf(bf16_hi(w.y), a.w, acc);
  acc = fmaf(bf16_lo(w.z), b.x, acc);
  acc = fmaf(bf16_hi(w.z), b.y, acc);
  acc = fmaf(bf16_lo(w.w), b.z, acc);
  acc = fmaf(bf16_hi(w.w), b.w, acc);
  return acc;
}

// s[i] += w_i * x_i for the 8 bf16 weights of a 16-byte vector: eight
// independent accumulators (no FMA chain between the elements).
__device__ __forceinline__ void acc8(uint4 w, float4 a, float4 b, float* s) {
  s[0] = fmaf(bf16_lo(w.x), a.x, s[0]);
  s[1] = fmaf(bf16_hi(w.x), a.y, s[1]);
  s[2] = fmaf(bf16_lo(w.y), a.z, s[2]);
  s[3] = fmaf(bf16_hi(w.y), a.w, s[3]);
  s[4] = fmaf(bf16_lo(w.z), b.x, s[4]);
  s[5] = fmaf(bf16_hi(w.z), b.y, s[5]);
  s[6] = fmaf(bf16_lo(w.w), b.z, s[6]);
  s[7] = fmaf(bf16_hi(w.w), b.w, s[7]);
}

// SiLU-gated product, written as the reference does
// (source/transformer.c:1481-1484): fc * (1 / (1 + expf(-fc))) * up.
__device__ __forceinline__ float swiglu(float fc, float up) {
  fc *= (1.0f / (1.0f + expf(-fc)));
  return fc * up;
}

// Launch with the programmatic-stream-serialization attribute (PDL), unless
// STRASGPT_PDL=0. Launch errors are fatal.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                   size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  SG_CUDA(cudaLaunchKernelEx(&cfg, kernel, ((KArgs)args)...));
}

}  // namespace sg
