// Tensor-parallel exchanges over NVLink peer memory (protocol in tp.h).
//
// Waits are bounded (TpComm::timeout_ns of %globaltimer, 60 s unless
// STRASGPT_WAIT_LIMIT_MS sets another limit): on timeout a kernel sets
// the rank's error flag, skips the data movement and returns; the host
// checks the flag after the step and stops with an error message. Every CTA
// posts the epoch itself (idempotent stores), so no CTA waits on another CTA
// of its own grid being scheduled.
#include "common.cuh"
#include "tp.h"

#include <string.h>

namespace sg {
namespace {

constexpr size_t kHeader = 256;  // flags, epoch, ticket

struct TpArgs {
  unsigned char* peer[kTpMaxRanks];
  int rank, world;
  size_t cap;
  int* err;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ unsigned* flags_of(unsigned char* b) { return (unsigned*)b; }
__device__ __forceinline__ unsigned* epoch_of(unsigned char* b) { return (unsigned*)(b + 64); }
__device__ __forceinline__ unsigned* ticket_of(unsigned char* b) { return (unsigned*)(b + 68); }
__device__ __forceinline__ float* data_of(unsigned char* b, size_t cap, unsigned par) {
  return reinterpret_cast<float*>(b + kHeader) + (size_t)par * cap;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_peer4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_peer(const float* p) {
  float v;
  asm volatile("ld.volatile.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread 0 of a CTA: post epoch e to every peer, then wait for every peer's
// post of e. Returns false on timeout (error flag set).
__device__ bool post_and_wait(const TpArgs& a, unsigned e) {
  unsigned char* me = a.peer[a.rank];
  __threadfence_system();
  for (int p = 0; p < a.world; p++) st_release_sys(flags_of(a.peer[p]) + a.rank, e);
  const unsigned* f = flags_of(me);
  unsigned long long t0 = 0;
  for (int p = 0; p < a.world; p++) {
    unsigned spins = 0;
    while ((int)(ld_acquire_sys(f + p) - e) < 0) {
      if ((++spins & 255) == 0) {
        if (*(volatile int*)a.err) return false;
        const unsigned long long t = now_ns();
        if (t0 == 0) t0 = t;
        if (t - t0 > a.timeout_ns) {
          atomicExch(a.err, 1);
          return false;
        }
      }
    }
  }
  return true;
}

// Last CTA of the grid to finish records the completed epoch.
__device__ void finish(const TpArgs& a, unsigned e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned char* me = a.peer[a.rank];
    __threadfence();
    if (atomicAdd(ticket_of(me), 1u) == gridDim.x - 1) {
      *ticket_of(me) = 0;
      *epoch_of(me) = e;
    }
  }
}

__global__ void k_tp_stage(TpArgs a, const float* __restrict__ src, size_t n) {
  pdl_trigger();
  pdl_wait();
  unsigned char* me = a.peer[a.rank];
  const unsigned e = *(volatile unsigned*)epoch_of(me) + 1;
  float* dst = data_of(me, a.cap, e & 1);
  const size_t n4 = n / 4;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride)
    reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
  for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = src[i];
}

__global__ void k_tp_allreduce_add(TpArgs a, float* __restrict__ x, size_t n) {
  __shared__ bool ok;
  pdl_trigger();
  pdl_wait();
  unsigned char* me = a.peer[a.rank];
  const unsigned e = *(volatile unsigned*)epoch_of(me) + 1;
  const unsigned par = e & 1;
  if (threadIdx.x == 0) ok = post_and_wait(a, e);
  __syncthreads();
  if (ok) {
    const size_t n4 = n / 4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
      float4 s = ld_peer4(data_of(a.peer[0], a.cap, par) + 4 * i);
      for (int r = 1; r < a.world; r++) {
        const float4 v = ld_peer4(data_of(a.peer[r], a.cap, par) + 4 * i);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      float4 xv = reinterpret_cast<float4*>(x)[i];
      xv.x += s.x;
      xv.y += s.y;
      xv.z += s.z;
      xv.w += s.w;
      reinterpret_cast<float4*>(x)[i] = xv;
    }
    for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      float s = ld_peer(data_of(a.peer[0], a.cap, par) + i);
      for (int r = 1; r < a.world; r++) s += ld_peer(data_of(a.peer[r], a.cap, par) + i);
      x[i] += s;
    }
  }
  finish(a, e);
}

__global__ void k_tp_gather_rows(TpArgs a, float* __restrict__ dst, int rows, int cols) {
  __shared__ bool ok;
  pdl_trigger();
  pdl_wait();
  unsigned char* me = a.peer[a.rank];
  const unsigned e = *(volatile unsigned*)epoch_of(me) + 1;
  const unsigned par = e & 1;
  if (threadIdx.x == 0) ok = post_and_wait(a, e);
  __syncthreads();
  if (ok) {
    const size_t per = (size_t)rows * cols;
    const size_t n = per * a.world;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      const size_t row = i / ((size_t)a.world * cols);
      const size_t rem = i % ((size_t)a.world * cols);
      const int r = (int)(rem / cols);
      const size_t j = rem % cols;
      dst[i] = ld_peer(data_of(a.peer[r], a.cap, par) + row * cols + j);
    }
  }
  finish(a, e);
}

__global__ void k_tp_barrier(TpArgs a) {
  pdl_trigger();
  pdl_wait();
  unsigned char* me = a.peer[a.rank];
  const unsigned e = *(volatile unsigned*)epoch_of(me) + 1;
  if (threadIdx.x == 0) post_and_wait(a, e);  // a timeout is recorded in *a.err
  finish(a, e);
}

TpArgs args_of(const TpComm& c) {
  if (!c.connected) SG_DIE("tensor-parallel exchange before strasgpt_tp_connect");
  TpArgs a;
  for (int r = 0; r < kTpMaxRanks; r++) a.peer[r] = c.peer[r];
  a.rank = c.rank;
  a.world = c.world;
  a.cap = c.cap;
  a.err = c.err;
  a.timeout_ns = c.timeout_ns;
  return a;
}

int blocks_for(size_t n, int per_thread) {
  size_t b = (n + (size_t)256 * per_thread - 1) / ((size_t)256 * per_thread);
  if (b < 1) b = 1;
  if (b > 148 * 4) b = 148 * 4;
  return (int)b;
}

void stage(TpComm& c, const float* src, size_t n, cudaStream_t s) {
  if (n > c.cap) SG_DIE("tensor-parallel exchange larger than the exchange buffer");
  if (((uintptr_t)src) % 16) SG_DIE("tensor-parallel exchange: source must be 16-byte aligned");
  launch(k_tp_stage, dim3(blocks_for(n, 16)), dim3(256), 0, s, args_of(c), src, n);
}

}  // namespace

size_t tp_buffer_bytes(size_t cap, size_t extra) {
  return kHeader + 2 * cap * sizeof(float) + (extra + 255) / 256 * 256;
}

void tp_alloc(TpComm* c, int rank, int world, size_t cap, size_t extra) {
  if (world < 1 || world > kTpMaxRanks || rank < 0 || rank >= world)
    SG_DIE("invalid tensor-parallel placement");
  c->rank = rank;
  c->world = world;
  c->timeout_ns = wait_limit_ns(60000);
  c->cap = (cap + 63) & ~(size_t)63;
  c->extra_off = kHeader + 2 * c->cap * sizeof(float);
  const size_t bytes = tp_buffer_bytes(c->cap, extra);
  SG_CUDA(cudaMalloc(&c->local, bytes));
  SG_CUDA(cudaMemset(c->local, 0, bytes));
  SG_CUDA(cudaMalloc(&c->err, sizeof(int)));
  SG_CUDA(cudaMemset(c->err, 0, sizeof(int)));
  for (int r = 0; r < kTpMaxRanks; r++) c->peer[r] = nullptr;
  c->peer[rank] = c->local;
  c->connected = (world == 1);
}

void tp_handle(const TpComm& c, void* out64) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  SG_CUDA(cudaIpcGetMemHandle(&h, c.local));
  memcpy(out64, &h, 64);
}

void tp_connect(TpComm* c, const void* handles) {
  if (c->connected) SG_DIE("tensor-parallel peers already connected");
  const unsigned char* hb = static_cast<const unsigned char*>(handles);
  for (int r = 0; r < c->world; r++) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + 64 * r, 64);
    void* p = nullptr;
    SG_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    c->peer[r] = static_cast<unsigned char*>(p);
  }
  c->connected = true;
  c->ipc = true;
}

void tp_connect_local(TpComm* c, unsigned char* const* buffers, const int* devices) {
  if (c->connected) SG_DIE("tensor-parallel peers already connected");
  int me = 0;
  SG_CUDA(cudaGetDevice(&me));
  for (int r = 0; r < c->world; r++) {
    c->peer[r] = buffers[r];
    if (r == c->rank || devices[r] == me) continue;
    int ok = 0;
    SG_CUDA(cudaDeviceCanAccessPeer(&ok, me, devices[r]));
    if (!ok) SG_DIE("single-process tensor parallelism: no peer access between the GPUs");
    const cudaError_t e = cudaDeviceEnablePeerAccess(devices[r], 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled)
      (void)cudaGetLastError();
    else
      SG_CUDA(e);
  }
  c->connected = true;
  c->ipc = false;
}

void tp_free(TpComm* c, cudaStream_t s) {
  if (c->world > 1 && c->connected) {
    // No peer may still read this buffer once it is released.
    tp_barrier(*c, s);
    cudaStreamSynchronize(s);
    if (c->ipc)
      for (int r = 0; r < c->world; r++)
        if (r != c->rank && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
  }
  if (c->local) cudaFree(c->local);
  if (c->err) cudaFree(c->err);
  c->local = nullptr;
  c->err = nullptr;
  c->connected = false;
}

void tp_allreduce_add(TpComm& c, const float* part, float* x, size_t n, cudaStream_t s) {
  stage(c, part, n, s);
  launch(k_tp_allreduce_add, dim3(blocks_for(n, 8)), dim3(256), 0, s, args_of(c), x, n);
}

void tp_gather_rows(TpComm& c, const float* src, int rows, int cols, float* dst,
                    cudaStream_t s) {
  const size_t n = (size_t)rows * cols;
  stage(c, src, n, s);
  launch(k_tp_gather_rows, dim3(blocks_for(n * c.world, 8)), dim3(256), 0, s, args_of(c), dst,
         rows, cols);
}

void tp_barrier(TpComm& c, cudaStream_t s) {
  launch(k_tp_barrier, dim3(1), dim3(32), 0, s, args_of(c));
}

int tp_wait_check(int timeout_ms, bool peer_posted, cudaStream_t s) {
  int dev = 0;
  SG_CUDA(cudaGetDevice(&dev));
  TpComm c;
  tp_alloc(&c, 0, 2, 64);
  c.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
  unsigned char* other = nullptr;  // rank 1's buffer: nothing runs rank 1
  const size_t bytes = tp_buffer_bytes(c.cap, 0);
  SG_CUDA(cudaMalloc(&other, bytes));
  SG_CUDA(cudaMemset(other, 0, bytes));
  unsigned char* bufs[2] = {c.local, other};
  const int devs[2] = {dev, dev};
  tp_connect_local(&c, bufs, devs);
  if (peer_posted) {
    // Rank 1's post of the first exchange epoch, as if it had run.
    const unsigned one = 1;
    SG_CUDA(cudaMemcpy(c.local + sizeof(unsigned), &one, sizeof(one), cudaMemcpyHostToDevice));
  }
  tp_barrier(c, s);
  SG_CUDA(cudaStreamSynchronize(s));
  int err = 0;
  SG_CUDA(cudaMemcpy(&err, c.err, sizeof(int), cudaMemcpyDeviceToHost));
  // No final barrier: rank 1 does not exist.
  SG_CUDA(cudaFree(other));
  SG_CUDA(cudaFree(c.local));
  SG_CUDA(cudaFree(c.err));
  return err != 0 ? 1 : 0;
}

}  // namespace sg
