// Tensor-parallel exchanges between the GPUs of one node over NVLink peer
// memory: one process per GPU (buffers shared through CUDA IPC), or all
// ranks in one process (buffers used directly, peer access enabled).
//
// Every rank owns one exchange buffer (a single cudaMalloc, shared with the
// other ranks through cudaIpcGetMemHandle / cudaIpcOpenMemHandle):
//   flags  u32 [kTpMaxRanks]   latest exchange epoch posted by each rank
//   epoch  u32                 this rank's last completed epoch (local)
//   ticket u32                 last-CTA detection of multi-CTA exchanges
//   data   f32 [2][cap]        staged operands, two halves by epoch parity
// An exchange with epoch e: the rank stages its operand into data[e & 1],
// posts e into every peer's flags[rank] (release, system scope), waits until
// its own flags[p] >= e for every peer p (acquire, bounded), then reads the
// peers' data[e & 1] over NVLink. A half is rewritten two exchanges later,
// after every peer has posted the epoch in between, i.e. has finished
// reading it. All ranks run the same exchanges in the same order; sums run
// in rank order, so every rank gets bit-identical results.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sg {

constexpr int kTpMaxRanks = 8;

struct TpComm {
  int rank = 0, world = 1;
  size_t cap = 0;                       // floats per data half
  size_t extra_off = 0;                 // byte offset of the extra region
  unsigned char* local = nullptr;       // this rank's exchange buffer
  unsigned char* peer[kTpMaxRanks] = {};  // every rank's buffer (own included)
  int* err = nullptr;                   // device int: non-zero after a timeout
  bool connected = false;
  bool ipc = false;                     // peers mapped through CUDA IPC
  unsigned long long timeout_ns = 0;    // bound of every wait on a peer
};

// Bytes of the exchange buffer for `cap` floats per half and `extra` bytes
// of a region other kernels share with the peers (zeroed, 256-aligned).
size_t tp_buffer_bytes(size_t cap, size_t extra);
// Allocates and zeroes this rank's buffer (and the error flag).
void tp_alloc(TpComm* c, int rank, int world, size_t cap, size_t extra = 0);
// 64-byte IPC handle of this rank's buffer.
void tp_handle(const TpComm& c, void* out64);
// Maps the peers' buffers from world x 64-byte handles (rank order).
void tp_connect(TpComm* c, const void* handles);
// Connects ranks that live in this process: every rank's buffer
// (buffers[r], allocated on devices[r]) is used directly; peer access from
// this rank's device to every other device is enabled. Call with this
// rank's device current.
void tp_connect_local(TpComm* c, unsigned char* const* buffers, const int* devices);
// Unmaps the peers (after a final barrier exchange) and frees the buffer.
void tp_free(TpComm* c, cudaStream_t s);

// x[i] += sum over ranks (in rank order) of part_r[i], i < n.
void tp_allreduce_add(TpComm& c, const float* part, float* x, size_t n, cudaStream_t s);
// dst[row][r * cols + j] = src_r[row][j] for every rank r (src rows `cols`
// floats apart, dst rows world * cols).
void tp_gather_rows(TpComm& c, const float* src, int rows, int cols, float* dst,
                    cudaStream_t s);
// Exchange without data: returns once every rank has reached it.
void tp_barrier(TpComm& c, cudaStream_t s);

// The bounded wait of an exchange, alone: a 2-rank barrier on this GPU
// whose rank 1 is a buffer nothing runs (peer_posted: its post already in
// place). Returns 1 when the wait ran out (the kernel returned with the
// error flag set), 0 when it completed.
int tp_wait_check(int timeout_ms, bool peer_posted, cudaStream_t s);

}  // namespace sg
