// Kernel-level C entry points (include/strasgpt_kernels.h).
#include "common.cuh"
#include "gemm_tc.h"
#include "kernels.h"
#include "tp.h"

extern "C" {
#include "strasgpt_kernels.h"
}

namespace {

// cudaFuncSetAttribute is per device: configure each device once.
void ensure_configured() {
  static unsigned long long done = 0;
  int dev = 0;
  SG_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !(done & (1ull << dev))) {
    sg::configure_kernels();
    sg::tc_configure();
    done |= 1ull << dev;
  }
}

sg::Epilogue epilogue(int epi) {
  if (epi < 0 || epi > 2) SG_DIE("unknown epilogue");
  return (sg::Epilogue)epi;
}

}  // namespace

extern "C" {

int strasgpt_k_matvec(const float* x, const uint16_t* norm_w, float eps,
                      const uint16_t* w, int k, int rows, float* out, int epi,
                      void* stream) {
  ensure_configured();
  if (k <= 0 || rows <= 0) SG_DIE("matvec: empty shape");
  sg::matvec(x, norm_w, eps, w, k, rows, out, epilogue(epi),
             (cudaStream_t)stream);
  SG_CUDA(cudaGetLastError());
  return 0;
}

int strasgpt_k_gemm_simt(const float* a, int lda, const uint16_t* w, int k,
                         int m, int n, float* c, int ldc, int epi,
                         void* stream) {
  ensure_configured();
  if (k <= 0 || m <= 0 || n <= 0) SG_DIE("gemm: empty shape");
  sg::gemm_simt(a, lda, w, k, m, n, c, ldc, epilogue(epi),
                (cudaStream_t)stream);
  SG_CUDA(cudaGetLastError());
  return 0;
}

int strasgpt_k_gemm_tc(const float* a, int lda, uint16_t* a_hi,
                       uint16_t* a_lo, const uint16_t* w, int k, int m, int n,
                       float* c, int ldc, int epi, int* err, void* stream) {
  ensure_configured();
  if (k <= 0 || m <= 0 || n <= 0) SG_DIE("gemm: empty shape");
  if (epi == STRASGPT_EPI_SWIGLU && n % 2) SG_DIE("gemm: odd swiglu rows");
  cudaStream_t s = (cudaStream_t)stream;
  sg::TcMap mw;
  sg::TcAct act;
  sg::tc_make_map(&mw, w, n, k);
  sg::tc_make_act(&act, a_hi, a_lo, m, k);
  sg::tc_split(a, lda, m, k, a_hi, a_lo, s);
  sg::tc_gemm(mw, act, m, c, ldc, epilogue(epi), err, s, false);
  SG_CUDA(cudaGetLastError());
  return 0;
}

int strasgpt_k_attn_prefill(const float* q, const float* k_cache,
                            const float* v_cache, int t, int kv_heads,
                            int group, int head_dim, int ctx, int pos0,
                            float* att, void* stream) {
  ensure_configured();
  if (t <= 0 || kv_heads <= 0 || group <= 0 || pos0 < 0)
    SG_DIE("attn_prefill: empty shape");
  if ((long)pos0 + t > ctx) SG_DIE("attn_prefill: positions beyond the cache");
  sg::AttnPrefillArgs a;
  a.q = q; a.k_cache = k_cache; a.v_cache = v_cache;
  a.T = t; a.KHl = kv_heads; a.G = group; a.HD = head_dim; a.ctx = ctx;
  a.pos0 = pos0; a.att = att;
  sg::attn_prefill(a, (cudaStream_t)stream);
  SG_CUDA(cudaGetLastError());
  return 0;
}

int strasgpt_k_rmsnorm_rows(const float* x, int t, int d, const uint16_t* w,
                            float eps, float* y, void* stream) {
  ensure_configured();
  if (t <= 0 || d <= 0) SG_DIE("rmsnorm: empty shape");
  sg::rmsnorm_rows(x, t, d, w, eps, y, (cudaStream_t)stream);
  SG_CUDA(cudaGetLastError());
  return 0;
}

int strasgpt_k_tp_wait_check(int timeout_ms, int peer_posted, void* stream) {
  if (timeout_ms <= 0 || timeout_ms > 60000) return -1;
  return sg::tp_wait_check(timeout_ms, peer_posted != 0, (cudaStream_t)stream);
}

}  // extern "C"
