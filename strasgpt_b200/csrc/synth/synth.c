// Deterministic, counter-based fill of synthetic model tensors.
//
// Every element is a pure function of (seed, stream, index), so a tensor can
// be filled in parallel, in any order, on any machine, with identical bits:
//   r(i)   = mix64(mix64(seed * PHI + stream) + i * PHI)       (splitmix64)
//   normal: Box-Muller on element pairs (2p, 2p+1) in double precision,
//           u1 = (r(2p) >> 11 + 1) * 2^-53, u2 = (r(2p+1) >> 11) * 2^-53,
//           z0 = sqrt(-2 ln u1) cos(2 pi u2), z1 = ... sin(...);
//           value = (float)(z * std), rounded to bf16 (nearest even).
//   bytes:  lo + r(i) % (hi - lo + 1).
// `stream` is the FNV-1a 64-bit hash of the tensor name.
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define PHI 0x9E3779B97F4A7C15ULL

static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

static inline uint64_t draw(uint64_t key, uint64_t i) {
  return mix64(key + i * PHI);
}

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) { // inf / nan: truncate, keep nan
    return (uint16_t)((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
  }
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

uint64_t synth_stream_id(const char* name) {
  uint64_t h = 0xCBF29CE484222325ULL;
  for (const unsigned char* p = (const unsigned char*)name; *p; p++) {
    h ^= *p;
    h *= 0x100000001B3ULL;
  }
  return h;
}

// N(0, std^2) in bf16 for elements [0, n).
void synth_normal_bf16(
    uint16_t* out, size_t n, uint64_t seed, uint64_t stream, float std
) {
  const uint64_t key = mix64(seed * PHI + stream);
  const double two_pi = 6.283185307179586476925286766559;
  const size_t pairs = (n + 1) / 2;
#pragma omp parallel for schedule(static)
  for (size_t p = 0; p < pairs; p++) {
    uint64_t a = draw(key, 2 * p);
    uint64_t b = draw(key, 2 * p + 1);
    double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    double z0 = r * cos(two_pi * u2);
    double z1 = r * sin(two_pi * u2);
    out[2 * p] = f32_to_bf16_rne((float)(z0 * (double)std));
    if (2 * p + 1 < n) {
      out[2 * p + 1] = f32_to_bf16_rne((float)(z1 * (double)std));
    }
  }
}

// Constant bf16 value (RMSNorm gains).
void synth_const_bf16(uint16_t* out, size_t n, float value) {
  uint16_t v = f32_to_bf16_rne(value);
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i++) {
    out[i] = v;
  }
}

// Uniform bytes in [lo, hi] (MXFP4 code pairs: [0,255]; e8m0 scales).
void synth_uniform_u8(
    uint8_t* out, size_t n, uint64_t seed, uint64_t stream, uint32_t lo,
    uint32_t hi
) {
  const uint64_t key = mix64(seed * PHI + stream);
  const uint64_t span = (uint64_t)(hi - lo) + 1;
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; i++) {
    out[i] = (uint8_t)(lo + draw(key, i) % span);
  }
}
