// Internal helpers shared by the libpxb translation units: status handling,
// launch geometry, monoid atomics and the Philox-4x32-10 word generator.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/pxb.h"

namespace pxb {

// Thread-local message of the last failing call on this host thread.
void set_error(const char *fmt, ...);
const char *last_error();

// Number of SMs of the current device, cached per device.
int sm_count();

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

#define PXB_REQUIRE(cond, ...)          \
  do {                                  \
    if (!(cond)) {                      \
      ::pxb::set_error(__VA_ARGS__);    \
      return PXB_EINVAL;                \
    }                                   \
  } while (0)

#define PXB_CUDA(call)                                                    \
  do {                                                                    \
    cudaError_t err_ = (call);                                            \
    if (err_ != cudaSuccess) {                                            \
      ::pxb::set_error("%s failed: %s", #call, cudaGetErrorString(err_)); \
      return PXB_ECUDA;                                                   \
    }                                                                     \
  } while (0)

#define PXB_LAUNCHED(name)                                                  \
  do {                                                                      \
    cudaError_t err_ = cudaGetLastError();                                  \
    if (err_ != cudaSuccess) {                                              \
      ::pxb::set_error("launch of %s failed: %s", name, cudaGetErrorString(err_)); \
      return PXB_ECUDA;                                                     \
    }                                                                       \
  } while (0)

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid for a grid-stride kernel: enough CTAs to fill every SM `per_sm` times,
// never more than the work needs.
inline int grid_for(int64_t work_items, int items_per_cta, int per_sm) {
  int64_t need = (work_items + items_per_cta - 1) / items_per_cta;
  int64_t full = static_cast<int64_t>(sm_count()) * per_sm;
  if (need < 1) need = 1;
  return static_cast<int>(need < full ? need : full);
}

// ---------------------------------------------------------------------------
// monoid combine (src/plastax/monoid.py:27-59)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float monoid_identity(int monoid) {
  return monoid == PXB_MONOID_SUM ? 0.0f
       : monoid == PXB_MONOID_MAX ? -__int_as_float(0x7f800000)
                                  : __int_as_float(0x7f800000);
}

__device__ __forceinline__ float monoid_pair(int monoid, float a, float b) {
  return monoid == PXB_MONOID_SUM ? a + b : monoid == PXB_MONOID_MAX ? fmaxf(a, b) : fminf(a, b);
}

// Float max/min through integer atomics: for v >= 0 the signed-int order of
// the bit patterns is the float order; for v < 0 the unsigned order is the
// reverse float order. Valid for a target that starts at a non-NaN value.
__device__ __forceinline__ void atomic_max_f32(float *addr, float v) {
  if (!(v < 0.0f)) atomicMax(reinterpret_cast<int *>(addr), __float_as_int(v));
  else atomicMin(reinterpret_cast<unsigned int *>(addr), __float_as_uint(v));
}
__device__ __forceinline__ void atomic_min_f32(float *addr, float v) {
  if (!(v < 0.0f)) atomicMin(reinterpret_cast<int *>(addr), __float_as_int(v));
  else atomicMax(reinterpret_cast<unsigned int *>(addr), __float_as_uint(v));
}

template <int MONOID>
__device__ __forceinline__ void atomic_combine(float *addr, float v) {
  if (MONOID == PXB_MONOID_SUM) atomicAdd(addr, v);
  else if (MONOID == PXB_MONOID_MAX) atomic_max_f32(addr, v);
  else atomic_min_f32(addr, v);
}

template <int MONOID>
__device__ __forceinline__ float combine2(float a, float b) {
  if (MONOID == PXB_MONOID_SUM) return a + b;
  if (MONOID == PXB_MONOID_MAX) return fmaxf(a, b);
  return fminf(a, b);
}

// ---------------------------------------------------------------------------
// unit activation functions and their derivative from the activation value
// ---------------------------------------------------------------------------
// A unit's activation kind from an apply's `act_kind` code and the unit's
// role (0 hidden, 1 input, 2 output): the code's low byte is the kind, and a
// non-zero second byte (kind + 1) overrides it for output units.
__device__ __forceinline__ int unit_act_kind(int32_t code, uint8_t role) {
  const int out = (code >> 8) & 0xff;
  return (role == 2 && out != 0) ? out - 1 : (code & 0xff);
}

__host__ __device__ __forceinline__ bool act_code_ok(int32_t code) {
  return code >= 0 && (code & 0xff) <= 3 && ((code >> 8) & 0xff) <= 4 && (code >> 16) == 0;
}

__device__ __forceinline__ float act_fn(int kind, float x) {
  switch (kind) {
    case PXB_ACT_TANH: return tanhf(x);
    case PXB_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case PXB_ACT_SIGMOID: return 1.0f / (1.0f + expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ float act_prime_from_act(int kind, float a) {
  switch (kind) {
    case PXB_ACT_TANH: return __fsub_rn(1.0f, __fmul_rn(a, a));
    case PXB_ACT_RELU: return a > 0.0f ? 1.0f : 0.0f;
    case PXB_ACT_SIGMOID: return __fmul_rn(a, __fsub_rn(1.0f, a));
    default: return 1.0f;
  }
}

// ---------------------------------------------------------------------------
// Philox-4x32-10, first output word (src/plastax/rng.py:109-142): counter
// block (ctr_lo, ctr_hi, seed_lo, seed_hi), key (seed_lo, seed_hi), the
// Salmon et al. (SC'11) multipliers and Weyl key increments.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t philox32(uint64_t seed, uint64_t counter) {
  uint32_t x0 = static_cast<uint32_t>(counter), x1 = static_cast<uint32_t>(counter >> 32);
  uint32_t x2 = static_cast<uint32_t>(seed), x3 = static_cast<uint32_t>(seed >> 32);
  uint32_t k0 = x2, k1 = x3;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * x0;
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * x2;
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    x0 = hi1 ^ x1 ^ k0;
    x1 = lo1;
    x2 = hi0 ^ x3 ^ k1;
    x3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return x0;
}

// float32(word >> 8) * 2^-24: exact, 24 bits of mantissa.
__host__ __device__ __forceinline__ float unit_float(uint32_t word) {
  return static_cast<float>(word >> 8) * (1.0f / 16777216.0f);
}

// min(uint32(u * n), n - 1) with one float32 multiply (no contraction).
__device__ __forceinline__ uint32_t uniform_int(float u, uint32_t n) {
  const float scaled = __fmul_rn(u, static_cast<float>(n));
  uint32_t v = static_cast<uint32_t>(scaled);
  return v < n - 1 ? v : n - 1;
}

// The site seed of (network_seed, step, stream, key): the keyed
// step/stream word in the high limb, the proposer key in the low limb.
__host__ __device__ __forceinline__ uint64_t site_seed(uint64_t network_seed, uint32_t step,
                                                       uint32_t stream, uint32_t key) {
  const uint64_t ctr = (static_cast<uint64_t>(step) << 8) | (stream & 0xFFu);
  const uint64_t hi = philox32(network_seed, ctr);
  return (hi << 32) | key;
}

__device__ __forceinline__ uint32_t site_draw(uint64_t seed, uint32_t j, uint32_t sub) {
  return philox32(seed, (static_cast<uint64_t>(j) << 16) | sub);
}

}  // namespace pxb
