// Exact fixed-point sums in shared memory, shared by the destination-grouped
// sweep (mirror.cu) and the fused pipeline training step (train.cu).
//
// A unit's shared accumulator is two 32-bit words: lo in units of 2^-F and
// hi in units of 1.0 (2^F lo units), F = 28 or 31 fractional bits. Shared
// integer atomics are native, where a float add is a compare-and-swap loop.
// A product of magnitude < 1 is rounded to the nearest lo unit (exact when
// its 24-bit mantissa ends at or above 2^-F; otherwise an error of at most
// 2^-(F+1)) and added to lo; the adding thread sees a signed wrap of lo
// exactly, from the value its atomic returns, and carries 2^(32-F) into hi.
// A product in [1, 2^20) is a multiple of 2^-23, so its fixed value is
// exact: the part above 2^F units goes to hi, the rest to lo. A product that
// is not finite or is >= 2^20 goes to a float side accumulator. A unit's
// value is (hi * 2^F + lo) lo units, exact in int64.
#pragma once

#include "pxb_common.cuh"

namespace pxb {

template <int F>
__device__ __forceinline__ float fix_scale() {
  return F == 31 ? 2147483648.0f : 268435456.0f;
}

template <int F>
__device__ __forceinline__ void lo_add(int32_t *lo, int32_t *hi, int32_t v) {
  const int32_t old = atomicAdd(lo, v);
  const int32_t now = static_cast<int32_t>(static_cast<uint32_t>(old) + static_cast<uint32_t>(v));
  constexpr int32_t carry = 1 << (32 - F);  // 2^32 lo units, in units of 1.0
  if (((old ^ now) & (v ^ now)) < 0) atomicAdd(hi, v > 0 ? carry : -carry);
}

template <int F>
__device__ __forceinline__ void fixed_add(int32_t *lo, int32_t *hi, float *gf, float p) {
  const float ap = fabsf(p);
  if (ap < 1.0f) {
    lo_add<F>(lo, hi, __float2int_rn(p * fix_scale<F>()));
  } else if (ap < 1048576.0f) {
    const long long v = __float2ll_rn(p * fix_scale<F>());
    atomicAdd(hi, static_cast<int32_t>(v >> F));
    lo_add<F>(lo, hi, static_cast<int32_t>(v & ((1ll << F) - 1)));
  } else {
    atomicAdd(gf, p);
  }
}

}  // namespace pxb
