// Order-preserving keys for exact selection over FP32 scores.
//
// order_key maps a float to a uint32 whose unsigned order is the float order
// (-inf lowest finite-side, +inf highest), with NaN below everything.  A
// selection composite packs (order_key(v), index) into one uint64 whose
// unsigned order is "larger value first, then smaller index": the tie rule of
// the exact top-k.  Composites of distinct indices are distinct, so a rank in
// composite order names exactly one element.
#pragma once
#include <cstdint>

namespace b200 {

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;  // NaN sorts below everything
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t select_composite(float v, int index) {
  return (uint64_t(order_key(v)) << 32) | uint32_t(0xFFFFFFFFu - uint32_t(index));
}

__device__ __forceinline__ int composite_index(uint64_t c) { return int(0xFFFFFFFFu - uint32_t(c)); }

__device__ __forceinline__ float composite_value(uint64_t c) { return key_value(uint32_t(c >> 32)); }

}  // namespace b200
