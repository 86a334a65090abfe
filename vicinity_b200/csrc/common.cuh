// Shared device helpers for the vicinity IVF-PQ engine (sm_100a).
//
// Exact-arithmetic rule: the reference (vicinity 0.12.0, Rust) rounds every
// multiply and add separately and sums in index order.  Device code on the
// parity path therefore uses the _rn intrinsics, which the compiler never
// contracts into FMA, and keeps the reference's summation order.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define VG_FULL_MASK 0xffffffffu

namespace vg {

// f32::total_cmp as an unsigned key: negative values flip every bit, others
// set the sign bit, so unsigned order equals total_cmp order (-0.0 < +0.0,
// NaNs at the ends).
__host__ __device__ __forceinline__ uint32_t order_key(float x) {
#ifdef __CUDA_ARCH__
  uint32_t b = __float_as_uint(x);
#else
  uint32_t b;
  __builtin_memcpy(&b, &x, 4);
#endif
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__host__ __device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  __builtin_memcpy(&f, &b, 4);
  return f;
#endif
}

// Candidate key: distance order first, then the 32-bit id.  Unique per id, so
// every selection below has exactly one answer.
__host__ __device__ __forceinline__ uint64_t pack_key(float dist, uint32_t id) {
  return (static_cast<uint64_t>(order_key(dist)) << 32) | id;
}
__host__ __device__ __forceinline__ float key_dist(uint64_t k) {
  return key_to_float(static_cast<uint32_t>(k >> 32));
}
__host__ __device__ __forceinline__ uint32_t key_id(uint64_t k) {
  return static_cast<uint32_t>(k & 0xffffffffu);
}
constexpr uint64_t kEmptyKey = ~0ull;

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int m) {
  return __shfl_xor_sync(VG_FULL_MASK, static_cast<unsigned long long>(v), m);
}
__device__ __forceinline__ uint64_t shfl64(uint64_t v, int src) {
  return __shfl_sync(VG_FULL_MASK, static_cast<unsigned long long>(v), src);
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

}  // namespace vg
