// Packed FP32 pairs (sm_100a `add/sub/mul.rn.f32x2`): one instruction does
// the same IEEE round-to-nearest operation on two independent f32 lanes, so
// each lane's result is bit-identical to the scalar __fadd_rn / __fsub_rn /
// __fmul_rn.  Used where the FP32 issue rate bounds a kernel (ADC table
// build): two table entries per instruction.
#pragma once

#include <cstdint>

namespace vg {

using f32x2 = unsigned long long;  // lo = first lane, hi = second lane

__device__ __forceinline__ f32x2 f2_pack(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ float2 f2_unpack(f32x2 v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

__device__ __forceinline__ f32x2 f2_sub(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ f32x2 f2_mul(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ f32x2 f2_add(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ f32x2 f2_fma(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Two squared distances of one residual subvector q (each element duplicated
// into both lanes) to two codewords c (lane-packed), each in the reference's
// order: ((d0*d0 + d1*d1) + d2*d2) + ...  (the 0 + s first step is exact).
//
// ptxas fuses a packed multiply whose only use is a packed add into one
// packed FMA even when both carry .rn (one rounding instead of two), and
// -fmad=false does not stop it.  Each square is therefore written as
// fma(d, d, z) with z = (-0, -0) supplied at run time: d*d + -0 rounds
// exactly like d*d (an exact +0 product stays +0), the compiler cannot fold
// an addend it does not know, and an FMA result is not contracted further.
template <int D>
__device__ __forceinline__ f32x2 sq_dist_x2(const f32x2 (&q)[D], const f32x2 (&c)[D], f32x2 z) {
  f32x2 d0 = f2_sub(q[0], c[0]);
  f32x2 acc = f2_fma(d0, d0, z);
#pragma unroll
  for (int j = 1; j < D; ++j) {
    f32x2 dj = f2_sub(q[j], c[j]);
    acc = f2_add(acc, f2_fma(dj, dj, z));
  }
  return acc;
}

}  // namespace vg
