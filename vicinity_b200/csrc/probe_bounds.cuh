// Pruning bounds of one probe, shared by the probe selection kernels.
//
// lb bounds every float ADC distance of the list from below: (|r| - R_l)^2
// less the float sum's rounding.  For 4-bit tables the quantised distance
// (pq_simd.rs:576-769) can lie below the float one by up to half a
// quantisation step per subspace, M scale / 2 with scale = range / 255 of the
// query's table; the table is not built yet, but every entry is at most gmax
// = (max_m |r_m| + C)^2 (C the largest codeword norm of any subspace, times
// the rounding of the entry's float sum), so scale <= gmax / 255.  A flat
// table (range < 2^-23) is quantised with scale 1, all entries 0; its distance
// M gmin is within M 2^-23 of the float sum, covered by a scale of at least
// 2^-22.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace vg {

__device__ __forceinline__ float lb_from_norm(double sq, float radius, int M, int dsub) {
  const double gap = sqrt(sq) - static_cast<double>(radius);
  double b = gap > 0.0 ? gap * gap : 0.0;
  b *= 1.0 - (static_cast<double>(M + dsub + 2) * 5.9604644775390625e-8 + 1e-12);
  return __double2float_rd(b);
}

__device__ __forceinline__ float lbq_from_lb(float lb, double gmax, int M, int dsub) {
  gmax *= 1.0 + static_cast<double>(dsub + 3) * 5.9604644775390625e-8;
  const double scale = fmax(gmax * (1.0 + 1e-5) / 255.0, 2.384185791015625e-7);
  const double b = static_cast<double>(lb) * (1.0 - 16 * 5.9604644775390625e-8) - 0.5 * M * scale * (1.0 + 1e-5);
  return __double2float_rd(b);
}

// gmax from smax >= max_m |r_m|^2 and C, every operation rounded up
__device__ __forceinline__ double table_max_bound(float smax, float C) {
  const float e = __fadd_ru(__fsqrt_ru(smax), C);
  return static_cast<double>(__fmul_ru(e, e));
}

// Store the bounds lb / lbq and the record of probe list l at index o of the
// bound arrays (zeros and an empty record for a padding slot or a list of
// another rank).  Called by one lane.
__device__ __forceinline__ void store_probe_bound(uint32_t l, bool real, size_t o, float lbf, float lbq,
                                                  const ProbeBoundArgs &bnd) {
  if (!real || (bnd.owner && !bnd.owner[l])) {
    bnd.lb[o] = 0.0f;
    if (bnd.lbq) bnd.lbq[o] = 0.0f;
    if (bnd.rec) bnd.rec[o] = ProbeRec{0xffffffffu, 0u, 0ull, 0ull, 0.0f, 0u};
    return;
  }
  bnd.lb[o] = lbf;
  if (bnd.lbq) bnd.lbq[o] = lbq;
  if (bnd.rec) {
    const uint64_t beg = bnd.list_off[l];
    bnd.rec[o] = ProbeRec{l, static_cast<uint32_t>(bnd.list_off[l + 1] - beg), beg, bnd.code_off[l], lbf, 0u};
  }
}

// The exact coarse dot product q . c (sum in j order from +0, every product
// and add rounded separately: the reference's scalar dot) and, from the same
// pass over c, the bounds of list l: lb from |q - c|^2 (double), and for 4-bit
// tables (bnd.lbq set) lbq from the largest subvector norm.  q in shared
// memory; c = cent + l d, read 32 floats ahead when rows are 16-byte aligned.
__device__ __forceinline__ float exact_dot_and_bounds(const float *q, const float *__restrict__ cent, int d,
                                                      bool vec, uint32_t l, const ProbeBoundArgs &bnd, float &lbf,
                                                      float &lbq) {
  const float *c = cent + static_cast<size_t>(l) * d;
  float dot = 0.0f, smax = 0.0f, sacc = 0.0f;
  double sq = 0.0;
  int cnt = 0;
  const bool want_q = bnd.lbq != nullptr;
  auto acc = [&](float qj, float cj) {
    dot = __fadd_rn(dot, __fmul_rn(qj, cj));
    const float r = __fsub_rn(qj, cj);
    sq += static_cast<double>(r) * r;
    if (want_q) {
      sacc = __fmaf_ru(r, r, sacc);
      if (++cnt == bnd.dsub) {
        smax = fmaxf(smax, sacc);
        sacc = 0.0f;
        cnt = 0;
      }
    }
  };
  int j = 0;
  if (vec) {
    const float4 *c4 = reinterpret_cast<const float4 *>(c);
    const float4 *q4 = reinterpret_cast<const float4 *>(q);
    for (; j + 32 <= d; j += 32) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(c4 + (j >> 2) + u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 w = q4[(j >> 2) + u];
        acc(w.x, v[u].x);
        acc(w.y, v[u].y);
        acc(w.z, v[u].z);
        acc(w.w, v[u].w);
      }
    }
  }
  for (; j < d; ++j) acc(q[j], __ldg(c + j));
  lbf = lb_from_norm(sq, bnd.radius[l], bnd.M, bnd.dsub);
  lbq = want_q ? lbq_from_lb(lbf, table_max_bound(smax, bnd.sub_radius[bnd.M]), bnd.M, bnd.dsub) : 0.0f;
  return dot;
}

// Bounds and record of probe list l of the query in qs (shared memory, d
// floats), written at index o of the bound arrays.  Called by one lane.
__device__ __forceinline__ void write_probe_bound(const float *qs, const float *__restrict__ cent, int d, bool cvec,
                                                  uint32_t l, bool real, size_t o, const ProbeBoundArgs &bnd) {
  if (!real || (bnd.owner && !bnd.owner[l])) {
    store_probe_bound(l, false, o, 0.0f, 0.0f, bnd);
    return;
  }
  const float *c = cent + static_cast<size_t>(l) * d;
  // |r|^2 in double; for 4-bit tables also the largest subvector norm
  // squared (float, rounded up), subspace by subspace in j order
  double sq = 0.0;
  float smax = 0.0f, sacc = 0.0f;
  int cnt = 0;
  const bool want_q = bnd.lbq != nullptr;
  auto acc = [&](float r) {
    sq += static_cast<double>(r) * r;
    if (want_q) {
      sacc = __fmaf_ru(r, r, sacc);
      if (++cnt == bnd.dsub) {
        smax = fmaxf(smax, sacc);
        sacc = 0.0f;
        cnt = 0;
      }
    }
  };
  int j = 0;
  if (cvec) {  // 32 floats of the centroid row in flight at a time
    const float4 *c4 = reinterpret_cast<const float4 *>(c);
    const float4 *q4 = reinterpret_cast<const float4 *>(qs);
    for (; j + 32 <= d; j += 32) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(c4 + (j >> 2) + u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 a = q4[(j >> 2) + u];
        acc(__fsub_rn(a.x, v[u].x));
        acc(__fsub_rn(a.y, v[u].y));
        acc(__fsub_rn(a.z, v[u].z));
        acc(__fsub_rn(a.w, v[u].w));
      }
    }
  }
  for (; j < d; ++j) acc(__fsub_rn(qs[j], __ldg(c + j)));
  const float lbf = lb_from_norm(sq, bnd.radius[l], bnd.M, bnd.dsub);
  store_probe_bound(l, true, o, lbf,
                    want_q ? lbq_from_lb(lbf, table_max_bound(smax, bnd.sub_radius[bnd.M]), bnd.M, bnd.dsub) : 0.0f,
                    bnd);
}

// sum_j q_j c_j with the sum taken in j order from +0, every product and add
// rounded separately (the reference's dot, simd.rs:83-127 scalar order).  q
// in shared memory; c a row in global memory, read 32 floats ahead when rows
// are 16-byte aligned.
__device__ __forceinline__ float exact_dot(const float *q, const float *__restrict__ c, int d, bool vec) {
  float acc = 0.0f;
  int j = 0;
  if (vec) {
    const float4 *c4 = reinterpret_cast<const float4 *>(c);
    const float4 *q4 = reinterpret_cast<const float4 *>(q);
    for (; j + 32 <= d; j += 32) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(c4 + (j >> 2) + u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 w = q4[(j >> 2) + u];
        acc = __fadd_rn(acc, __fmul_rn(w.x, v[u].x));
        acc = __fadd_rn(acc, __fmul_rn(w.y, v[u].y));
        acc = __fadd_rn(acc, __fmul_rn(w.z, v[u].z));
        acc = __fadd_rn(acc, __fmul_rn(w.w, v[u].w));
      }
    }
  }
  for (; j < d; ++j) acc = __fadd_rn(acc, __fmul_rn(q[j], __ldg(c + j)));
  return acc;
}

}  // namespace vg
