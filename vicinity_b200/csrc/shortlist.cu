// Probe shortlist over a row-major matrix of approximate coarse products
// (binary16 or f32), as the tensor-core GEMM of tc_select.cu writes it.
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "probe_bounds.cuh"
#include "topk.cuh"

namespace vg {

namespace {
constexpr int kSelectWarps = 8;
}  // namespace

// ---------------------------------------------------------------------------
// Probe shortlist from approximate coarse products (search.rs:1602-1617).
//
// s[row][l] approximates q . c_l (a tensor-core product) within eps(row) =
// rel |q| cmax + abs_coef (1 + cmax) + 2^-20, the coefficients set by the
// caller for the operand and result formats (rounding or truncation of both
// operands, accumulation, the result's own rounding, the rounding of the exact
// sequential dot and of the subtractions from 1; binary16 adds an absolute
// term for subnormal operands).  With
// A = 1 - s, every probe of the exact top-P has A <= A_P + 2 eps, where A_P is
// the P-th smallest A: those are gathered (under an upper bound on A_P taken
// from the lanes' 2R smallest), re-scored with the reference's arithmetic --
// 1 - (sum_j q_j c_j in j order, separately rounded products and adds) -- and
// the exact top-P is kept.  A row whose window overflows the buffer, or whose
// inputs are not finite, is scored exactly over every centroid.
// ---------------------------------------------------------------------------
namespace {
constexpr int kShortBuf = 256;  // gathered candidates per warp
constexpr int kChunkBuf = 256;  // candidate chunks per warp (chunk-maxima path)

// 1 - sum_j q_j c_j in the reference's order (the exact coarse distance).
__device__ __forceinline__ float exact_one_minus_dot(const float *q, const float *__restrict__ c, int d, bool vec) {
  return __fsub_rn(1.0f, exact_dot(q, c, d, vec));
}

// Four products of a row as floats: from a float4, or from four halves.
__device__ __forceinline__ float4 quad_to_float(const float4 v) { return v; }
__device__ __forceinline__ float4 quad_to_float(const uint2 v) {
  const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ float elem_to_float(float v) { return v; }
__device__ __forceinline__ float elem_to_float(__half v) { return __half2float(v); }
template <typename TS> struct QuadOf { using type = float4; };
template <> struct QuadOf<__half> { using type = uint2; };

// Visit columns [0, L) of a row of TS (float or half), four at a time:
// fn(col, v, valid[4]) with v the four approximate products.  Trip counts are
// warp-uniform (fn may use warp votes); rows must be aligned to four elements
// with L % 4 == 0 when vec is set.  The last visit (kLast) streams the row
// past L2 with evict-first loads.
template <bool kLast, typename TS, typename F>
__device__ __forceinline__ void for_each_quad(const TS *__restrict__ srow, size_t L, bool vec, int lane, F &&fn) {
  using Q = typename QuadOf<TS>::type;
  if (vec) {
    const Q *r4 = reinterpret_cast<const Q *>(srow);
    const size_t n4 = L >> 2;
    size_t b = 0;
    for (; b + 128 <= n4; b += 128) {
      Q v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = kLast ? __ldcs(r4 + b + u * 32 + lane) : __ldg(r4 + b + u * 32 + lane);
#pragma unroll
      for (int u = 0; u < 4; ++u) fn((b + u * 32 + lane) * 4, quad_to_float(v[u]), true, true, true, true);
    }
    for (; b < n4; b += 32) {
      const size_t i = b + lane;
      Q v{};
      if (i < n4) v = kLast ? __ldcs(r4 + i) : __ldg(r4 + i);
      fn(i * 4, quad_to_float(v), i < n4, i < n4, i < n4, i < n4);
    }
  } else {
    for (size_t b = 0; b < L; b += 128) {
      const size_t c = b + lane * 4;
      float4 v;
      v.x = c < L ? elem_to_float(srow[c]) : 0.f;
      v.y = c + 1 < L ? elem_to_float(srow[c + 1]) : 0.f;
      v.z = c + 2 < L ? elem_to_float(srow[c + 2]) : 0.f;
      v.w = c + 3 < L ? elem_to_float(srow[c + 3]) : 0.f;
      fn(c, v, c < L, c + 1 < L, c + 2 < L, c + 3 < L);
    }
  }
}

// Visit a half row of L % 4 == 0 columns, 8-byte aligned, as raw quads: fn(col,
// lo, hi, valid) with lo / hi the half2 pairs (col, col + 1) and (col + 2, col + 3).
// Trip counts are warp-uniform.  Blocks of 128 quads are software-pipelined:
// the next block's loads are in flight while fn runs over the current one.
template <bool kLast, typename F>
__device__ __forceinline__ void for_each_half_quad(const __half *__restrict__ srow, size_t L, int lane, F &&fn) {
  const uint2 *r4 = reinterpret_cast<const uint2 *>(srow);
  const size_t n4 = L >> 2;
  auto load = [&](size_t i) { return kLast ? __ldcs(r4 + i) : __ldg(r4 + i); };
  size_t b = 0;
  if (n4 >= 128) {
    uint2 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = load(u * 32 + lane);
    for (;; b += 128) {  // v holds block b, which is whole
      const bool more = b + 256 <= n4;
      uint2 w[4];
      if (more) {
#pragma unroll
        for (int u = 0; u < 4; ++u) w[u] = load(b + 128 + u * 32 + lane);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        fn((b + u * 32 + lane) * 4, *reinterpret_cast<const __half2 *>(&v[u].x),
           *reinterpret_cast<const __half2 *>(&v[u].y), true);
      if (!more) break;
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = w[u];
    }
    b += 128;
  }
  for (; b < n4; b += 32) {
    const size_t i = b + lane;
    uint2 v = make_uint2(0u, 0u);
    if (i < n4) v = kLast ? __ldcs(r4 + i) : __ldg(r4 + i);
    fn(i * 4, *reinterpret_cast<const __half2 *>(&v.x), *reinterpret_cast<const __half2 *>(&v.y), i < n4);
  }
}

template <int R, typename TS>
__global__ void __launch_bounds__(kSelectWarps * 32, 4)
    shortlist_kernel(const TS *__restrict__ s, size_t rows, size_t L, size_t ld, const float *__restrict__ qn,
                     int d, const float *__restrict__ cent, const float *__restrict__ cmax_p, double rel,
                     double abs_coef, int k, uint32_t *__restrict__ out_ids, float *__restrict__ out_dist,
                     size_t out_ld, const ProbeBoundArgs bnd, const __half *__restrict__ cmx, size_t cstride) {
  extern __shared__ __align__(16) unsigned char sh[];
  constexpr int R2 = 2 * R;
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const size_t row = static_cast<size_t>(blockIdx.x) * kSelectWarps + warp;
  if (row >= rows) return;
  uint32_t *buf = reinterpret_cast<uint32_t *>(sh) + static_cast<size_t>(warp) * kShortBuf;
  const int dpad = (d + 3) & ~3;
  float *qs = reinterpret_cast<float *>(reinterpret_cast<uint32_t *>(sh) + kSelectWarps * kShortBuf) +
              static_cast<size_t>(warp) * dpad;
  uint32_t *cl = reinterpret_cast<uint32_t *>(reinterpret_cast<float *>(reinterpret_cast<uint32_t *>(sh) +
                                                                        kSelectWarps * kShortBuf) +
                                              static_cast<size_t>(kSelectWarps) * dpad) +
                 static_cast<size_t>(warp) * kChunkBuf;  // candidate chunk ids
  // pruning bounds of the gathered candidates, by buffer position
  float *lbv = reinterpret_cast<float *>(cl + static_cast<size_t>(kSelectWarps - warp) * kChunkBuf) +
               static_cast<size_t>(warp) * 2 * kShortBuf;
  float *lbqv = lbv + kShortBuf;
  const TS *srow = s + row * ld;
  const float *qrow = qn + row * d;
  for (int j = lane; j < d; j += 32) qs[j] = qrow[j];
  __syncwarp();
  double qq = 0.0;
  for (int j = lane; j < d; j += 32) qq += static_cast<double>(qs[j]) * qs[j];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) qq += __shfl_xor_sync(VG_FULL_MASK, qq, off);
  const double cmax = static_cast<double>(*cmax_p);
  const double eps = rel * sqrt(qq) * cmax * 1.01 + abs_coef * (1.0 + cmax) + 1.0 / 1048576;
  bool exact_all = !(eps < 1.0);  // non-finite or useless bound
  const bool svec = (L & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(s) % (4 * sizeof(TS))) == 0;
  const bool cvec = (d & 3) == 0 && (reinterpret_cast<uintptr_t>(cent) & 15) == 0;

  // pass 1: each lane's 2R smallest approximate distances (values only: the
  // bound needs no list ids; NaN never enters, +inf marks an empty slot)
  const float kInf = __int_as_float(0x7f800000);
  float a[R2];
#pragma unroll
  for (int r = 0; r < R2; ++r) a[r] = kInf;
  auto insert = [&](float x) {
#pragma unroll
    for (int r = 0; r < R2; ++r) {
      const float lo = fminf(x, a[r]);
      x = fmaxf(x, a[r]);
      a[r] = lo;
    }
  };
  bool half_fast = false;
  if constexpr (std::is_same<TS, __half>::value) half_fast = svec;
  // chunk maxima: the largest product of every 32 columns, a subset of the
  // products, so their P-th largest still bounds A_P, and a chunk whose
  // maximum is below the window holds no candidate
  const __half *crow = cmx ? cmx + row * cstride : nullptr;
  const size_t nch = ((L + 127) / 128) * 4;  // chunk maxima per row, whole tiles of 4
  const bool chunked = half_fast && crow != nullptr;
  if (!exact_all && half_fast) {
    if constexpr (std::is_same<TS, __half>::value) {
      // the largest products are the smallest distances: keep the 2R largest
      // of each half2 sublane with packed max / min (NaN never enters), then
      // the 2R largest of the lane's two sorted sublanes (bitonic step)
      const __half2 ninf = __halves2half2(__ushort_as_half(0xFC00u), __ushort_as_half(0xFC00u));
      __half2 a2[R2];
#pragma unroll
      for (int r = 0; r < R2; ++r) a2[r] = ninf;
      auto insert2 = [&](__half2 x) {
#pragma unroll
        for (int r = 0; r < R2; ++r) {
          const __half2 hi = __hmax2(x, a2[r]);
          x = __hmin2(x, a2[r]);
          a2[r] = hi;
        }
      };
      for_each_half_quad<false>(chunked ? crow : srow, chunked ? nch : L, lane,
                                [&](size_t, __half2 lo, __half2 hi, bool ok) {
                                  insert2(ok ? lo : ninf);
                                  insert2(ok ? hi : ninf);
                                });
#pragma unroll
      for (int r = 0; r < R2; ++r) {
        const float s = fmaxf(__low2float(a2[r]), __high2float(a2[R2 - 1 - r]));
        a[r] = s == -kInf ? kInf : __fsub_rn(1.0f, s);
      }
    }
  } else if (!exact_all) {
    for_each_quad<false, TS>(srow, L, svec, lane, [&](size_t, float4 v, bool ox, bool oy, bool oz, bool ow) {
      if (ox) insert(__fsub_rn(1.0f, v.x));
      if (oy) insert(__fsub_rn(1.0f, v.y));
      if (oz) insert(__fsub_rn(1.0f, v.z));
      if (ow) insert(__fsub_rn(1.0f, v.w));
    });
  }
  // the k-th smallest of the lanes' 32 x 2R values: bisection on the order
  // key, counting the values at or below the midpoint over the warp
  // (0xffffffff marks an empty slot and is never counted)
  uint32_t okey[R2];
  int have = 0;
#pragma unroll
  for (int r = 0; r < R2; ++r) {
    okey[r] = a[r] == kInf ? 0xffffffffu : order_key(a[r]);
    have += okey[r] != 0xffffffffu;
  }
  const bool full = __reduce_add_sync(VG_FULL_MASK, static_cast<unsigned>(have)) >= static_cast<unsigned>(k);
  uint32_t klo = 0, khi = 0xfffffffeu;
  while (full && klo < khi) {
    const uint32_t mid = klo + ((khi - klo) >> 1);
    int c = 0;
#pragma unroll
    for (int r = 0; r < R2; ++r) c += okey[r] <= mid;
    if (__reduce_add_sync(VG_FULL_MASK, static_cast<unsigned>(c)) >= static_cast<unsigned>(k))
      khi = mid;
    else
      klo = mid + 1;
  }
  // every exact top-k list has approximate distance <= limit (rounded up)
  const float limit = !full ? __int_as_float(0x7f800000)
                            : __double2float_ru(static_cast<double>(key_to_float(klo)) + 2.0 * eps);
  if (!(limit < __int_as_float(0x7f800000)) && full) exact_all = true;

  int n = 0;
  auto gather = [&](size_t c, float4 v, bool ox, bool oy, bool oz, bool ow) {
    const bool t[4] = {ox && !(__fsub_rn(1.0f, v.x) > limit), oy && !(__fsub_rn(1.0f, v.y) > limit),
                       oz && !(__fsub_rn(1.0f, v.z) > limit), ow && !(__fsub_rn(1.0f, v.w) > limit)};
    if (!__any_sync(VG_FULL_MASK, t[0] || t[1] || t[2] || t[3])) return;  // nearly every quad
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const unsigned m = __ballot_sync(VG_FULL_MASK, t[h]);
      const int pos = n + __popc(m & ((1u << lane) - 1u));
      if (t[h] && pos < kShortBuf) buf[pos] = static_cast<uint32_t>(c + h);
      n += __popc(m);
    }
  };
  if (!exact_all && half_fast) {
    if constexpr (std::is_same<TS, __half>::value) {
      // a product below s_lo cannot give a distance <= limit (1 - s > limit
      // by more than a rounding of 1 - s): one packed test per pair, the
      // exact test only in quads where a lane may hold a candidate
      const float s_lo = __double2float_rd(1.0 - static_cast<double>(limit) -
                                           1e-6 * (1.0 + fabs(static_cast<double>(limit))));
      const __half2 slo2 = __half2half2(__float2half_rd(s_lo));
      if (chunked) {
        // the ids of chunks whose maximum reaches s_lo (no product read yet),
        // in ascending order (lane-major: each lane holds four consecutive
        // chunks), then one chunk per lane, its 64 bytes in flight at once;
        // the candidates land in the buffer in ascending list order
        const __half slo = __float2half_rd(s_lo);
        int nc = 0;
        for_each_half_quad<false>(crow, nch, lane, [&](size_t c4, __half2 lo, __half2 hi, bool ok) {
          const bool mt[4] = {ok && !__hlt(__low2half(lo), slo), ok && !__hlt(__high2half(lo), slo),
                              ok && !__hlt(__low2half(hi), slo), ok && !__hlt(__high2half(hi), slo)};
          const int cnt = static_cast<int>(mt[0]) + mt[1] + mt[2] + mt[3];
          if (!__any_sync(VG_FULL_MASK, cnt != 0)) return;
          int incl = cnt;
#pragma unroll
          for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(VG_FULL_MASK, incl, off);
            if (lane >= off) incl += y;
          }
          int pos = nc + incl - cnt;
#pragma unroll
          for (int h = 0; h < 4; ++h)
            if (mt[h]) {
              if (pos < kChunkBuf) cl[pos] = static_cast<uint32_t>(c4 + h);
              ++pos;
            }
          nc += __shfl_sync(VG_FULL_MASK, incl, 31);
        });
        __syncwarp();
        if (nc > kChunkBuf) {
          exact_all = true;  // a window this wide: every list scored exactly
        } else {
          const bool vload = (L & 7) == 0 && (reinterpret_cast<uintptr_t>(srow) & 15) == 0;
          for (int i0 = 0; i0 < nc; i0 += 32) {
            const bool have = i0 + lane < nc;
            const size_t c0 = have ? static_cast<size_t>(cl[i0 + lane]) * 32 : 0;
            uint32_t w[16];  // 32 binary16 products
            if (have && vload && c0 + 32 <= L) {
              const uint4 *src = reinterpret_cast<const uint4 *>(srow + c0);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint4 x = __ldcs(src + u);
                w[4 * u] = x.x;
                w[4 * u + 1] = x.y;
                w[4 * u + 2] = x.z;
                w[4 * u + 3] = x.w;
              }
            } else {
#pragma unroll
              for (int u = 0; u < 16; ++u) {
                const size_t a = c0 + 2 * u, b = a + 1;
                const unsigned short lo16 = have && a < L ? __half_as_ushort(srow[a]) : 0xFC00u;  // -inf past L
                const unsigned short hi16 = have && b < L ? __half_as_ushort(srow[b]) : 0xFC00u;
                w[u] = static_cast<uint32_t>(lo16) | (static_cast<uint32_t>(hi16) << 16);
              }
            }
            uint32_t take = 0;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[u]));
              take |= (have && !(__fsub_rn(1.0f, f.x) > limit) ? 1u : 0u) << (2 * u);
              take |= (have && !(__fsub_rn(1.0f, f.y) > limit) ? 1u : 0u) << (2 * u + 1);
            }
            // lanes' candidates side by side: exclusive prefix sum of the counts
            const int cnt = __popc(take);
            int incl = cnt;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
              const int y = __shfl_up_sync(VG_FULL_MASK, incl, off);
              if (lane >= off) incl += y;
            }
            int pos = n + incl - cnt;
            while (take) {
              const int j = __ffs(take) - 1;
              take &= take - 1;
              if (pos < kShortBuf) buf[pos] = static_cast<uint32_t>(c0 + j);
              ++pos;
            }
            n += __shfl_sync(VG_FULL_MASK, incl, 31);
          }
        }
      } else {
      for_each_half_quad<true>(srow, L, lane, [&](size_t c, __half2 lo, __half2 hi, bool ok) {
        const bool maybe = ok && (!__hblt2(lo, slo2) || !__hblt2(hi, slo2));
        if (!__any_sync(VG_FULL_MASK, maybe)) return;
        const float2 fl = __half22float2(lo), fh = __half22float2(hi);
        gather(c, make_float4(fl.x, fl.y, fh.x, fh.y), ok, ok, ok, ok);
      });
      }
    }
  } else if (!exact_all) {
    for_each_quad<true, TS>(srow, L, svec, lane, gather);
  }
  if (!exact_all) exact_all = n > kShortBuf;
  // The row of products is not read again: drop its lines from L2 without
  // writing them back (whole 128-byte lines inside the row only), so the
  // search kernels that follow do not pay for its write-back.
  __syncwarp();
  {
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(srow) + 127) & ~uintptr_t(127);
    const uintptr_t hi = (reinterpret_cast<uintptr_t>(srow + L)) & ~uintptr_t(127);
    for (uintptr_t a = lo + 128 * static_cast<uintptr_t>(lane); a < hi; a += 128 * 32)
      asm volatile("discard.global.L2 [%0], 128;" ::"l"(a) : "memory");
  }
  __syncwarp();
  WarpTopK<R> tk;
  tk.init();
  // the chunked gather leaves the buffer in ascending list order, so keys of
  // (distance, buffer position) order as (distance, list) do; the pruning
  // bounds then come from the same pass over each centroid row
  const bool by_pos = !exact_all && chunked && bnd.lb != nullptr;
  if (by_pos) {
    for (int i0 = 0; i0 < n; i0 += 32) {
      uint64_t key = kEmptyKey;
      const int i = i0 + lane;
      if (i < n) {
        float lbf, lbq;
        const float dot = exact_dot_and_bounds(qs, cent, d, cvec, buf[i], bnd, lbf, lbq);
        lbv[i] = lbf;
        lbqv[i] = lbq;
        key = pack_key(__fsub_rn(1.0f, dot), static_cast<uint32_t>(i));
      }
      tk.add(key);
    }
  } else if (!exact_all) {
    for (int i0 = 0; i0 < n; i0 += 32) {
      uint64_t key = kEmptyKey;
      if (i0 + lane < n) {
        const uint32_t c = buf[i0 + lane];
        key = pack_key(exact_one_minus_dot(qs, cent + static_cast<size_t>(c) * d, d, cvec), c);
      }
      tk.add(key);
    }
  } else {
    for (size_t c0 = 0; c0 < L; c0 += 32) {
      const size_t c = c0 + lane;
      tk.add(c < L ? pack_key(exact_one_minus_dot(qs, cent + c * d, d, cvec), static_cast<uint32_t>(c)) : kEmptyKey);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    if (i < k) {
      const uint64_t key = tk.v[r];
      const bool real = key != kEmptyKey;
      const uint32_t pos = key_id(key);
      const uint32_t l = !real ? 0xffffffffu : by_pos ? buf[pos] : pos;
      out_ids[row * out_ld + i] = l;
      out_dist[row * out_ld + i] = real ? key_dist(key) : __int_as_float(0x7f800000);
      if (by_pos)
        store_probe_bound(l, real, row * out_ld + i, real ? lbv[pos] : 0.0f, real ? lbqv[pos] : 0.0f, bnd);
      else if (bnd.lb)
        write_probe_bound(qs, cent, d, cvec, l, real, row * out_ld + i, bnd);
    }
  }
}

template <int R, typename TS>
cudaError_t launch_shortlist_impl(const TS *s, size_t rows, size_t L, size_t ld, const float *qn, int d,
                                  const float *cent, const float *cmax, double rel, double abs_coef, int k,
                                  uint32_t *ids, float *dst, size_t out_ld, const ProbeBoundArgs &bnd,
                                  cudaStream_t st, const __half *cmx, size_t cstride) {
  const size_t smem = static_cast<size_t>(kSelectWarps) *
                      (kShortBuf * 4 + static_cast<size_t>((d + 3) & ~3) * 4 + kChunkBuf * 4 + 2 * kShortBuf * 4);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(shortlist_kernel<R, TS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  dim3 grid(static_cast<unsigned>((rows + kSelectWarps - 1) / kSelectWarps));
  shortlist_kernel<R, TS><<<grid, kSelectWarps * 32, smem, st>>>(s, rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k,
                                                                  ids, dst, out_ld, bnd, cmx, cstride);
  return cudaGetLastError();
}

template <typename TS>
cudaError_t shortlist_dispatch(const TS *s, size_t rows, size_t L, size_t ld, const float *qn, int d,
                               const float *cent, const float *cmax, double rel, double abs_coef, int k,
                               uint32_t *ids, float *dst, size_t out_ld, const ProbeBoundArgs &bnd, cudaStream_t st,
                               const __half *cmx, size_t cstride) {
  if (k <= 32) return launch_shortlist_impl<1>(s, rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k, ids, dst, out_ld, bnd, st, cmx, cstride);
  if (k <= 64) return launch_shortlist_impl<2>(s, rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k, ids, dst, out_ld, bnd, st, cmx, cstride);
  if (k <= 128) return launch_shortlist_impl<4>(s, rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k, ids, dst, out_ld, bnd, st, cmx, cstride);
  if (k <= 256) return launch_shortlist_impl<8>(s, rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k, ids, dst, out_ld, bnd, st, cmx, cstride);
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_probe_shortlist(const void *s, bool s_half, size_t rows, size_t L, size_t ld, const float *qn,
                                   int d, const float *cent, const float *cmax, double rel, double abs_coef, int k,
                                   uint32_t *out_ids, float *out_dist, size_t out_ld, const ProbeBoundArgs &bnd,
                                   cudaStream_t st, const void *chunk_max, size_t chunk_stride) {
  if (rows == 0 || k <= 0) return cudaSuccess;
  if (s_half)
    return shortlist_dispatch(static_cast<const __half *>(s), rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k,
                              out_ids, out_dist, out_ld, bnd, st, static_cast<const __half *>(chunk_max), chunk_stride);
  return shortlist_dispatch(static_cast<const float *>(s), rows, L, ld, qn, d, cent, cmax, rel, abs_coef, k, out_ids,
                            out_dist, out_ld, bnd, st, nullptr, 0);
}


}  // namespace vg
