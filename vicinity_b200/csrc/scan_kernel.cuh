// Fused IVF-PQ probe kernel: for one (query, inverted list) pair at a time,
//   1. query residual  q - c_list                      (search.rs:1239-1245)
//   2. ADC table       T[m][c] = sum_j (r_mj - cw_mcj)^2 (pq.rs:573-643)
//   3. code scan       dist = sum_m T[m][code_m]       (pq_simd.rs:314-369),
//      or for 16-entry codebooks on lists of >= 16 vectors the FastScan
//      path: u8-quantised table (pq_simd.rs:576-611), integer sums and
//      dist = sum * scale + min * M                    (pq_simd.rs:721-769)
//   4. the pair's k best (distance, internal id) keys  (search.rs:64-75)
//
// Persistent blocks (one per SM) pull pairs from a list-major work array
// with an atomic counter, so concurrently running blocks tend to share a
// list and its codes stay in L2.  When DSUB > 0 each thread keeps EPT
// codewords of the product-quantizer codebook in registers for the whole
// kernel, so building a table costs no codebook memory traffic; DSUB == 0 is
// the general-shape variant that reads codewords through the L1 cache.
#pragma once

#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace vg {

constexpr int kScanThreads = 512;
constexpr int kScanWarps = kScanThreads / 32;

__host__ __device__ inline size_t scan_smem_bytes(int d, int M, int ks, int R, bool four) {
  size_t b = static_cast<size_t>(kScanWarps) * 32 * R * 8;
  b += static_cast<size_t>((d + 3) & ~3) * 4;
  b += static_cast<size_t>(M) * ks * 4;
  if (four) b += (static_cast<size_t>(M) * 16 + 15) & ~static_cast<size_t>(15);
  return b;
}

template <int DSUB, int EPT, int R, bool FOUR>
__global__ void __launch_bounds__(kScanThreads, 1) ivfpq_scan_kernel(const ScanParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(smem);  // [warps][32R]
  float *qres = reinterpret_cast<float *>(smem + static_cast<size_t>(kScanWarps) * 32 * R * 8);
  float *lut = qres + ((p.d + 3) & ~3);
  uint8_t *qlut = reinterpret_cast<uint8_t *>(lut + p.M * p.ks);

  __shared__ uint32_t s_item;
  __shared__ float s_rmin[kScanWarps], s_rmax[kScanWarps];
  __shared__ float s_off, s_inv, s_scale, s_base;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nent = p.M * p.ks;

  constexpr int kD = DSUB > 0 ? DSUB : 1;
  constexpr int kE = EPT > 0 ? EPT : 1;
  float cb[kE][kD];
  if (DSUB > 0) {
#pragma unroll
    for (int i = 0; i < kE; ++i) {
      int e = tid + i * kScanThreads;
#pragma unroll
      for (int j = 0; j < kD; ++j)
        cb[i][j] = e < nent ? p.codebooks[static_cast<size_t>(e) * kD + j] : 0.0f;
    }
  }

  const uint32_t total = *p.total;
  for (;;) {
    if (tid == 0) s_item = atomicAdd(p.counter, 1u);
    __syncthreads();
    const uint32_t item = s_item;
    if (item >= total) break;
    const uint32_t pair = p.work[item];
    const uint32_t qi = pair / static_cast<uint32_t>(p.P);
    const uint32_t list = p.probes[pair];
    const float *qv = p.qn + static_cast<size_t>(qi) * p.d;
    const float *cv = p.centroids + static_cast<size_t>(list) * p.d;
    for (int i = tid; i < p.d; i += kScanThreads) qres[i] = __fsub_rn(qv[i], cv[i]);
    __syncthreads();

    // ---- ADC table: sequential sum over the subvector, no FMA ----------
    float lmin = __int_as_float(0x7f800000), lmax = -__int_as_float(0x7f800000);
    if (DSUB > 0) {
#pragma unroll
      for (int i = 0; i < kE; ++i) {
        int e = tid + i * kScanThreads;
        if (e < nent) {
          const float *qs = qres + (e / p.ks) * kD;
          float acc = 0.0f;
#pragma unroll
          for (int j = 0; j < kD; ++j) {
            float diff = __fsub_rn(qs[j], cb[i][j]);
            acc = __fadd_rn(acc, __fmul_rn(diff, diff));
          }
          lut[e] = acc;
          lmin = fminf(lmin, acc);
          lmax = fmaxf(lmax, acc);
        }
      }
    } else {
      for (int e = tid; e < nent; e += kScanThreads) {
        const float *qs = qres + (e / p.ks) * p.dsub;
        const float *cw = p.codebooks + static_cast<size_t>(e) * p.dsub;
        float acc = 0.0f;
        for (int j = 0; j < p.dsub; ++j) {
          float diff = __fsub_rn(qs[j], __ldg(cw + j));
          acc = __fadd_rn(acc, __fmul_rn(diff, diff));
        }
        lut[e] = acc;
        lmin = fminf(lmin, acc);
        lmax = fmaxf(lmax, acc);
      }
    }

    const uint64_t lbeg = p.list_off[list];
    const uint64_t len = p.list_off[list + 1] - lbeg;
    const bool fast = FOUR && len >= 16;  // search.rs:1261 (SIMD_BATCH_THRESHOLD)
    if (FOUR && fast) {
      // Global min/max of the table (pq_simd.rs:587-598); fminf/fmaxf skip
      // NaNs as the reference's `<` / `>` comparisons do.
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        lmin = fminf(lmin, __shfl_xor_sync(VG_FULL_MASK, lmin, off));
        lmax = fmaxf(lmax, __shfl_xor_sync(VG_FULL_MASK, lmax, off));
      }
      if (lane == 0) {
        s_rmin[warp] = lmin;
        s_rmax[warp] = lmax;
      }
      __syncthreads();
      if (tid == 0) {
        float gmin = s_rmin[0], gmax = s_rmax[0];
        for (int w = 1; w < kScanWarps; ++w) {
          gmin = fminf(gmin, s_rmin[w]);
          gmax = fmaxf(gmax, s_rmax[w]);
        }
        float range = __fsub_rn(gmax, gmin);
        bool flat = range < FLT_EPSILON;
        s_off = gmin;
        s_scale = flat ? 1.0f : __fdiv_rn(range, 255.0f);
        s_inv = flat ? 0.0f : __fdiv_rn(255.0f, range);
        s_base = __fmul_rn(gmin, static_cast<float>(p.M));
      }
      __syncthreads();
      const float off = s_off, inv = s_inv;
      for (int e = tid; e < nent; e += kScanThreads) {
        // round half away from zero, clamp; NaN -> 0 (pq_simd.rs:607-609)
        float t = roundf(__fmul_rn(__fsub_rn(lut[e], off), inv));
        t = fminf(fmaxf(t, 0.0f), 255.0f);
        qlut[e] = static_cast<uint8_t>(t);
      }
    }
    __syncthreads();

    // ---- scan ---------------------------------------------------------
    WarpTopK<R> tk;
    tk.init();
    const uint32_t *ids = p.list_ids + lbeg;
    const int M = p.M, ks = p.ks;
    for (uint64_t b0 = static_cast<uint64_t>(warp) * 32; b0 < len; b0 += kScanThreads) {
      const uint64_t c = b0 + lane;
      uint64_t key = kEmptyKey;
      if (c < len) {
        float dist;
        if (FOUR && fast) {
          const uint8_t *bp = p.packed + p.pack_off[list] + (c >> 5) * static_cast<uint64_t>(M) * 16;
          const int col = static_cast<int>(c & 15);
          const bool hi = (c & 31) >= 16;
          uint32_t acc = 0;
          for (int m = 0; m < M; ++m) {
            uint32_t byte = bp[m * 16 + col];
            uint32_t nib = hi ? (byte >> 4) : (byte & 15u);
            acc += qlut[m * 16 + nib];
          }
          dist = __fadd_rn(__fmul_rn(__uint2float_rn(acc), s_scale), s_base);
        } else {
          const uint8_t *cp = p.list_codes + p.code_off[list] + c * static_cast<uint64_t>(M);
          float acc = 0.0f;
          if ((M & 15) == 0) {
            for (int m0 = 0; m0 < M; m0 += 16) {
              uint4 w = *reinterpret_cast<const uint4 *>(cp + m0);
              uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int b = 0; b < 16; ++b) {
                uint32_t code = (ws[b >> 2] >> ((b & 3) * 8)) & 0xffu;
                acc = __fadd_rn(acc, lut[(m0 + b) * ks + code]);
              }
            }
          } else {
            for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, lut[m * ks + cp[m]]);
          }
          dist = acc;
        }
        key = pack_key(dist, ids[c]);
      }
      tk.add(key);
    }

    // ---- block merge of the per-warp lists (binary tree) --------------
    const uint64_t busy_warps = (len + 31) / 32;
    const int active = busy_warps < kScanWarps ? static_cast<int>(busy_warps) : kScanWarps;
    if (warp < active) {
#pragma unroll
      for (int r = 0; r < R; ++r) wl[warp * 32 * R + r * 32 + lane] = tk.v[r];
    }
    __syncthreads();
    for (int stride = 1; stride < active; stride <<= 1) {
      if ((warp % (2 * stride)) == 0 && warp + stride < active) {
        const unsigned long long *other = wl + (warp + stride) * 32 * R;
#pragma unroll
        for (int r = 0; r < R; ++r) tk.merge_sorted_row(other[r * 32 + lane]);
#pragma unroll
        for (int r = 0; r < R; ++r) wl[warp * 32 * R + r * 32 + lane] = tk.v[r];
      }
      __syncthreads();
    }
    if (warp == 0) {
      unsigned long long *out = p.pair_out + static_cast<size_t>(pair) * p.k;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        int i = r * 32 + lane;
        if (i < p.k) out[i] = active > 0 ? tk.v[r] : kEmptyKey;
      }
    }
  }
}

template <int DSUB, int EPT, int R, bool FOUR>
cudaError_t launch_scan_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_scan_kernel<DSUB, EPT, R, FOUR>;
  size_t smem = scan_smem_bytes(p.d, p.M, p.ks, R, FOUR);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  kern<<<num_sms * per_sm, kScanThreads, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace vg
