// Fused IVF-PQ probe kernel.  For each (query, inverted list) pair:
//   1. query residual  q - c_list                      (search.rs:1239-1245)
//   2. ADC table       T[m][c] = sum_j (r_mj - cw_mcj)^2 (pq.rs:573-643)
//   3. code scan       dist = sum_m T[m][code_m]       (pq_simd.rs:314-369),
//      or for 16-entry codebooks on lists of >= 16 vectors the FastScan
//      path: u8-quantised table (pq_simd.rs:576-611), integer sums and
//      dist = sum * scale + min * M                    (pq_simd.rs:721-769)
//   4. the pair's k best (distance, vector id) keys    (search.rs:64-75)
//
// Persistent blocks (one per SM) pull batches of up to kMaxBatch pairs from
// a list-major work array with an atomic counter.  Per batch:
//   - every thread builds its fixed share of each pair's table; when DSUB > 0
//     the thread's EPT codewords live in registers for the whole kernel and
//     their subspace offsets are precomputed, so a table entry costs dsub
//     subtract/multiply/add triples plus one shared store;
//   - all 512 threads score the batch's candidates (one candidate per
//     thread, sequential sum over subspaces) into a shared distance array;
//   - warp g selects pair g's top-k from that array.  A per-query bound
//     tau[q] (the k-th best key of any finished pair of q; a valid upper
//     bound on q's final k-th key) rejects almost every candidate with one
//     comparison; survivors are inserted into a sorted warp list.
// Keys are (total_cmp order of the distance, vector id), unique per vector,
// so the selected set is exactly the reference's up to its arbitrary order
// of equal distances, which the id breaks.
#pragma once

#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace vg {

constexpr int kScanThreads = 512;
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kMaxBatch = 4;
constexpr int kDistCap = 4096;  // candidates scored per shared-memory chunk

__host__ __device__ inline size_t scan_pair_bytes(int d, int M, int ks, bool four) {
  size_t b = static_cast<size_t>(M) * ks * 4 + static_cast<size_t>((d + 3) & ~3) * 4;
  if (four) b += (static_cast<size_t>(M) * 16 + 15) & ~static_cast<size_t>(15);
  return b;
}

__host__ __device__ inline size_t scan_smem_bytes(int d, int M, int ks, bool four, int batch) {
  return static_cast<size_t>(kDistCap) * 4 + static_cast<size_t>(batch) * scan_pair_bytes(d, M, ks, four);
}

template <int R>
__device__ __forceinline__ void topk_insert_one(WarpTopK<R> &tk, uint64_t key) {
  if (R == 1) {
    const int lane = lane_id();
    if (key >= shfl64(tk.v[0], 31)) return;
    unsigned below = __ballot_sync(VG_FULL_MASK, tk.v[0] < key);
    int rank = __popc(below);
    uint64_t up = __shfl_up_sync(VG_FULL_MASK, static_cast<unsigned long long>(tk.v[0]), 1);
    tk.v[0] = lane < rank ? tk.v[0] : (lane == rank ? key : up);
  } else {
    tk.add(lane_id() == 0 ? key : kEmptyKey);
  }
}

template <int DSUB, int EPT, int R, bool FOUR>
__global__ void __launch_bounds__(kScanThreads, 1) ivfpq_scan_kernel(const ScanParams p, const int batch) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, ks = p.ks, d = p.d;
  const int nent = M * ks;
  const int dpad = (d + 3) & ~3;
  float *sdist = reinterpret_cast<float *>(smem);
  float *lut = sdist + kDistCap;                   // [batch][nent]
  float *qres = lut + static_cast<size_t>(batch) * nent;  // [batch][dpad]
  uint8_t *qlut = reinterpret_cast<uint8_t *>(qres + static_cast<size_t>(batch) * dpad);  // [batch][M*16]
  const int qlut_stride = (M * 16 + 15) & ~15;

  __shared__ uint32_t s_base;
  __shared__ uint32_t s_pair[kMaxBatch], s_q[kMaxBatch], s_list[kMaxBatch];
  __shared__ uint64_t s_lbeg[kMaxBatch];
  __shared__ uint32_t s_prefix[kMaxBatch + 1];
  __shared__ float s_rmin[kMaxBatch][kScanWarps], s_rmax[kMaxBatch][kScanWarps];
  __shared__ float s_scale[kMaxBatch], s_fbase[kMaxBatch];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // register-resident codewords and their subspace offsets (fixed per thread)
  constexpr int kD = DSUB > 0 ? DSUB : 1;
  constexpr int kE = EPT > 0 ? EPT : 1;
  float cb[kE][kD];
  if (DSUB > 0) {
#pragma unroll
    for (int i = 0; i < kE; ++i) {
      int e = tid + i * kScanThreads;
#pragma unroll
      for (int j = 0; j < kD; ++j) cb[i][j] = e < nent ? p.codebooks[static_cast<size_t>(e) * kD + j] : 0.0f;
    }
  }
  // subspace offset of entry tid + i*512: an arithmetic progression in i
  // when ks divides 512, otherwise one division per entry
  const bool ks_divides = (kScanThreads % ks) == 0;
  const int qoff0 = (tid / ks) * kD;
  const int qstep = ks_divides ? (kScanThreads / ks) * kD : 0;

  const uint32_t total = *p.total;
  for (;;) {
    if (tid == 0) s_base = atomicAdd(p.counter, static_cast<uint32_t>(batch));
    __syncthreads();
    const uint32_t base = s_base;
    if (base >= total) break;
    const int nb = static_cast<int>(min(static_cast<uint32_t>(batch), total - base));
    if (tid < kMaxBatch) {
      if (tid < nb) {
        uint32_t pair = p.work[base + tid];
        uint32_t list = p.probes[pair];
        s_pair[tid] = pair;
        s_q[tid] = pair / static_cast<uint32_t>(p.P);
        s_list[tid] = list;
        s_lbeg[tid] = p.list_off[list];
      }
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t acc = 0;
      for (int g = 0; g < kMaxBatch; ++g) {
        s_prefix[g] = acc;
        if (g < nb) acc += static_cast<uint32_t>(p.list_off[s_list[g] + 1] - s_lbeg[g]);
      }
      s_prefix[kMaxBatch] = acc;
    }
    for (int i = tid; i < nb * d; i += kScanThreads) {
      int g = i / d, j = i - g * d;
      qres[g * dpad + j] = __fsub_rn(p.qn[static_cast<size_t>(s_q[g]) * d + j],
                                     p.centroids[static_cast<size_t>(s_list[g]) * d + j]);
    }
    __syncthreads();

    // ---- ADC tables: sequential sum over the subvector, no FMA ----------
#pragma unroll 1
    for (int g = 0; g < nb; ++g) {
      const float *qg = qres + g * dpad;
      float *lg = lut + static_cast<size_t>(g) * nent;
      float lmin = __int_as_float(0x7f800000), lmax = -__int_as_float(0x7f800000);
      if (DSUB > 0) {
#pragma unroll
        for (int i = 0; i < kE; ++i) {
          int e = tid + i * kScanThreads;
          if (e < nent) {
            const float *qs = qg + (ks_divides ? qoff0 + i * qstep : (e / ks) * kD);
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < kD; ++j) {
              float diff = __fsub_rn(qs[j], cb[i][j]);
              acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
            lg[e] = acc;
            if (FOUR) {
              lmin = fminf(lmin, acc);
              lmax = fmaxf(lmax, acc);
            }
          }
        }
      } else {
        for (int e = tid; e < nent; e += kScanThreads) {
          const float *qs = qg + (e / ks) * p.dsub;
          const float *cw = p.codebooks + static_cast<size_t>(e) * p.dsub;
          float acc = 0.0f;
          for (int j = 0; j < p.dsub; ++j) {
            float diff = __fsub_rn(qs[j], __ldg(cw + j));
            acc = __fadd_rn(acc, __fmul_rn(diff, diff));
          }
          lg[e] = acc;
          if (FOUR) {
            lmin = fminf(lmin, acc);
            lmax = fmaxf(lmax, acc);
          }
        }
      }
      if (FOUR) {
        // Global min/max per table (pq_simd.rs:587-598); fminf/fmaxf skip
        // NaNs as the reference's `<` / `>` comparisons do.
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          lmin = fminf(lmin, __shfl_xor_sync(VG_FULL_MASK, lmin, off));
          lmax = fmaxf(lmax, __shfl_xor_sync(VG_FULL_MASK, lmax, off));
        }
        if (lane == 0) {
          s_rmin[g][warp] = lmin;
          s_rmax[g][warp] = lmax;
        }
      }
    }
    if (FOUR) {
      __syncthreads();
      if (tid < nb) {
        const int g = tid;
        float gmin = s_rmin[g][0], gmax = s_rmax[g][0];
        for (int w = 1; w < kScanWarps; ++w) {
          gmin = fminf(gmin, s_rmin[g][w]);
          gmax = fmaxf(gmax, s_rmax[g][w]);
        }
        float range = __fsub_rn(gmax, gmin);
        bool flat = range < FLT_EPSILON;
        s_rmin[g][0] = gmin;  // offset
        s_rmax[g][0] = flat ? 0.0f : __fdiv_rn(255.0f, range);  // inverse scale
        s_scale[g] = flat ? 1.0f : __fdiv_rn(range, 255.0f);
        s_fbase[g] = __fmul_rn(gmin, static_cast<float>(M));
      }
      __syncthreads();
      for (int i = tid; i < nb * nent; i += kScanThreads) {
        int g = i / nent, e = i - g * nent;
        // round half away from zero, clamp; NaN -> 0 (pq_simd.rs:607-609)
        float t = roundf(__fmul_rn(__fsub_rn(lut[i], s_rmin[g][0]), s_rmax[g][0]));
        t = fminf(fmaxf(t, 0.0f), 255.0f);
        qlut[g * qlut_stride + e] = static_cast<uint8_t>(t);
      }
    }
    __syncthreads();

    // ---- score candidates in chunks, select per pair -------------------
    const uint32_t ctotal = s_prefix[kMaxBatch];
    const bool selector = warp < nb;
    WarpTopK<R> tk;
    tk.init();
    uint64_t thr = kEmptyKey;
    uint32_t sel_beg = 0, sel_end = 0;
    const uint32_t *sel_ids = nullptr;
    if (selector) {
      sel_beg = s_prefix[warp];
      sel_end = s_prefix[warp + 1];
      sel_ids = p.list_ids + s_lbeg[warp];
      thr = p.tau[s_q[warp]];
    }
    for (uint32_t c0 = 0; c0 < ctotal; c0 += kDistCap) {
      const uint32_t c1 = min(ctotal, c0 + static_cast<uint32_t>(kDistCap));
      for (uint32_t x = c0 + tid; x < c1; x += kScanThreads) {
        const int g = (x >= s_prefix[1]) + (x >= s_prefix[2]) + (x >= s_prefix[3]);
        const uint32_t c = x - s_prefix[g];
        const uint32_t list = s_list[g];
        const uint32_t len = s_prefix[g + 1] - s_prefix[g];
        float dist;
        if (FOUR && len >= 16) {  // search.rs:1261 (SIMD_BATCH_THRESHOLD)
          const uint8_t *bp = p.packed + p.pack_off[list] + static_cast<uint64_t>(c >> 5) * M * 16;
          const uint8_t *ql = qlut + g * qlut_stride;
          const int col = c & 15;
          const bool hi = (c & 31) >= 16;
          uint32_t acc = 0;
          for (int m = 0; m < M; ++m) {
            uint32_t byte = bp[m * 16 + col];
            acc += ql[m * 16 + (hi ? (byte >> 4) : (byte & 15u))];
          }
          dist = __fadd_rn(__fmul_rn(__uint2float_rn(acc), s_scale[g]), s_fbase[g]);
        } else {
          const uint8_t *cp = p.list_codes + p.code_off[list] + static_cast<uint64_t>(c) * M;
          const float *lg = lut + static_cast<size_t>(g) * nent;
          float acc = 0.0f;
          if ((M & 15) == 0) {
            for (int m0 = 0; m0 < M; m0 += 16) {
              uint4 w = *reinterpret_cast<const uint4 *>(cp + m0);
              uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int b = 0; b < 16; ++b) {
                uint32_t code = (ws[b >> 2] >> ((b & 3) * 8)) & 0xffu;
                acc = __fadd_rn(acc, lg[(m0 + b) * ks + code]);
              }
            }
          } else {
            for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, lg[m * ks + cp[m]]);
          }
          dist = acc;
        }
        sdist[x - c0] = dist;
      }
      __syncthreads();
      if (selector) {
        const uint32_t b = max(sel_beg, c0), e = min(sel_end, c1);
        for (uint32_t x0 = b; x0 < e; x0 += 32) {
          const uint32_t x = x0 + lane;
          uint32_t dk = 0xffffffffu;
          if (x < e) dk = order_key(sdist[x - c0]);
          const bool pass = x < e && dk <= static_cast<uint32_t>(thr >> 32);
          unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
          if (!mask) continue;
          const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | sel_ids[x - sel_beg]) : kEmptyKey;
          if (__popc(mask) > 4) {
            tk.add(key < thr ? key : kEmptyKey);
          } else {
            while (mask) {
              int src = __ffs(mask) - 1;
              mask &= mask - 1;
              uint64_t kx = shfl64(key, src);
              if (kx < thr) topk_insert_one(tk, kx);
            }
          }
          uint64_t w = tk.worst();
          thr = w < thr ? w : thr;
        }
      }
      __syncthreads();
    }
    if (selector) {
      unsigned long long *out = p.pair_out + static_cast<size_t>(s_pair[warp]) * p.k;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        int i = r * 32 + lane;
        if (i < p.k) out[i] = tk.v[r];
      }
      // the pair's k-th key bounds the query's final k-th key
      uint64_t kth = tk.get(p.k - 1);
      if (lane == 0 && kth != kEmptyKey) atomicMin(p.tau + s_q[warp], kth);
    }
  }
}

template <int DSUB, int EPT, int R, bool FOUR>
cudaError_t launch_scan_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_scan_kernel<DSUB, EPT, R, FOUR>;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t reserve = 4096;  // static shared memory of the kernel
  int batch = kMaxBatch;
  while (batch > 1 && scan_smem_bytes(p.d, p.M, p.ks, FOUR, batch) + reserve > static_cast<size_t>(optin)) --batch;
  size_t smem = scan_smem_bytes(p.d, p.M, p.ks, FOUR, batch);
  if (smem + reserve > static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  kern<<<num_sms * per_sm, kScanThreads, smem, s>>>(p, batch);
  return cudaGetLastError();
}

}  // namespace vg
