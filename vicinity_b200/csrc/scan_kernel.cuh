// Fused IVF-PQ search kernel: one block owns one query at a time and runs
// the reference's per-query loop (search.rs:1175-1391) over its probed lists:
//   1. query residual  q - c_list                      (search.rs:1239-1245)
//   2. ADC table       T[m][c] = sum_j (r_mj - cw_mcj)^2 (pq.rs:573-643)
//   3. code scan       dist = sum_m T[m][code_m]       (pq_simd.rs:314-369),
//      or for 16-entry codebooks on lists of >= 16 vectors the FastScan
//      path: u8-quantised table (pq_simd.rs:576-611), integer sums and
//      dist = sum * scale + min * M                    (pq_simd.rs:721-769)
//   4. top-k by (distance, vector id)                  (search.rs:64-75)
//
// Persistent blocks (one per SM) take queries from an atomic counter and walk
// the query's probes nearest-first, kMaxBatch lists at a time:
//   - every thread builds its fixed share of each list's table; when DSUB > 0
//     the thread's EPT codewords live in registers for the whole kernel, so a
//     table entry costs dsub subtract/multiply/add triples and one store;
//   - the 512 threads score the batch's candidates, one candidate per thread
//     with the reference's sequential sum over subspaces;
//   - each warp keeps its own sorted top-k for the whole query and admits a
//     candidate only if its key is below min(own k-th key, block bound).  The
//     block bound is the smallest k-th key any warp has reached -- a valid
//     upper bound on the query's final k-th key -- so after the nearest lists
//     almost every candidate is rejected by one comparison;
//   - at the end of the query the warp lists are merged and written out.
// Keys are (total_cmp order of the distance, vector id), unique per vector:
// the result is the reference's exactly, with its arbitrary order of equal
// distances fixed by the id.
#pragma once

#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace vg {

constexpr int kScanThreads = 512;
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kMaxBatch = 4;

__host__ __device__ inline size_t scan_pair_bytes(int d, int M, int ks, bool four) {
  size_t b = static_cast<size_t>(M) * ks * 4 + static_cast<size_t>((d + 3) & ~3) * 4;
  if (four) b += (static_cast<size_t>(M) * 16 + 15) & ~static_cast<size_t>(15);
  return b;
}

__host__ __device__ inline size_t scan_smem_bytes(int d, int M, int ks, bool four, int batch, int R) {
  return static_cast<size_t>(kScanWarps) * 32 * R * 8 + static_cast<size_t>(batch) * scan_pair_bytes(d, M, ks, four);
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

// Sequential table sum for one candidate's codes (row layout [m][ks]).
template <int KS>
__device__ __forceinline__ float adc_row_sum(const uint8_t *cp, const float *lg, int M, int ks) {
  const int row_len = KS > 0 ? KS : ks;
  float acc = 0.0f;
  if ((M & 15) == 0) {
    for (int m0 = 0; m0 < M; m0 += 16) {
      uint4 w = *reinterpret_cast<const uint4 *>(cp + m0);
      uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      const float *row = lg + m0 * row_len;
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        uint32_t code = __byte_perm(ws[b >> 2], 0u, 0x4440u + (b & 3));
        acc = __fadd_rn(acc, row[b * row_len + code]);
      }
    }
  } else {
    for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, lg[m * row_len + cp[m]]);
  }
  return acc;
}

template <int DSUB, int EPT, int R, bool FOUR, int KS>
__global__ void __launch_bounds__(kScanThreads, 1) ivfpq_query_kernel(const ScanParams p, const int batch) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, ks = p.ks, d = p.d, P = p.P, k = p.k;
  const int nent = M * ks;
  const int dpad = (d + 3) & ~3;
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(smem);  // [warps][32R]
  float *lut = reinterpret_cast<float *>(wl + kScanWarps * 32 * R);       // [batch][nent]
  float *qres = lut + static_cast<size_t>(batch) * nent;                   // [batch][dpad]
  uint8_t *qlut = reinterpret_cast<uint8_t *>(qres + static_cast<size_t>(batch) * dpad);  // [batch][M*16]
  const int qlut_stride = (M * 16 + 15) & ~15;

  __shared__ uint32_t s_query;
  __shared__ int s_nb, s_next;
  __shared__ uint32_t s_list[kMaxBatch];
  __shared__ uint64_t s_lbeg[kMaxBatch];
  __shared__ uint32_t s_prefix[kMaxBatch + 1];
  __shared__ unsigned long long s_bound;
  __shared__ float s_rmin[kMaxBatch][kScanWarps], s_rmax[kMaxBatch][kScanWarps];
  __shared__ float s_scale[kMaxBatch], s_fbase[kMaxBatch];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

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

  for (;;) {
    if (tid == 0) {
      s_query = atomicAdd(p.counter, 1u);
      s_next = 0;
      s_bound = kEmptyKey;
    }
    __syncthreads();
    const uint32_t q = s_query;
    if (q >= static_cast<uint32_t>(p.nq)) break;
    const uint32_t *probes = p.probes + static_cast<size_t>(q) * P;
    const float *qv = p.qn + static_cast<size_t>(q) * d;
    WarpTopK<R> tk;
    tk.init();

    for (;;) {
      // next batch of probed lists (nearest first), skipping lists this
      // device does not own
      if (tid == 0) {
        int nb = 0, i = s_next;
        uint32_t acc = 0;
        while (i < P && nb < batch) {
          uint32_t l = probes[i++];
          if (l == 0xffffffffu || (p.owner && !p.owner[l])) continue;
          uint64_t b = p.list_off[l];
          s_list[nb] = l;
          s_lbeg[nb] = b;
          s_prefix[nb] = acc;
          acc += static_cast<uint32_t>(p.list_off[l + 1] - b);
          ++nb;
        }
        for (int g = nb; g <= kMaxBatch; ++g) s_prefix[g] = acc;
        s_nb = nb;
        s_next = i;
      }
      __syncthreads();
      const int nb = s_nb;
      if (nb == 0) break;
      for (int i = tid; i < nb * d; i += kScanThreads) {
        int g = i / d, j = i - g * d;
        qres[g * dpad + j] = __fsub_rn(qv[j], p.centroids[static_cast<size_t>(s_list[g]) * d + j]);
      }
      __syncthreads();

      // ---- ADC tables: sequential sum over the subvector, no FMA --------
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
          // global min/max of the table (pq_simd.rs:587-598); fminf/fmaxf
          // skip NaNs as the reference's `<` / `>` comparisons do
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
          s_rmin[g][0] = gmin;                                    // offset
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

      // ---- score and select ---------------------------------------------
      const uint32_t ctotal = s_prefix[kMaxBatch];
      for (uint32_t x0 = warp * 32; x0 < ctotal; x0 += kScanThreads) {
        const uint32_t x = x0 + lane;
        float dist = 0.0f;
        int g = 0;
        uint32_t c = 0;
        if (x < ctotal) {
          g = (x >= s_prefix[1]) + (x >= s_prefix[2]) + (x >= s_prefix[3]);
          c = x - s_prefix[g];
          const uint32_t list = s_list[g];
          const uint32_t len = s_prefix[g + 1] - s_prefix[g];
          if (FOUR && len >= 16) {  // search.rs:1261 (SIMD_BATCH_THRESHOLD)
            const uint8_t *bp = p.packed + p.pack_off[list] + static_cast<uint64_t>(c >> 5) * M * 16;
            const uint8_t *ql = qlut + g * qlut_stride;
            const int col = c & 15;
            const int sh = (c & 31) >= 16 ? 4 : 0;
            uint32_t acc = 0;
            for (int m = 0; m < M; ++m) acc += ql[m * 16 + ((bp[m * 16 + col] >> sh) & 15u)];
            dist = __fadd_rn(__fmul_rn(__uint2float_rn(acc), s_scale[g]), s_fbase[g]);
          } else {
            const uint8_t *cp = p.list_codes + p.code_off[list] + static_cast<uint64_t>(c) * M;
            dist = adc_row_sum<KS>(cp, lut + static_cast<size_t>(g) * nent, M, ks);
          }
        }
        uint64_t thr = tk.worst();
        const uint64_t bound = s_bound;
        thr = bound < thr ? bound : thr;
        const uint32_t dk = order_key(dist);
        const bool pass = x < ctotal && dk <= static_cast<uint32_t>(thr >> 32);
        unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
        if (!mask) continue;
        const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | p.list_ids[s_lbeg[g] + c]) : kEmptyKey;
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
        const uint64_t kth = tk.get(k - 1);
        if (lane == 0 && kth < bound) atomicMin(&s_bound, kth);
      }
      __syncthreads();  // tables and batch metadata are rewritten next
    }

    // ---- merge the warp lists (binary tree) and emit -----------------------
#pragma unroll
    for (int r = 0; r < R; ++r) wl[warp * 32 * R + r * 32 + lane] = tk.v[r];
    __syncthreads();
    for (int stride = 1; stride < kScanWarps; stride <<= 1) {
      if ((warp % (2 * stride)) == 0) {
        const unsigned long long *other = wl + (warp + stride) * 32 * R;
        if (other[0] < tk.worst()) {
#pragma unroll
          for (int r = 0; r < R; ++r) tk.merge_sorted_row(other[r * 32 + lane]);
#pragma unroll
          for (int r = 0; r < R; ++r) wl[warp * 32 * R + r * 32 + lane] = tk.v[r];
        }
      }
      __syncthreads();
    }
    if (warp == 0) {
      uint32_t count = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        const uint64_t key = tk.v[r];
        const bool real = i < k && key != kEmptyKey;
        count += __popc(__ballot_sync(VG_FULL_MASK, real));
        if (i < k) {
          const size_t o = static_cast<size_t>(q) * k + i;
          if (p.out_keys) p.out_keys[o] = key;
          if (p.out_ids) {
            p.out_ids[o] = real ? p.doc_ids[key_id(key)] : 0xffffffffu;
            p.out_dist[o] = real ? key_dist(key) : __int_as_float(0x7f800000);
          }
        }
      }
      if (p.out_count && lane == 0) p.out_count[q] = count;
    }
  }
}

template <int DSUB, int EPT, int R, bool FOUR, int KS>
cudaError_t launch_scan_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_query_kernel<DSUB, EPT, R, FOUR, KS>;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t reserve = 2048;  // static shared memory of the kernel
  int batch = kMaxBatch;
  while (batch > 1 && scan_smem_bytes(p.d, p.M, p.ks, FOUR, batch, R) + reserve > static_cast<size_t>(optin)) --batch;
  const size_t smem = scan_smem_bytes(p.d, p.M, p.ks, FOUR, batch, R);
  if (smem + reserve > static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int grid = num_sms * per_sm;
  if (grid > p.nq) grid = p.nq;
  kern<<<grid, kScanThreads, smem, s>>>(p, batch);
  return cudaGetLastError();
}

}  // namespace vg
