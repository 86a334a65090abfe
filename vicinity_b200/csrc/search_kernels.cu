// Search-side kernels: query normalisation, exact coarse distances, row
// top-k selection, list-major pair grouping and the final merges.
//
// Reference behaviour restated here (vicinity 0.12.0):
//   normalize_query            src/ivf_pq/search.rs:55-62
//   find_nearest_centroids     src/ivf_pq/search.rs:1602-1617 (1 - dot,
//                              select nprobe smallest, sort ascending)
//   finish_top_k_by_distance   src/ivf_pq/search.rs:64-75
//   doc-id mapping             src/ivf_pq/search.rs:1087-1093
//   batch padding              src/python.rs:745-795 (-1 / +inf)
#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "f32x2.cuh"
#include "kernels.h"
#include "probe_bounds.cuh"
#include "topk.cuh"

namespace vg {

// ---------------------------------------------------------------------------
// Normalisation: 32 rows per block staged through shared memory (row stride
// d+1 floats so the per-row sequential sums are bank-conflict free).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) normalize_rows_kernel(const float *__restrict__ x, size_t n,
                                                             int d, float *__restrict__ out) {
  extern __shared__ float tile[];  // [32][d+1]
  __shared__ float norms[32];
  __shared__ int do_div[32];
  const size_t row0 = static_cast<size_t>(blockIdx.x) * 32;
  const int rows = (n - row0) < 32 ? static_cast<int>(n - row0) : 32;
  const int stride = d + 1;
  for (int i = threadIdx.x; i < rows * d; i += blockDim.x) {
    int r = i / d, j = i - r * d;
    tile[r * stride + j] = x[(row0 + r) * d + j];
  }
  __syncthreads();
  if (threadIdx.x < rows) {
    const float *row = tile + threadIdx.x * stride;
    float s = 0.0f;
    for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(row[j], row[j]));
    float norm = __fsqrt_rn(s);
    do_div[threadIdx.x] = norm > 1e-10f;
    norms[threadIdx.x] = norm;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * d; i += blockDim.x) {
    int r = i / d, j = i - r * d;
    float v = tile[r * stride + j];
    out[(row0 + r) * d + j] = do_div[r] ? __fdiv_rn(v, norms[r]) : v;
  }
}

cudaError_t launch_normalize_rows(const float *x, size_t n, int d, float *out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  size_t smem = static_cast<size_t>(32) * (d + 1) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(normalize_rows_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  dim3 grid(static_cast<unsigned>((n + 31) / 32));
  normalize_rows_kernel<<<grid, 256, smem, s>>>(x, n, d, out);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Exact dot-product tiles.  Each thread owns an 8x8 block of (row, column)
// accumulators and walks the shared dimension in order, so every accumulator
// is the reference's sequential sum sum_j a_j*b_j with separately rounded
// multiply and add.  Zero padding beyond d adds +0 products, which leaves the
// sum unchanged.
// ---------------------------------------------------------------------------
namespace {
constexpr int kTileM = 128, kTileN = 128, kTileK = 16, kTileThreads = 256;
enum DotMode { kWriteOneMinus = 0, kArgminOneMinus = 1, kWriteNeg = 2, kWriteDot = 3 };

template <int MODE>
__global__ void __launch_bounds__(kTileThreads)
    dot_tile_kernel(const float *__restrict__ a, size_t rows, const float *__restrict__ b, size_t cols,
                    int d, float *__restrict__ out, size_t ld, unsigned long long *__restrict__ best,
                    float neg_zero) {
  // A is staged with every value in both halves of a pair ({a, a}), so one
  // 16-byte load yields two ready operands for the packed products below.
  __shared__ __align__(16) f32x2 as[kTileK][kTileM + 2];
  __shared__ __align__(16) float bs[kTileK][kTileN + 4];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const size_t row0 = static_cast<size_t>(blockIdx.y) * kTileM;
  const size_t col0 = static_cast<size_t>(blockIdx.x) * kTileN;
  const f32x2 nz = f2_pack(neg_zero, neg_zero);

  // acc2[i][h] holds columns (2h, 2h + 1) of row i of this thread's 8 x 8
  // block; each lane sums its products in k order from 0, as the scalar
  // __fadd_rn(acc, __fmul_rn(a, b)) does (the product is an FMA with a
  // run-time -0 addend so it cannot be fused into the add).
  f32x2 acc2[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int h = 0; h < 4; ++h) acc2[i][h] = 0ull;

  for (int k0 = 0; k0 < d; k0 += kTileK) {
#pragma unroll
    for (int t = 0; t < (kTileM * kTileK) / kTileThreads; ++t) {
      int i = tid + t * kTileThreads;
      int r = i >> 4, kk = i & 15;
      size_t gr = row0 + r;
      int gk = k0 + kk;
      const float av = (gr < rows && gk < d) ? a[gr * d + gk] : 0.0f;
      as[kk][r] = f2_pack(av, av);
      size_t gc = col0 + r;
      bs[kk][r] = (gc < cols && gk < d) ? b[gc * d + gk] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kTileK; ++kk) {
      f32x2 av[8];
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const ulonglong2 t2 = *reinterpret_cast<const ulonglong2 *>(&as[kk][ty * 8 + i]);
        av[i] = t2.x;
        av[i + 1] = t2.y;
      }
      const ulonglong2 b01 = *reinterpret_cast<const ulonglong2 *>(&bs[kk][tx * 8]);
      const ulonglong2 b23 = *reinterpret_cast<const ulonglong2 *>(&bs[kk][tx * 8 + 4]);
      const f32x2 bv[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int h = 0; h < 4; ++h) acc2[i][h] = f2_add(acc2[i][h], f2_fma(av[i], bv[h], nz));
    }
    __syncthreads();
  }
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 v = f2_unpack(acc2[i][h]);
      acc[i][2 * h] = v.x;
      acc[i][2 * h + 1] = v.y;
    }

  if (MODE == kArgminOneMinus) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      size_t r = row0 + ty * 8 + i;
      unsigned long long kbest = kEmptyKey;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        size_t c = col0 + tx * 8 + j;
        if (c < cols) {
          unsigned long long key = pack_key(__fsub_rn(1.0f, acc[i][j]), static_cast<uint32_t>(c));
          kbest = key < kbest ? key : kbest;
        }
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) {
        unsigned long long o = __shfl_xor_sync(VG_FULL_MASK, kbest, off);
        kbest = o < kbest ? o : kbest;
      }
      if (tx == 0 && r < rows && kbest != kEmptyKey) atomicMin(best + r, kbest);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      size_t r = row0 + ty * 8 + i;
      if (r >= rows) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        size_t c = col0 + tx * 8 + j;
        if (c < cols)
          out[r * ld + c] = MODE == kWriteOneMinus ? __fsub_rn(1.0f, acc[i][j])
                            : MODE == kWriteNeg    ? -acc[i][j]
                                                   : acc[i][j];
      }
    }
  }
}

template <int MODE>
cudaError_t launch_dot(const float *a, size_t rows, const float *b, size_t cols, int d, float *out,
                       size_t ld, unsigned long long *best, cudaStream_t s) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((cols + kTileN - 1) / kTileN),
            static_cast<unsigned>((rows + kTileM - 1) / kTileM));
  if (grid.y > 65535) return cudaErrorInvalidValue;
  dot_tile_kernel<MODE><<<grid, kTileThreads, 0, s>>>(a, rows, b, cols, d, out, ld, best, -0.0f);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_coarse_dist(const float *q, size_t B, const float *cent, size_t L, int d,
                               float *dist, size_t ld, cudaStream_t s) {
  return launch_dot<kWriteOneMinus>(q, B, cent, L, d, dist, ld, nullptr, s);
}

cudaError_t launch_coarse_argmin(const float *q, size_t B, const float *cent, size_t L, int d,
                                 unsigned long long *best, cudaStream_t s) {
  return launch_dot<kArgminOneMinus>(q, B, cent, L, d, nullptr, 0, best, s);
}

cudaError_t launch_neg_dot(const float *q, size_t B, const float *db, size_t n, int d, float *dist,
                           size_t ld, cudaStream_t s) {
  return launch_dot<kWriteNeg>(q, B, db, n, d, dist, ld, nullptr, s);
}

cudaError_t launch_rotate_rows(const float *x, size_t n, int d, const float *rotation, float *out,
                               cudaStream_t s) {
  // out[i][r] = sum_j x[i][j] * R[r][j]: the rows of R are the columns of the tile
  return launch_dot<kWriteDot>(x, n, rotation, static_cast<size_t>(d), d, out, static_cast<size_t>(d), nullptr, s);
}

// ---------------------------------------------------------------------------
// Row selection: one warp per row, WarpTopK over the row's columns.
// ---------------------------------------------------------------------------
namespace {
constexpr int kSelectWarps = 8;
constexpr int kSelectBuf = 256;  // keys per warp gathered under the bound

// Exact per-row top-k of [rows][cols] values as (order key, column) keys,
// one warp per row, in two passes over the row:
//  1. every lane keeps its 2R smallest keys (sorted insertion); the k-th
//     smallest of these 64R keys bounds the row's k-th key from above (they
//     are keys of the row);
//  2. the keys <= that bound -- the row's k smallest among them -- are
//     gathered in shared memory (ballot / popc append, no sorting in the
//     loop) and selected with one warp top-k.  If more than kSelectBuf keys
//     fall under the bound the warp selects from the row directly.
template <int R>
__global__ void __launch_bounds__(kSelectWarps * 32)
    select_rows_kernel(const float *__restrict__ dist, size_t rows, size_t cols, size_t ld, int k,
                       uint32_t *__restrict__ out_ids, float *__restrict__ out_dist,
                       unsigned long long *__restrict__ out_keys, size_t out_ld, uint32_t col_base) {
  __shared__ unsigned long long s_buf[kSelectWarps][kSelectBuf];
  constexpr int R2 = 2 * R;
  const size_t row = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const float *drow = dist + row * ld;
  auto key_at = [&](size_t c) { return pack_key(drow[c], col_base + static_cast<uint32_t>(c)); };

  // pass 1: per-lane 2R smallest, four independent loads in flight
  uint64_t a[R2];
#pragma unroll
  for (int r = 0; r < R2; ++r) a[r] = kEmptyKey;
  auto insert = [&](uint64_t key) {
#pragma unroll
    for (int r = 0; r < R2; ++r) {
      const uint64_t lo = key < a[r] ? key : a[r];
      key = key < a[r] ? a[r] : key;
      a[r] = lo;
    }
  };
  size_t c = lane;
  for (; c + 96 < cols; c += 128) {
    const uint64_t k0 = key_at(c), k1 = key_at(c + 32), k2 = key_at(c + 64), k3 = key_at(c + 96);
    insert(k0);
    insert(k1);
    insert(k2);
    insert(k3);
  }
  for (; c < cols; c += 32) insert(key_at(c));
  WarpTopK<R2> cand;
  cand.init();
#pragma unroll
  for (int r = 0; r < R2; ++r) cand.add(a[r]);
  const uint64_t bound = cand.get(k - 1);  // kEmptyKey when the row has fewer than k columns

  // pass 2: gather the keys under the bound
  unsigned long long *buf = s_buf[warp];
  int n = 0;
  bool overflow = false;
  for (size_t c0 = 0; c0 < cols && !overflow; c0 += 32) {
    const size_t cc = c0 + lane;
    const uint64_t key = cc < cols ? key_at(cc) : kEmptyKey;
    const bool take = cc < cols && key <= bound;
    const unsigned m = __ballot_sync(VG_FULL_MASK, take);
    if (n + __popc(m) > kSelectBuf) {
      overflow = true;
      break;
    }
    if (take) buf[n + __popc(m & ((1u << lane) - 1u))] = key;
    n += __popc(m);
  }
  __syncwarp();
  WarpTopK<R> tk;
  tk.init();
  if (!overflow) {
    for (int i0 = 0; i0 < n; i0 += 32) tk.add(i0 + lane < n ? buf[i0 + lane] : kEmptyKey);
  } else {
    for (size_t c0 = 0; c0 < cols; c0 += 32) tk.add(c0 + lane < cols ? key_at(c0 + lane) : kEmptyKey);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    if (i < k) {
      const uint64_t key = tk.v[r];
      if (out_keys) out_keys[row * out_ld + i] = key;
      if (out_ids) {
        const bool real = key != kEmptyKey;
        out_ids[row * out_ld + i] = real ? key_id(key) : 0xffffffffu;
        out_dist[row * out_ld + i] = real ? key_dist(key) : __int_as_float(0x7f800000);
      }
    }
  }
}

template <int R>
cudaError_t launch_select_impl(const float *dist, size_t rows, size_t cols, size_t ld, int k,
                               uint32_t *ids, float *dst, unsigned long long *keys, size_t out_ld,
                               uint32_t col_base, cudaStream_t s) {
  dim3 grid(static_cast<unsigned>((rows + kSelectWarps - 1) / kSelectWarps));
  select_rows_kernel<R><<<grid, kSelectWarps * 32, 0, s>>>(dist, rows, cols, ld, k, ids, dst, keys, out_ld, col_base);
  return cudaGetLastError();
}

cudaError_t select_dispatch(const float *dist, size_t rows, size_t cols, size_t ld, int k,
                            uint32_t *ids, float *dst, unsigned long long *keys, size_t out_ld,
                            uint32_t col_base, cudaStream_t s) {
  if (rows == 0 || k <= 0) return cudaSuccess;
  if (k <= 32) return launch_select_impl<1>(dist, rows, cols, ld, k, ids, dst, keys, out_ld, col_base, s);
  if (k <= 64) return launch_select_impl<2>(dist, rows, cols, ld, k, ids, dst, keys, out_ld, col_base, s);
  if (k <= 128) return launch_select_impl<4>(dist, rows, cols, ld, k, ids, dst, keys, out_ld, col_base, s);
  if (k <= 256) return launch_select_impl<8>(dist, rows, cols, ld, k, ids, dst, keys, out_ld, col_base, s);
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t launch_select_rows(const float *dist, size_t rows, size_t cols, size_t ld, int k,
                               uint32_t *out_ids, float *out_dist, size_t out_ld, uint32_t col_base,
                               cudaStream_t s) {
  return select_dispatch(dist, rows, cols, ld, k, out_ids, out_dist, nullptr, out_ld, col_base, s);
}

cudaError_t launch_select_rows_keys(const float *dist, size_t rows, size_t cols, size_t ld, int k,
                                    unsigned long long *out_keys, size_t out_ld, uint32_t col_base,
                                    cudaStream_t s) {
  return select_dispatch(dist, rows, cols, ld, k, nullptr, nullptr, out_keys, out_ld, col_base, s);
}

// ---------------------------------------------------------------------------
// List-major pair grouping (counting sort by list id).
// ---------------------------------------------------------------------------
namespace {
constexpr uint32_t kNoList = 0xffffffffu;

__global__ void count_pairs_kernel(const uint32_t *__restrict__ probes, size_t total,
                                   const uint8_t *__restrict__ owner, size_t L, uint32_t *counts,
                                   const uint64_t *__restrict__ list_off, int M, bool four_bit,
                                   unsigned long long *stats) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  uint32_t l = probes[i];
  if (l == kNoList || l >= L) return;
  if (owner && !owner[l]) return;
  atomicAdd(counts + l, 1u);
  if (stats) {
    unsigned long long len = list_off[l + 1] - list_off[l];
    unsigned long long bytes = (four_bit && len >= 16) ? ((len + 31) / 32) * 16ull * M : len * M;
    atomicAdd(stats + 0, 1ull);
    atomicAdd(stats + 1, len);
    atomicAdd(stats + 2, bytes);
  }
}

// Exclusive scan of counts[0..L) into cursor, total into *d_total.  One block
// of 1024 threads; each thread owns a contiguous chunk.
__global__ void __launch_bounds__(1024) scan_counts_kernel(const uint32_t *__restrict__ counts,
                                                           size_t L, uint32_t *__restrict__ cursor,
                                                           uint32_t *__restrict__ d_total) {
  __shared__ uint32_t warp_sums[32];
  const int tid = threadIdx.x;
  const size_t chunk = (L + 1023) / 1024;
  const size_t beg = tid * chunk < L ? tid * chunk : L;
  const size_t end = beg + chunk < L ? beg + chunk : L;
  uint32_t local = 0;
  for (size_t i = beg; i < end; ++i) local += counts[i];
  // inclusive warp scan
  uint32_t v = local;
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t o = __shfl_up_sync(VG_FULL_MASK, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = warp_sums[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      uint32_t o = __shfl_up_sync(VG_FULL_MASK, w, off);
      if (lane >= off) w += o;
    }
    warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  uint32_t excl = v - local + (warp > 0 ? warp_sums[warp - 1] : 0u);
  for (size_t i = beg; i < end; ++i) {
    cursor[i] = excl;
    excl += counts[i];
  }
  if (tid == 1023) *d_total = warp_sums[31];
}

__global__ void scatter_pairs_kernel(const uint32_t *__restrict__ probes, size_t total,
                                     const uint8_t *__restrict__ owner, size_t L,
                                     uint32_t *cursor, uint32_t *__restrict__ work) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  uint32_t l = probes[i];
  if (l == kNoList || l >= L) return;
  if (owner && !owner[l]) return;
  uint32_t pos = atomicAdd(cursor + l, 1u);
  work[pos] = static_cast<uint32_t>(i);
}
}  // namespace

cudaError_t launch_build_pairs(const uint32_t *probes, size_t B, int P, const uint8_t *owner, size_t L,
                               uint32_t *counts, uint32_t *cursor, uint32_t *work, uint32_t *d_total,
                               const uint64_t *list_off, int M, bool four_bit, unsigned long long *stats,
                               cudaStream_t s) {
  size_t total = B * static_cast<size_t>(P);
  cudaError_t e = cudaMemsetAsync(counts, 0, L * sizeof(uint32_t), s);
  if (e != cudaSuccess) return e;
  if (total == 0) return cudaMemsetAsync(d_total, 0, sizeof(uint32_t), s);
  dim3 grid(static_cast<unsigned>((total + 255) / 256));
  count_pairs_kernel<<<grid, 256, 0, s>>>(probes, total, owner, L, counts, list_off, M, four_bit,
                                          list_off ? stats : nullptr);
  scan_counts_kernel<<<1, 1024, 0, s>>>(counts, L, cursor, d_total);
  scatter_pairs_kernel<<<grid, 256, 0, s>>>(probes, total, owner, L, cursor, work);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Profiling counters of scanned work (block-reduced, three atomics per block).
// ---------------------------------------------------------------------------
namespace {
__global__ void probe_stats_kernel(const uint32_t *__restrict__ probes, size_t total,
                                   const uint8_t *__restrict__ owner, size_t L,
                                   const uint64_t *__restrict__ list_off, int M, bool four_bit,
                                   unsigned long long *stats) {
  __shared__ unsigned long long part[3][8];
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  unsigned long long pairs = 0, vecs = 0, bytes = 0;
  if (i < total) {
    uint32_t l = probes[i];
    if (l != kNoList && l < L && (!owner || owner[l])) {
      unsigned long long len = list_off[l + 1] - list_off[l];
      pairs = 1;
      vecs = len;
      bytes = (four_bit && len >= 16) ? ((len + 31) / 32) * 16ull * M : len * M;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    pairs += __shfl_xor_sync(VG_FULL_MASK, pairs, off);
    vecs += __shfl_xor_sync(VG_FULL_MASK, vecs, off);
    bytes += __shfl_xor_sync(VG_FULL_MASK, bytes, off);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    part[0][w] = pairs;
    part[1][w] = vecs;
    part[2][w] = bytes;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    unsigned long long t = 0;
    for (int j = 0; j < static_cast<int>(blockDim.x >> 5); ++j) t += part[threadIdx.x][j];
    if (t) atomicAdd(stats + threadIdx.x, t);
  }
}
}  // namespace

cudaError_t launch_probe_stats(const uint32_t *probes, size_t B, int P, const uint8_t *owner, size_t L,
                               const uint64_t *list_off, int M, bool four_bit, unsigned long long *stats,
                               cudaStream_t s) {
  size_t total = B * static_cast<size_t>(P);
  if (total == 0 || !stats) return cudaSuccess;
  probe_stats_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(probes, total, owner, L, list_off, M,
                                                                              four_bit, stats);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Merges: warp per row over segmented key arrays.
// Candidate j of row r lives at keys[(j / seg_len) * seg_stride + r * row_stride + j % seg_len].
// ---------------------------------------------------------------------------
namespace {
template <int R>
__global__ void __launch_bounds__(256)
    merge_kernel(const unsigned long long *__restrict__ keys, size_t rows, size_t width,
                 size_t seg_len, size_t seg_stride, size_t row_stride, int k,
                 const uint32_t *__restrict__ ids_map, uint32_t *__restrict__ out_ids,
                 float *__restrict__ out_dist, uint32_t *__restrict__ out_count,
                 unsigned long long *__restrict__ out_keys) {
  const size_t row = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const int lane = lane_id();
  WarpTopK<R> tk;
  tk.init();
  for (size_t j0 = 0; j0 < width; j0 += 32) {
    size_t j = j0 + lane;
    uint64_t key = kEmptyKey;
    if (j < width) {
      size_t seg = j / seg_len, off = j - seg * seg_len;
      key = keys[seg * seg_stride + row * row_stride + off];
    }
    tk.add(key);
  }
  uint32_t count = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int i = r * 32 + lane;
    uint64_t key = tk.v[r];
    bool real = (i < k) && key != kEmptyKey;
    count += __popc(__ballot_sync(VG_FULL_MASK, real));
    if (i < k) {
      if (out_keys) out_keys[row * k + i] = key;
      if (out_ids) {
        out_ids[row * k + i] = real ? (ids_map ? ids_map[key_id(key)] : key_id(key)) : 0xffffffffu;
        out_dist[row * k + i] = real ? key_dist(key) : __int_as_float(0x7f800000);
      }
    }
  }
  if (out_count && lane == 0) out_count[row] = count;
}

cudaError_t merge_dispatch(const unsigned long long *keys, size_t rows, size_t width, size_t seg_len,
                           size_t seg_stride, size_t row_stride, int k, const uint32_t *ids_map,
                           uint32_t *out_ids, float *out_dist, uint32_t *out_count,
                           unsigned long long *out_keys, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((rows * 32 + 255) / 256));
#define VG_MERGE(RR)                                                                               \
  merge_kernel<RR><<<grid, 256, 0, s>>>(keys, rows, width, seg_len, seg_stride, row_stride, k,     \
                                        ids_map, out_ids, out_dist, out_count, out_keys)
  if (k <= 32)
    VG_MERGE(1);
  else if (k <= 64)
    VG_MERGE(2);
  else if (k <= 128)
    VG_MERGE(4);
  else if (k <= 256)
    VG_MERGE(8);
  else
    return cudaErrorInvalidValue;
#undef VG_MERGE
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_merge_keys(const unsigned long long *keys, size_t rows, size_t width, size_t row_stride,
                              int k, const uint32_t *ids_map, uint32_t *out_ids, float *out_dist,
                              uint32_t *out_count, unsigned long long *out_keys, cudaStream_t s) {
  size_t seg = width ? width : 1;
  return merge_dispatch(keys, rows, width, seg, 0, row_stride, k, ids_map, out_ids, out_dist, out_count,
                        out_keys, s);
}

namespace {
__device__ __forceinline__ void push_work(uint32_t item, bool heavy, uint32_t *work, uint32_t *count,
                                          uint32_t cap) {
  if (heavy)
    work[atomicAdd(count, 1u)] = item;
  else
    work[cap - 1 - atomicAdd(count + 1, 1u)] = item;
}

__global__ void order_seed_kernel(const uint32_t *__restrict__ probes, int P, const uint8_t *__restrict__ owner,
                                  const uint64_t *__restrict__ list_off, size_t nq, uint32_t heavy,
                                  uint32_t *__restrict__ work, uint32_t *__restrict__ count, uint32_t cap,
                                  uint32_t *__restrict__ seed_next) {
  const size_t q = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const uint32_t l = probes[q * P];
  if (l == 0xffffffffu || (owner && !owner[l])) {
    if (seed_next)
      seed_next[q] = 1;
    else
      push_work(static_cast<uint32_t>(q), false, work, count, cap);
    return;
  }
  push_work(static_cast<uint32_t>(q), list_off[l + 1] - list_off[l] >= heavy, work, count, cap);
}

__global__ void order_units_kernel(const uint32_t *__restrict__ probes, int P, int G,
                                   const uint8_t *__restrict__ owner, const uint64_t *__restrict__ list_off,
                                   const float *__restrict__ bound, const unsigned long long *__restrict__ ceiling,
                                   const uint32_t *__restrict__ first, size_t nq, uint32_t heavy,
                                   uint32_t *__restrict__ work, uint32_t *__restrict__ count, uint32_t cap) {
  const uint32_t U = static_cast<uint32_t>((P + G - 1) / G);
  const size_t it = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (it >= nq * U) return;
  const size_t q = it / U;
  const int g = static_cast<int>(it - q * U);
  const int lo = max(first ? static_cast<int>(first[q]) : 0, g * G), hi = min(P, (g + 1) * G);
  const uint64_t c = ceiling ? ceiling[q] : kEmptyKey;
  uint64_t vecs = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t l = probes[q * P + i];
    if (l == 0xffffffffu || (owner && !owner[l])) continue;
    if (bound && c != kEmptyKey && bound[q * P + i] > key_dist(c + 1)) continue;  // the scan prunes it
    vecs += list_off[l + 1] - list_off[l];
  }
  if (vecs) push_work(static_cast<uint32_t>(it), vecs >= heavy, work, count, cap);
}
}  // namespace

cudaError_t launch_order_seed(const uint32_t *probes, int P, const uint8_t *owner, const uint64_t *list_off,
                              size_t nq, uint32_t heavy, uint32_t *work, uint32_t *count, uint32_t cap,
                              uint32_t *seed_next, cudaStream_t s) {
  if (nq == 0) return cudaSuccess;
  if (nq > cap) return cudaErrorInvalidValue;
  order_seed_kernel<<<static_cast<unsigned>((nq + 255) / 256), 256, 0, s>>>(probes, P, owner, list_off, nq, heavy,
                                                                            work, count, cap, seed_next);
  return cudaGetLastError();
}

cudaError_t launch_order_units(const uint32_t *probes, int P, int G, const uint8_t *owner, const uint64_t *list_off,
                               const float *bound, const unsigned long long *ceiling, const uint32_t *first,
                               size_t nq, uint32_t heavy, uint32_t *work, uint32_t *count, uint32_t cap,
                               cudaStream_t s) {
  if (G < 1 || P < 1) return cudaErrorInvalidValue;
  const size_t items = nq * static_cast<size_t>((P + G - 1) / G);
  if (items == 0) return cudaSuccess;
  if (items > cap) return cudaErrorInvalidValue;
  order_units_kernel<<<static_cast<unsigned>((items + 255) / 256), 256, 0, s>>>(
      probes, P, G, owner, list_off, bound, ceiling, first, nq, heavy, work, count, cap);
  return cudaGetLastError();
}

cudaError_t launch_merge_shards(const unsigned long long *keys, int G, size_t rows, int k,
                                const uint32_t *ids_map, uint32_t *out_ids, float *out_dist,
                                uint32_t *out_count, unsigned long long *out_keys, cudaStream_t s) {
  return merge_dispatch(keys, rows, static_cast<size_t>(G) * k, static_cast<size_t>(k), rows * k,
                        static_cast<size_t>(k), k, ids_map, out_ids, out_dist, out_count, out_keys, s);
}

// ---------------------------------------------------------------------------
// Filtered search helpers.
// ---------------------------------------------------------------------------
namespace {
__global__ void category_counts_kernel(const uint8_t *__restrict__ category, const uint32_t *__restrict__ assign,
                                       size_t n, uint32_t *counts) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t c = category[i];
  if (c < 64) atomicAdd(counts + static_cast<size_t>(assign[i]) * 64 + c, 1u);
}

__global__ void filter_widen_kernel(const uint32_t *__restrict__ probes, size_t nq, int P,
                                    const uint64_t *__restrict__ bitmask, const uint32_t *__restrict__ counts,
                                    int want, size_t k, uint8_t *__restrict__ widen) {
  const size_t q = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  uint64_t found = 0;
  for (int i = 0; i < P; ++i) {
    const uint32_t l = probes[q * P + i];
    if (l != 0xffffffffu && ((bitmask[l] >> want) & 1ull)) found += counts[static_cast<size_t>(l) * 64 + want];
  }
  widen[q] = found < k ? 1 : 0;
}
}  // namespace

cudaError_t launch_category_counts(const uint8_t *category, const uint32_t *assign, size_t n, uint32_t *counts,
                                   cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  category_counts_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(category, assign, n, counts);
  return cudaGetLastError();
}

cudaError_t launch_filter_widen(const uint32_t *probes, size_t nq, int P, const uint64_t *bitmask,
                                const uint32_t *counts, int want, size_t k, uint8_t *widen, cudaStream_t s) {
  if (nq == 0) return cudaSuccess;
  filter_widen_kernel<<<static_cast<unsigned>((nq + 127) / 128), 128, 0, s>>>(probes, nq, P, bitmask, counts, want,
                                                                            k, widen);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// List pruning bounds.  For candidate i of list l the exact value of the sums
// the scan computes is E_i = ||r - w_i||^2 (r: the float residual, w_i: the
// concatenated codewords), which is >= (||r|| - ||w_i||)^2 >= (||r|| - R_l)^2
// when ||r|| > R_l.  The computed sum of non-negative terms is >= E_i (1-u)^n
// with n = M + dsub + 1 roundings on the longest chain (u = 2^-24).  Norms are
// taken in double from the float values, so the bound is rigorous; it is
// scaled by 1 - (n + 1) u and rounded down to float.
// ---------------------------------------------------------------------------
namespace {
__global__ void probe_lb_kernel(const float *__restrict__ qn, size_t nq, int d, const uint32_t *__restrict__ probes,
                                int P, const float *__restrict__ centroids, const ProbeBoundArgs b) {
  const size_t pair = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (pair >= nq * P) return;
  const int lane = lane_id();
  const size_t q = pair / P;
  const uint32_t l = probes[pair];
  if (l == 0xffffffffu || (b.owner && !b.owner[l])) {
    if (lane == 0) {
      b.lb[pair] = 0.0f;
      if (b.lbq) b.lbq[pair] = 0.0f;
      if (b.rec) b.rec[pair] = ProbeRec{0xffffffffu, 0u, 0ull, 0ull, 0.0f, 0u};
    }
    return;
  }
  const float *qv = qn + q * d;
  const float *c = centroids + static_cast<size_t>(l) * d;
  // lane m takes subspaces m, m + 32, ...: their squared residual norms give
  // both |r|^2 and the 4-bit table bound
  double s = 0.0;
  float smax = 0.0f;
  for (int m = lane; m < b.M; m += 32) {
    float sm = 0.0f;
    for (int jj = 0; jj < b.dsub; ++jj) {
      const float r = __fsub_rn(qv[m * b.dsub + jj], c[m * b.dsub + jj]);  // the scan kernels' residual
      s += static_cast<double>(r) * r;
      sm = __fmaf_ru(r, r, sm);
    }
    smax = fmaxf(smax, sm);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    s += __shfl_xor_sync(VG_FULL_MASK, s, off);
    smax = fmaxf(smax, __shfl_xor_sync(VG_FULL_MASK, smax, off));
  }
  if (lane == 0) {
    // double rounding of d squares and sums: relative < 1e-13, covered by lb_from_norm
    const float lbf = lb_from_norm(s, b.radius[l], b.M, b.dsub);
    b.lb[pair] = lbf;
    if (b.lbq) b.lbq[pair] = lbq_from_lb(lbf, table_max_bound(smax, b.sub_radius[b.M]), b.M, b.dsub);
    if (b.rec) {
      const uint64_t beg = b.list_off[l];
      b.rec[pair] = ProbeRec{l, static_cast<uint32_t>(b.list_off[l + 1] - beg), beg, b.code_off[l], lbf, 0u};
    }
  }
}
}  // namespace

cudaError_t launch_probe_lb(const float *qn, size_t nq, int d, const uint32_t *probes, int P,
                            const float *centroids, const ProbeBoundArgs &b, cudaStream_t s) {
  const size_t pairs = nq * static_cast<size_t>(P);
  if (pairs == 0) return cudaSuccess;
  probe_lb_kernel<<<static_cast<unsigned>((pairs * 32 + 255) / 256), 256, 0, s>>>(qn, nq, d, probes, P, centroids, b);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Exact rerank (search.rs:1117-1158): each approximate candidate is re-scored
// with cosine_distance_normalized = 1 - dot(q, x) (distance.rs:104-109), the
// dot summed in index order, then the k best are kept.  Warp per query; lane
// i scores candidates i, i+32, ...
// ---------------------------------------------------------------------------
namespace {
template <int R>
__global__ void __launch_bounds__(256)
    rerank_kernel(const float *__restrict__ qn, const float *__restrict__ vectors, int d,
                  const unsigned long long *__restrict__ cand, size_t rows, int width, int k,
                  const uint32_t *__restrict__ ids_map, uint32_t *__restrict__ out_ids,
                  float *__restrict__ out_dist, uint32_t *__restrict__ out_count) {
  const size_t row = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const int lane = lane_id();
  const float *q = qn + row * d;
  WarpTopK<R> tk;
  tk.init();
  for (int j0 = 0; j0 < width; j0 += 32) {
    int j = j0 + lane;
    uint64_t key = kEmptyKey;
    if (j < width) {
      uint64_t c = cand[row * width + j];
      if (c != kEmptyKey) {
        const float *x = vectors + static_cast<size_t>(key_id(c)) * d;
        float dot = 0.0f;
        for (int t = 0; t < d; ++t) dot = __fadd_rn(dot, __fmul_rn(q[t], x[t]));
        key = pack_key(__fsub_rn(1.0f, dot), key_id(c));
      }
    }
    tk.add(key);
  }
  uint32_t count = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    int i = r * 32 + lane;
    uint64_t key = tk.v[r];
    bool real = (i < k) && key != kEmptyKey;
    count += __popc(__ballot_sync(VG_FULL_MASK, real));
    if (i < k) {
      out_ids[row * k + i] = real ? ids_map[key_id(key)] : 0xffffffffu;
      out_dist[row * k + i] = real ? key_dist(key) : __int_as_float(0x7f800000);
    }
  }
  if (out_count && lane == 0) out_count[row] = count;
}
}  // namespace

cudaError_t launch_rerank(const float *qn, const float *vectors, int d, const unsigned long long *cand,
                          size_t rows, int width, int k, const uint32_t *ids_map, uint32_t *out_ids,
                          float *out_dist, uint32_t *out_count, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((rows * 32 + 255) / 256));
#define VG_RERANK(RR) \
  rerank_kernel<RR><<<grid, 256, 0, s>>>(qn, vectors, d, cand, rows, width, k, ids_map, out_ids, out_dist, out_count)
  if (k <= 32)
    VG_RERANK(1);
  else if (k <= 64)
    VG_RERANK(2);
  else if (k <= 128)
    VG_RERANK(4);
  else if (k <= 256)
    VG_RERANK(8);
  else
    return cudaErrorInvalidValue;
#undef VG_RERANK
  return cudaGetLastError();
}

}  // namespace vg

// ---------------------------------------------------------------------------
// List-sharded search helpers.
// ---------------------------------------------------------------------------
namespace vg {
namespace {
__global__ void probe_records_kernel(const uint32_t *__restrict__ probes, const float *__restrict__ lb, size_t n,
                                     const uint8_t *__restrict__ owner, const uint64_t *__restrict__ list_off,
                                     const uint64_t *__restrict__ code_off, ProbeRec *__restrict__ rec) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t l = probes[i];
  if (l == 0xffffffffu || (owner && !owner[l])) {
    rec[i] = ProbeRec{0xffffffffu, 0u, 0ull, 0ull, 0.0f, 0u};
    return;
  }
  const uint64_t beg = list_off[l];
  rec[i] = ProbeRec{l, static_cast<uint32_t>(list_off[l + 1] - beg), beg, code_off[l], lb[i], 0u};
}

// block per segment: bytes[s] bytes from src + src_off[s] to dst + dst_off[s]
__global__ void copy_segments_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                     const uint64_t *__restrict__ src_off, const uint64_t *__restrict__ dst_off,
                                     const uint64_t *__restrict__ bytes) {
  const size_t sgm = blockIdx.x;
  const uint8_t *a = src + src_off[sgm];
  uint8_t *b = dst + dst_off[sgm];
  const uint64_t nb = bytes[sgm];
  if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) == 0) {
    const uint64_t n16 = nb >> 4;
    for (uint64_t i = threadIdx.x; i < n16; i += blockDim.x)
      reinterpret_cast<uint4 *>(b)[i] = reinterpret_cast<const uint4 *>(a)[i];
    for (uint64_t i = (n16 << 4) + threadIdx.x; i < nb; i += blockDim.x) b[i] = a[i];
  } else {
    for (uint64_t i = threadIdx.x; i < nb; i += blockDim.x) b[i] = a[i];
  }
}
}  // namespace

cudaError_t launch_probe_records(const uint32_t *probes, const float *lb, size_t n, const uint8_t *owner,
                                 const uint64_t *list_off, const uint64_t *code_off, ProbeRec *rec, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  probe_records_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(probes, lb, n, owner, list_off,
                                                                              code_off, rec);
  return cudaGetLastError();
}

cudaError_t launch_copy_segments(const void *src, void *dst, const uint64_t *src_off, const uint64_t *dst_off,
                                 const uint64_t *bytes, size_t count, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  copy_segments_kernel<<<static_cast<unsigned>(count), 256, 0, s>>>(static_cast<const uint8_t *>(src),
                                                                    static_cast<uint8_t *>(dst), src_off, dst_off,
                                                                    bytes);
  return cudaGetLastError();
}
}  // namespace vg
