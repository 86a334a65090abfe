// Build-side kernels: residual encoding, list construction, FastScan packing
// and the deterministic Lloyd updates used by training.
//
// Reference behaviour restated here (vicinity 0.12.0):
//   residuals                 src/ivf_pq/search.rs:720-729
//   ProductQuantizer::quantize src/ivf_pq/pq.rs:136-160 (strict <, first
//                             minimum wins; sequential squared-L2 sum)
//   lists in vector order     src/ivf_pq/search.rs:623-718
//   list-contiguous codes     src/ivf_pq/file_storage.rs:39-72
//   PackedCodes4bit::pack     src/pq_simd.rs:426-486
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"
#include "kernels.h"

namespace vg {

namespace {
constexpr int kMaxRegDsub = 16;

// One thread per vector for subspace m = blockIdx.y; the subspace codebook
// sits in shared memory and every lane of a warp reads the same codeword.
template <bool HAS_CENT>
__global__ void __launch_bounds__(256)
    encode_kernel(const float *__restrict__ x, size_t n, int d, const uint32_t *__restrict__ assign,
                  const float *__restrict__ cent, const float *__restrict__ codebooks, int M, int ks,
                  uint8_t *__restrict__ codes) {
  extern __shared__ float cw[];  // [ks][dsub]
  const int m = blockIdx.y;
  const int dsub = d / M;
  for (int i = threadIdx.x; i < ks * dsub; i += blockDim.x)
    cw[i] = codebooks[static_cast<size_t>(m) * ks * dsub + i];
  __syncthreads();
  const size_t v = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (v >= n) return;
  const float *xv = x + v * d + m * dsub;
  const float *cv = HAS_CENT ? cent + static_cast<size_t>(assign[v]) * d + m * dsub : nullptr;
  int best = 0;
  float best_dist = __int_as_float(0x7f800000);
  if (dsub <= kMaxRegDsub) {
    float r[kMaxRegDsub];
#pragma unroll
    for (int j = 0; j < kMaxRegDsub; ++j)
      r[j] = j < dsub ? (HAS_CENT ? __fsub_rn(xv[j], cv[j]) : xv[j]) : 0.0f;
    for (int c = 0; c < ks; ++c) {
      const float *w = cw + c * dsub;
      float dist = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxRegDsub; ++j) {
        if (j < dsub) {
          float diff = __fsub_rn(r[j], w[j]);
          dist = __fadd_rn(dist, __fmul_rn(diff, diff));
        }
      }
      if (dist < best_dist) {
        best_dist = dist;
        best = c;
      }
    }
  } else {
    for (int c = 0; c < ks; ++c) {
      const float *w = cw + c * dsub;
      float dist = 0.0f;
      for (int j = 0; j < dsub; ++j) {
        float rj = HAS_CENT ? __fsub_rn(xv[j], cv[j]) : xv[j];
        float diff = __fsub_rn(rj, w[j]);
        dist = __fadd_rn(dist, __fmul_rn(diff, diff));
      }
      if (dist < best_dist) {
        best_dist = dist;
        best = c;
      }
    }
  }
  codes[v * M + m] = static_cast<uint8_t>(best < 255 ? best : 255);
}

template <bool HAS_CENT>
cudaError_t launch_encode_impl(const float *x, size_t n, int d, const uint32_t *assign, const float *cent,
                               const float *codebooks, int M, int ks, uint8_t *codes, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int dsub = d / M;
  size_t smem = static_cast<size_t>(ks) * dsub * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(encode_kernel<HAS_CENT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  dim3 grid(static_cast<unsigned>((n + 255) / 256), static_cast<unsigned>(M));
  encode_kernel<HAS_CENT><<<grid, 256, smem, s>>>(x, n, d, assign, cent, codebooks, M, ks, codes);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_encode(const float *xn, size_t n, int d, const uint32_t *assign, const float *cent,
                          const float *codebooks, int M, int ks, uint8_t *codes, cudaStream_t s) {
  return launch_encode_impl<true>(xn, n, d, assign, cent, codebooks, M, ks, codes, s);
}

cudaError_t launch_encode_residuals(const float *r, size_t n, int d, const float *codebooks, int M, int ks,
                                    uint8_t *codes, cudaStream_t s) {
  return launch_encode_impl<false>(r, n, d, nullptr, nullptr, codebooks, M, ks, codes, s);
}

namespace {
__global__ void residuals_kernel(const float *__restrict__ x, size_t n, int d, const uint32_t *__restrict__ assign,
                                 const float *__restrict__ cent, float *__restrict__ out) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * d) return;
  size_t v = i / d;
  int j = static_cast<int>(i - v * d);
  out[i] = __fsub_rn(x[i], cent[static_cast<size_t>(assign[v]) * d + j]);
}

__global__ void keys_to_assign_kernel(const unsigned long long *__restrict__ best, size_t n,
                                      uint32_t *__restrict__ assign, const uint32_t *__restrict__ prev,
                                      unsigned int *changed) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t a = static_cast<uint32_t>(best[i] & 0xffffffffull);
  assign[i] = a;
  if (prev && prev[i] != a) atomicAdd(changed, 1u);
}

__global__ void gather_list_codes_kernel(const uint8_t *__restrict__ codes, const uint32_t *__restrict__ sorted_ids,
                                         const uint32_t *__restrict__ sorted_lists, size_t n, int M,
                                         const uint64_t *__restrict__ list_off,
                                         const uint64_t *__restrict__ code_off, uint8_t *__restrict__ out) {
  size_t p = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= n) return;
  uint32_t l = sorted_lists[p];
  const uint8_t *src = codes + static_cast<size_t>(sorted_ids[p]) * M;
  uint8_t *dst = out + code_off[l] + (p - list_off[l]) * M;
  for (int m = 0; m < M; ++m) dst[m] = src[m];
}

// 4-bit codes of every list with at least 16 vectors (the lists the
// reference scans with quantised tables, search.rs:816-848) repacked for the
// GPU scan: vector-major, two codes per byte (code 2j in the low nibble,
// 2j + 1 in the high one), ceil(M/2) bytes per vector, so one thread loads a
// whole vector with a few wide loads.  Lists under 16 vectors keep no packed
// copy (search.rs:824-828).
__global__ void pack_nibbles_kernel(const uint8_t *__restrict__ list_codes, const uint64_t *__restrict__ list_off,
                                    const uint64_t *__restrict__ code_off, const uint64_t *__restrict__ pack_off,
                                    int M, uint8_t *__restrict__ packed) {
  const size_t l = blockIdx.x;
  const uint64_t len = list_off[l + 1] - list_off[l];
  if (len < 16) return;
  const int vs = (M + 1) / 2;
  const uint8_t *src = list_codes + code_off[l];
  uint8_t *dst = packed + pack_off[l];
  for (uint64_t i = threadIdx.x; i < len * vs; i += blockDim.x) {
    const uint64_t v = i / vs;
    const int j = static_cast<int>(i - v * vs);
    const uint8_t lo = src[v * M + 2 * j] & 0x0f;
    const uint8_t hi = 2 * j + 1 < M ? (src[v * M + 2 * j + 1] & 0x0f) : 0;
    dst[i] = static_cast<uint8_t>(lo | (hi << 4));
  }
}

// Largest reconstructed-residual norm of each list (double, rounded up).
__global__ void list_radius_kernel(const uint8_t *__restrict__ list_codes, const uint64_t *__restrict__ code_off,
                                   const uint64_t *__restrict__ list_off, int M, int ks, int dsub,
                                   const float *__restrict__ codebooks, float *__restrict__ radius) {
  __shared__ double red[32];
  const size_t l = blockIdx.x;
  const uint64_t len = list_off[l + 1] - list_off[l];
  const uint8_t *codes = list_codes + code_off[l];
  double best = 0.0;
  for (uint64_t v = threadIdx.x; v < len; v += blockDim.x) {
    double s = 0.0;
    for (int m = 0; m < M; ++m) {
      const float *cw = codebooks + (static_cast<size_t>(m) * ks + codes[v * M + m]) * dsub;
      for (int j = 0; j < dsub; ++j) s += static_cast<double>(cw[j]) * static_cast<double>(cw[j]);
    }
    best = s > best ? s : best;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const double o = __shfl_xor_sync(0xffffffffu, best, off);
    best = o > best ? o : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (unsigned w = 1; w < (blockDim.x + 31) / 32; ++w) best = red[w] > best ? red[w] : best;
    radius[l] = __double2float_ru(sqrt(best) * (1.0 + 1e-12));
  }
}

// Largest codeword norm of each subspace (double, rounded up): rad[m] =
// max_c |codebooks[m][c]|, and rad[M] = max_m rad[m].  One block.
__global__ void subspace_radius_kernel(const float *__restrict__ codebooks, int M, int ks, int dsub,
                                       float *__restrict__ rad) {
  __shared__ float red[32];
  float top = 0.0f;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    double best = 0.0;
    for (int c = 0; c < ks; ++c) {
      const float *cw = codebooks + (static_cast<size_t>(m) * ks + c) * dsub;
      double s = 0.0;
      for (int j = 0; j < dsub; ++j) s += static_cast<double>(cw[j]) * static_cast<double>(cw[j]);
      best = (s > best || s != s) ? s : best;
    }
    const float r = __double2float_ru(sqrt(best) * (1.0 + 1e-12));
    rad[m] = r;
    top = (r > top || r != r) ? r : top;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, top, off);
    top = (o > top || o != o) ? o : top;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = top;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (unsigned w = 1; w < (blockDim.x + 31) / 32; ++w) top = (red[w] > top || red[w] != red[w]) ? red[w] : top;
    rad[M] = top;
  }
}

// Largest centroid norm, rounded up; NaN when any centroid holds a NaN (so
// that a consumer's bound fails its finiteness test).  One block.
__global__ void centroid_norm_max_kernel(const float *__restrict__ cent, size_t L, int d, float *__restrict__ out) {
  __shared__ double red[32];
  double best = 0.0;
  for (size_t l = threadIdx.x; l < L; l += blockDim.x) {
    double s = 0.0;
    for (int j = 0; j < d; ++j) s += static_cast<double>(cent[l * d + j]) * static_cast<double>(cent[l * d + j]);
    best = (s > best || s != s) ? s : best;
  }
  for (int off = 16; off > 0; off >>= 1) {
    const double o = __shfl_xor_sync(0xffffffffu, best, off);
    best = (o > best || o != o) ? o : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (unsigned w = 1; w < (blockDim.x + 31) / 32; ++w) best = (red[w] > best || red[w] != red[w]) ? red[w] : best;
    *out = __double2float_ru(sqrt(best) * (1.0 + 1e-12));
  }
}

// Deterministic cluster mean: members are visited in ascending order and
// each dimension is summed sequentially by one thread.
__global__ void kmeans_update_kernel(const float *__restrict__ x, int d, const uint32_t *__restrict__ sorted_ids,
                                     const uint32_t *__restrict__ seg, const float *__restrict__ old_cent,
                                     float *__restrict__ new_cent, int spherical) {
  __shared__ float red[32];
  const size_t c = blockIdx.x;
  const uint32_t beg = seg[c], end = seg[c + 1];
  float *out = new_cent + c * d;
  if (beg == end) {
    for (int j = threadIdx.x; j < d; j += blockDim.x) out[j] = old_cent[c * d + j];
    return;
  }
  const float inv_count = 1.0f / static_cast<float>(end - beg);
  float sq = 0.0f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float s = 0.0f;
    for (uint32_t t = beg; t < end; ++t) s += x[static_cast<size_t>(sorted_ids[t]) * d + j];
    float mean = s * inv_count;
    out[j] = mean;
    sq += mean * mean;
  }
  if (!spherical) return;
  for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(VG_FULL_MASK, sq, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? red[threadIdx.x] : 0.0f;
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(VG_FULL_MASK, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float norm = sqrtf(red[0]);
  if (norm > 1e-10f)
    for (int j = threadIdx.x; j < d; j += blockDim.x) out[j] = out[j] / norm;
}

// PQ codeword means: segment (m, c) lists the residual rows coded c in m.
__global__ void pq_update_kernel(const float *__restrict__ x, int d, int M, int ks,
                                 const uint32_t *__restrict__ sorted_rows, const uint32_t *__restrict__ seg,
                                 const float *__restrict__ old_cb, float *__restrict__ new_cb) {
  const size_t sidx = blockIdx.x;  // m * ks + c
  const int m = static_cast<int>(sidx / ks);
  const int dsub = d / M;
  const uint32_t beg = seg[sidx], end = seg[sidx + 1];
  float *out = new_cb + sidx * dsub;
  for (int j = threadIdx.x; j < dsub; j += blockDim.x) {
    if (beg == end) {
      out[j] = old_cb[sidx * dsub + j];
      continue;
    }
    float s = 0.0f;
    for (uint32_t t = beg; t < end; ++t) s += x[static_cast<size_t>(sorted_rows[t]) * d + m * dsub + j];
    out[j] = s / static_cast<float>(end - beg);
  }
}

__global__ void gather_rows_kernel(const float *__restrict__ x, int d, const uint32_t *__restrict__ rows,
                                   size_t n, float *__restrict__ out) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * d) return;
  size_t r = i / d;
  out[i] = x[static_cast<size_t>(rows[r]) * d + (i - r * d)];
}

__global__ void iota_kernel(uint32_t *out, size_t n) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<uint32_t>(i);
}

// keys[i] = m * ks + codes[row][m] for i = row * M + m; vals[i] = row.
__global__ void pq_keys_kernel(const uint8_t *__restrict__ codes, size_t n, int M, int ks,
                               uint32_t *__restrict__ keys, uint32_t *__restrict__ vals) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * M) return;
  size_t row = i / M;
  int m = static_cast<int>(i - row * M);
  keys[i] = static_cast<uint32_t>(m * ks + codes[i]);
  vals[i] = static_cast<uint32_t>(row);
}

// seg[c] = first position whose sorted key >= c (lower bound), c in [0, nseg].
__global__ void segments_kernel(const uint32_t *__restrict__ sorted_keys, size_t n, size_t nseg,
                                uint32_t *__restrict__ seg) {
  size_t c = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c > nseg) return;
  size_t lo = 0, hi = n;
  while (lo < hi) {
    size_t mid = (lo + hi) >> 1;
    if (sorted_keys[mid] < c)
      lo = mid + 1;
    else
      hi = mid;
  }
  seg[c] = static_cast<uint32_t>(lo);
}

inline dim3 grid_for(size_t n, int threads = 256) { return dim3(static_cast<unsigned>((n + threads - 1) / threads)); }
}  // namespace

cudaError_t launch_residuals(const float *xn, size_t n, int d, const uint32_t *assign, const float *cent,
                             float *out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  residuals_kernel<<<grid_for(n * d), 256, 0, s>>>(xn, n, d, assign, cent, out);
  return cudaGetLastError();
}

cudaError_t launch_keys_to_assign(const unsigned long long *best, size_t n, uint32_t *assign,
                                  const uint32_t *prev, unsigned int *changed, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  keys_to_assign_kernel<<<grid_for(n), 256, 0, s>>>(best, n, assign, prev, changed);
  return cudaGetLastError();
}

cudaError_t launch_gather_list_codes(const uint8_t *codes, const uint32_t *sorted_ids, const uint32_t *sorted_lists,
                                     size_t n, int M, const uint64_t *list_off, const uint64_t *code_off,
                                     uint8_t *list_codes, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  gather_list_codes_kernel<<<grid_for(n), 256, 0, s>>>(codes, sorted_ids, sorted_lists, n, M, list_off,
                                                       code_off, list_codes);
  return cudaGetLastError();
}

cudaError_t launch_pack_lists_4bit(const uint8_t *list_codes, const uint64_t *list_off, const uint64_t *code_off,
                                   const uint64_t *pack_off, size_t L, int M, uint8_t *packed,
                                   cudaStream_t s) {
  if (L == 0) return cudaSuccess;
  pack_nibbles_kernel<<<static_cast<unsigned>(L), 256, 0, s>>>(list_codes, list_off, code_off, pack_off, M, packed);
  return cudaGetLastError();
}

cudaError_t launch_list_radius(const uint8_t *list_codes, const uint64_t *code_off, const uint64_t *list_off,
                               size_t L, int M, int ks, int dsub, const float *codebooks, float *radius,
                               cudaStream_t s) {
  if (L == 0) return cudaSuccess;
  list_radius_kernel<<<static_cast<unsigned>(L), 256, 0, s>>>(list_codes, code_off, list_off, M, ks, dsub,
                                                              codebooks, radius);
  return cudaGetLastError();
}

cudaError_t launch_subspace_radius(const float *codebooks, int M, int ks, int dsub, float *rad, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  subspace_radius_kernel<<<1, 256, 0, s>>>(codebooks, M, ks, dsub, rad);
  return cudaGetLastError();
}

cudaError_t launch_centroid_norm_max(const float *cent, size_t L, int d, float *out, cudaStream_t s) {
  centroid_norm_max_kernel<<<1, 1024, 0, s>>>(cent, L, d, out);
  return cudaGetLastError();
}

cudaError_t launch_kmeans_update(const float *x, int d, const uint32_t *sorted_ids, const uint32_t *seg, size_t k,
                                 const float *old_cent, float *new_cent, int spherical, cudaStream_t s) {
  if (k == 0) return cudaSuccess;
  int threads = d >= 256 ? 256 : ((d + 31) / 32) * 32;
  kmeans_update_kernel<<<static_cast<unsigned>(k), threads, 0, s>>>(x, d, sorted_ids, seg, old_cent, new_cent,
                                                                    spherical);
  return cudaGetLastError();
}

cudaError_t launch_pq_update(const float *x, size_t, int d, int M, int ks, const uint32_t *sorted_rows,
                             const uint32_t *seg, const float *old_cb, float *new_cb, cudaStream_t s) {
  int dsub = d / M;
  int threads = dsub >= 128 ? 128 : ((dsub + 31) / 32) * 32;
  pq_update_kernel<<<static_cast<unsigned>(M * ks), threads, 0, s>>>(x, d, M, ks, sorted_rows, seg, old_cb,
                                                                     new_cb);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float *x, int d, const uint32_t *rows, size_t n, float *out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  gather_rows_kernel<<<grid_for(n * d), 256, 0, s>>>(x, d, rows, n, out);
  return cudaGetLastError();
}

cudaError_t launch_iota(uint32_t *out, size_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  iota_kernel<<<grid_for(n), 256, 0, s>>>(out, n);
  return cudaGetLastError();
}

cudaError_t launch_pq_keys(const uint8_t *codes, size_t n, int M, int ks, uint32_t *keys, uint32_t *vals,
                           cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  pq_keys_kernel<<<grid_for(n * M), 256, 0, s>>>(codes, n, M, ks, keys, vals);
  return cudaGetLastError();
}

cudaError_t launch_segments(const uint32_t *sorted_keys, size_t n, size_t nseg, uint32_t *seg, cudaStream_t s) {
  segments_kernel<<<grid_for(nseg + 1), 256, 0, s>>>(sorted_keys, n, nseg, seg);
  return cudaGetLastError();
}

namespace {
template <typename T>
__global__ void count_diff_kernel(const T *__restrict__ a, const T *__restrict__ b, size_t n,
                                  unsigned int *changed) {
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool diff = i < n && a[i] != b[i];
  unsigned int votes = __popc(__ballot_sync(VG_FULL_MASK, diff));
  if ((threadIdx.x & 31) == 0 && votes) atomicAdd(changed, votes);
}
}  // namespace

cudaError_t launch_count_diff_u8(const uint8_t *a, const uint8_t *b, size_t n, unsigned int *changed,
                                 cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_diff_kernel<uint8_t><<<grid_for(n), 256, 0, s>>>(a, b, n, changed);
  return cudaGetLastError();
}

cudaError_t launch_count_diff_u32(const uint32_t *a, const uint32_t *b, size_t n, unsigned int *changed,
                                  cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  count_diff_kernel<uint32_t><<<grid_for(n), 256, 0, s>>>(a, b, n, changed);
  return cudaGetLastError();
}

cudaError_t sort_pairs_u32(void *temp, size_t &temp_bytes, const uint32_t *kin, uint32_t *kout,
                           const uint32_t *vin, uint32_t *vout, size_t n, int end_bit, cudaStream_t s) {
  return cub::DeviceRadixSort::SortPairs(temp, temp_bytes, kin, kout, vin, vout, static_cast<int64_t>(n), 0,
                                         end_bit, s);
}

}  // namespace vg
