// Tensor-core products with a fused candidate window (tcgen05, sm_100a).
//
// Three reference computations are "the rows whose dot product with a query is
// among the P largest", with the reference's exact f32 arithmetic deciding:
//   find_nearest_centroids   src/ivf_pq/search.rs:1602-1617  (1 - q.c, P = nprobe)
//   KMeans::assign_clusters  src/partitioning/kmeans.rs:97-107 (argmin 1 - x.c, P = 1)
//   exact inner-product top-k src/distance.rs:125-130 with the exhaustive
//                             ground truth of src/benchmark/evaluation.rs:250-268
// The products are computed on the 5th-generation tensor cores in binary16 with
// f32 accumulation; nothing of the product matrix reaches memory.  Per 128-row
// block of queries the kernel sweeps the columns twice:
//   pass 0  every product goes into a per-row 256-bin histogram of 1 - s
//           (shared memory), or, for P = 1, a running maximum;
//   pass 1  the same products are recomputed and every column whose 1 - s lies
//           within the window (the histogram's bound on the P-th smallest, plus
//           twice the error bound) is appended to the row's candidate list.
// A finishing kernel (warp per row) takes the P-th smallest approximate
// distance over the candidates, re-scores every candidate within 2 eps of it
// with the reference's sequential f32 dot and keeps the exact top-P by (distance,
// column) key -- the same result as scoring every column exactly.  A row whose
// window overflows, or whose bound is not finite, is scored exactly over every
// column.
//
// Window kernel roles (one CTA per SM, persistent over work units):
//   warp 0      bulk copies (cp.async.bulk) of operand tiles into shared memory
//   warp 1      one thread issues tcgen05.mma into one of two TMEM accumulators
//   warps 2..5  read the accumulator (tcgen05.ld) and run the pass's epilogue
// Operands live in memory as "images": 128-row tiles of the binary16 rows, each
// tile holding Kp/64 blocks of 128 rows x 128 bytes in the 128-byte-swizzled
// K-major layout the tensor core reads, so one contiguous bulk copy stages a
// tile.  Every wait is bounded: a protocol error sets the error flag and the
// kernel drains its copies and MMAs, frees its TMEM and returns.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "kernels.h"
#include "pipeline.cuh"
#include "probe_bounds.cuh"
#include "topk.cuh"

namespace vg {

namespace {

constexpr int kTile = 128;                            // UMMA M (query rows) and N (columns) per tile
constexpr int kKBlock = 64;                           // binary16 elements per 128-byte swizzle row
constexpr uint32_t kBlockBytes = kTile * 128;         // one K-block of one tile: 16 KB
constexpr int kStages = 3;                            // column tiles in flight
constexpr int kBins = 256;                            // histogram bins of 1 - s over [0, 2)
constexpr int kWinThreads = 192;                      // 6 warps
constexpr uint32_t kTmemCols = 2 * kTile;             // two f32 accumulators of 128 columns
constexpr int kFinWarps = 8;
constexpr int kFinBuf = 512;                          // re-scored candidates per row (finisher)
constexpr uint32_t kMaxSplitCols = 511u * kTile;      // histogram counts are u16

// tcgen05.mma instruction descriptor, kind::f16: D f32, A and B binary16,
// both K-major, N = 128 (bits 17-22, N >> 3), M = 128 (bits 24-28, M >> 4).
constexpr uint32_t kIdesc = (1u << 4) | (static_cast<uint32_t>(kTile >> 3) << 17) |
                            (static_cast<uint32_t>(kTile >> 4) << 24);

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle:
// start address >> 4, leading offset 16 B (unused with this swizzle), 1024 B
// between 8-row groups, descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Arrive once on *bar when every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 32 consecutive f32 accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint16_t lds_u16(uint32_t a) {
  uint16_t x;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(x) : "r"(a));
  return x;
}
__device__ __forceinline__ void sts_u16(uint32_t a, uint16_t x) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(x) : "memory");
}

struct WinParams {
  const uint8_t *a_img, *b_img;  // operand images (tile = kp * 256 bytes)
  size_t rows, cols;
  int kp, P, top1;               // top1: running maximum instead of the histogram
  int splits;                    // column ranges per row block (work unit = row block x range)
  uint32_t split_cols;           // columns per range, a multiple of 128, <= kMaxSplitCols
  int cap;                       // candidates kept per (row, range)
  const float *eps;              // [rows] error bound of the approximate products
  uint2 *cand;                   // [rows][splits][cap] (column, bits of s)
  uint32_t *count;               // [rows][splits] candidates found (> cap: overflow)
  int *error;                    // set nonzero when a bounded wait gives up
};

__device__ __forceinline__ void win_fail(const WinParams &p, volatile int *abort_flag, int code) {
  *abort_flag = 1;
  if (p.error) *reinterpret_cast<volatile int *>(p.error) = code;
}

__global__ void __launch_bounds__(kWinThreads, 1) tc_window_kernel(const WinParams p) {
  extern __shared__ uint8_t win_raw[];
  const uint32_t raw = smem_u32(win_raw);
  uint8_t *sm = win_raw + (((raw + 1023u) & ~1023u) - raw);  // swizzled tiles need 1024-byte alignment
  const int nkb = p.kp / kKBlock;
  const uint32_t tile_bytes = static_cast<uint32_t>(nkb) * kBlockBytes;
  uint8_t *sA = sm;
  uint8_t *sB = sm + tile_bytes;
  uint16_t *hist = reinterpret_cast<uint16_t *>(sB + kStages * tile_bytes);  // [kBins][128 rows]
  uint64_t *bars = reinterpret_cast<uint64_t *>(hist + kBins * kTile);
  uint64_t *full = bars, *empty = bars + kStages, *afull = bars + 2 * kStages, *aempty = afull + 1;
  uint64_t *accfull = aempty + 1, *accempty = accfull + 2, *drain = accempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(afull, 1);
    mbar_init(aempty, 1);
    mbar_init(accfull, 1);
    mbar_init(accfull + 1, 1);
    mbar_init(accempty, 4);
    mbar_init(accempty + 1, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const size_t rblocks = (p.rows + kTile - 1) / kTile;
  const size_t units = rblocks * static_cast<size_t>(p.splits);
  auto unit_range = [&](size_t u, size_t &rb, int &sp, size_t &c0, uint32_t &ntiles) {
    rb = u / p.splits;
    sp = static_cast<int>(u - rb * p.splits);
    c0 = static_cast<size_t>(sp) * p.split_cols;
    const size_t c1 = min(p.cols, c0 + p.split_cols);
    ntiles = static_cast<uint32_t>((c1 - c0 + kTile - 1) / kTile);
  };

  if (warp == 0) {
    // ---- producer: A tile per unit, then the unit's column tiles twice ----
    if (lane == 0) {
      uint32_t it = 0, ul = 0;
      long long a_issued = -1;  // last unit whose A tile was issued
      int last_stage_it[kStages];
      for (int s = 0; s < kStages; ++s) last_stage_it[s] = -1;
      bool ok = true;
      for (size_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++ul) {
        size_t rb, c0;
        int sp;
        uint32_t ntiles;
        unit_range(u, rb, sp, c0, ntiles);
        if (*abort_flag || (ul > 0 && !mbar_wait(aempty, (ul - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(afull, tile_bytes);
        bulk_copy_g2s(sA, p.a_img + rb * tile_bytes, tile_bytes, afull);
        a_issued = ul;
        const size_t t0 = c0 / kTile;
        for (int pass = 0; ok && pass < 2; ++pass) {
          for (uint32_t t = 0; t < ntiles; ++t, ++it) {
            const uint32_t stage = it % kStages, ph = (it / kStages) & 1;
            if (*abort_flag || !mbar_wait(empty + stage, ph ^ 1)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(full + stage, tile_bytes);
            bulk_copy_g2s(sB + stage * tile_bytes, p.b_img + (t0 + t) * tile_bytes, tile_bytes, full + stage);
            last_stage_it[stage] = static_cast<int>(it);
          }
        }
      }
      if (!ok) {
        win_fail(p, abort_flag, 1);
        // copies still in flight land in shared memory: wait for them (bounded)
        for (int s = 0; s < kStages; ++s)
          if (last_stage_it[s] >= 0) mbar_wait(full + s, (static_cast<uint32_t>(last_stage_it[s]) / kStages) & 1);
        if (a_issued >= 0) mbar_wait(afull, static_cast<uint32_t>(a_issued) & 1);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      uint32_t it = 0, tc = 0, ul = 0;
      bool ok = true;
      for (size_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++ul) {
        size_t rb, c0;
        int sp;
        uint32_t ntiles;
        unit_range(u, rb, sp, c0, ntiles);
        if (!mbar_wait(afull, ul & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA);
        for (int pass = 0; ok && pass < 2; ++pass) {
          for (uint32_t t = 0; t < ntiles; ++t, ++it, ++tc) {
            const uint32_t stage = it % kStages, ph = (it / kStages) & 1;
            const uint32_t acc = tc & 1, aph = (tc >> 1) & 1;
            if (!mbar_wait(full + stage, ph) || !mbar_wait(accempty + acc, aph ^ 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b_base = smem_u32(sB + stage * tile_bytes);
            const uint32_t d_tmem = tmem + acc * kTile;
            for (int kb = 0; kb < nkb; ++kb) {
#pragma unroll
              for (int j = 0; j < kKBlock / 16; ++j) {
                const uint32_t off = static_cast<uint32_t>(kb) * kBlockBytes + static_cast<uint32_t>(j) * 32u;
                umma_f16(d_tmem, umma_desc(a_base + off), umma_desc(b_base + off), (kb | j) != 0);
              }
            }
            umma_commit(empty + stage);
            umma_commit(accfull + acc);
          }
        }
        if (ok) umma_commit(aempty);
      }
      if (!ok) win_fail(p, abort_flag, 2);
      // every MMA issued is complete before the accumulators are released
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 ----
    const int ew = warp & 3;
    const int rloc = ew * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(ew * 32) << 16);
    const uint32_t hbase = smem_u32(hist) + static_cast<uint32_t>(rloc) * 2u;
    uint32_t tc = 0;
    bool ok = true;
    for (size_t u = blockIdx.x; ok && u < units; u += gridDim.x) {
      size_t rb, c0;
      int sp;
      uint32_t ntiles;
      unit_range(u, rb, sp, c0, ntiles);
      const size_t row = rb * kTile + rloc;
      const bool rv = row < p.rows;
      const double eps = rv ? static_cast<double>(p.eps[row]) : 0.0;
      const size_t c1 = min(p.cols, c0 + p.split_cols);
      if (!p.top1)
        for (int b = 0; b < kBins; ++b) hist[b * kTile + rloc] = 0;
      float smax = -__int_as_float(0x7f800000);
      float s_lo = 0.0f;
      uint32_t n = 0;
      uint2 *cand = p.cand + (row * p.splits + sp) * static_cast<size_t>(p.cap);
      for (int pass = 0; ok && pass < 2; ++pass) {
        if (pass == 1) {
          // lower bound on s for 1 - s within 2 eps of the bound on the P-th smallest
          double lo = -__longlong_as_double(0x7ff0000000000000ll);
          if (p.top1) {
            if (smax > -__int_as_float(0x7f800000))
              lo = static_cast<double>(smax) - 2.0 * eps * (1.0 + 9.5367431640625e-7) -
                   9.5367431640625e-7 * (1.0 + fabs(static_cast<double>(smax)));
          } else {
            uint32_t cum = 0;
            int bstar = kBins - 1;
            for (int b = 0; b < kBins - 1; ++b) {
              cum += hist[b * kTile + rloc];
              if (cum >= static_cast<uint32_t>(p.P)) {
                bstar = b;
                break;
              }
            }
            // bin b holds 128 (1 - s) rounded to nearest: 1 - s <= (b + 0.5) / 128
            if (bstar < kBins - 1) {
              const double T = (bstar + 0.5) / 128.0;
              lo = 1.0 - (T + 2.0 * eps) * (1.0 + 9.5367431640625e-7) - 9.5367431640625e-7;
            }
          }
          s_lo = eps < 1.0 ? __double2float_rd(lo) : -__int_as_float(0x7f800000);
        }
        for (uint32_t t = 0; t < ntiles; ++t, ++tc) {
          const uint32_t acc = tc & 1, aph = (tc >> 1) & 1;
          if (!__all_sync(VG_FULL_MASK, mbar_wait(accfull + acc, aph))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const size_t col0 = c0 + static_cast<size_t>(t) * kTile;
          const int nval = static_cast<int>(min(static_cast<size_t>(kTile), c1 - col0));
#pragma unroll 1
          for (int ch = 0; ch < kTile / 32; ++ch) {
            if (ch * 32 >= nval) break;
            uint32_t v[32];
            tmem_ld32(t_lane + acc * kTile + ch * 32, v);
            const int lim = nval - ch * 32;
            if (pass == 0) {
              if (p.top1) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < lim) smax = fmaxf(smax, __uint_as_float(v[j]));
              } else {
                // 8 counts loaded, then 8 stored: two equal bins in one group
                // lose an increment, which only loosens the bound (a count
                // never exceeds the true one; u16 wrap-around likewise)
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                  uint32_t a[8];
                  uint16_t c[8];
#pragma unroll
                  for (int uu = 0; uu < 8; ++uu) {
                    const int j = g * 8 + uu;
                    const float tt = fmaf(__uint_as_float(v[j]), -128.0f, 8388736.0f);  // 2^23 + 128 (1 - s)
                    int b = static_cast<int>(__float_as_uint(tt)) - 0x4B000000;
                    b = min(max(b, 0), kBins - 1);
                    if (j >= lim) b = kBins - 1;
                    a[uu] = hbase + (static_cast<uint32_t>(b) << 8);
                  }
#pragma unroll
                  for (int uu = 0; uu < 8; ++uu) c[uu] = lds_u16(a[uu]);
#pragma unroll
                  for (int uu = 0; uu < 8; ++uu) sts_u16(a[uu], static_cast<uint16_t>(c[uu] + 1));
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j < lim && __uint_as_float(v[j]) >= s_lo) {
                  if (rv && n < static_cast<uint32_t>(p.cap))
                    cand[n] = make_uint2(static_cast<uint32_t>(col0 + ch * 32 + j), v[j]);
                  ++n;
                }
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(accempty + acc);
        }
      }
      if (rv && ok) p.count[row * p.splits + sp] = n;
    }
    if (!ok) win_fail(p, abort_flag, 3);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

size_t win_smem_bytes(int kp) {
  const size_t tile = static_cast<size_t>(kp / kKBlock) * kBlockBytes;
  return 1024 + tile * (1 + kStages) + static_cast<size_t>(kBins) * kTile * 2 + 16 * 8 + 16;
}

// ---- operand images ------------------------------------------------------

// Element (r, k) of a row-major binary16 matrix in the image: tile r / 128,
// K-block k / 64, 8-row group, row in group, 16-byte chunk XOR row (mod 8).
__host__ __device__ inline size_t image_chunk(size_t r, int chunk, int kp) {
  const size_t t = r / kTile;
  const uint32_t rr = static_cast<uint32_t>(r % kTile);
  const uint32_t kb = static_cast<uint32_t>(chunk) >> 3, c = static_cast<uint32_t>(chunk) & 7u;
  const size_t byte = t * static_cast<size_t>(kTile) * kp * 2 + kb * kBlockBytes + (rr >> 3) * 1024u +
                      (rr & 7u) * 128u + ((c ^ (rr & 7u)) << 4);
  return byte >> 4;  // in 16-byte units
}

// One thread per 16-byte chunk (8 elements); the kp / 8 threads of a row
// reduce its squared norm for the error bound when eps is set.
__global__ void umma_image_kernel(const float *__restrict__ x, size_t rows, size_t rows_img, int d, int kp,
                                  uint4 *__restrict__ img, const float *__restrict__ cmax_p, double rel,
                                  double abs_coef, float *__restrict__ eps) {
  const int tpr = kp >> 3;
  const size_t gid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t r = gid / tpr;
  const int j = static_cast<int>(gid % tpr);
  if (r >= rows_img) return;  // whole rows exit together (rows_img * tpr is a multiple of the block)
  float v[8];
  double ss = 0.0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int k = j * 8 + e;
    v[e] = (r < rows && k < d) ? x[r * d + k] : 0.0f;
    ss += static_cast<double>(v[e]) * v[e];
  }
  uint4 o;
  __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
  __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
  o.x = *reinterpret_cast<uint32_t *>(&h0);
  o.y = *reinterpret_cast<uint32_t *>(&h1);
  o.z = *reinterpret_cast<uint32_t *>(&h2);
  o.w = *reinterpret_cast<uint32_t *>(&h3);
  img[image_chunk(r, j, kp)] = o;
  if (eps) {
    for (int off = tpr >> 1; off > 0; off >>= 1) ss += __shfl_xor_sync(VG_FULL_MASK, ss, off, tpr);
    if (j == 0 && r < rows) {
      const double cmax = static_cast<double>(*cmax_p), xn = sqrt(ss);
      const double e = rel * xn * cmax * 1.01 + abs_coef * (1.0 + xn + cmax) + 1.0 / 1048576;
      // a row this long may hold entries past the binary16 range: exact path
      eps[r] = xn < 16384.0 ? __double2float_ru(e) : __int_as_float(0x7f800000);
    }
  }
}

// ---- finisher ------------------------------------------------------------

struct FinParams {
  const uint2 *cand;
  const uint32_t *count;
  int splits, cap;
  const float *eps;
  const float *q;  // [rows][d] f32 query rows
  const float *x;  // [cols][d] f32 column rows
  size_t rows, cols;
  int d, P, mode;  // mode 0: 1 - dot (probes), 1: -dot (inner-product search)
  uint32_t *out_ids;
  float *out_dist;
  size_t out_ld;
  uint32_t *out_count;  // nullable
  ProbeBoundArgs bnd;   // probes only (bnd.lb nullable)
};

template <int R>
__global__ void __launch_bounds__(kFinWarps * 32) tc_finish_kernel(const FinParams p) {
  extern __shared__ __align__(16) unsigned char fin_sm[];
  const int lane = lane_id(), warp = threadIdx.x >> 5;
  const size_t row = static_cast<size_t>(blockIdx.x) * kFinWarps + warp;
  if (row >= p.rows) return;
  const int d = p.d, dpad = (d + 3) & ~3;
  float *qs = reinterpret_cast<float *>(fin_sm) + static_cast<size_t>(warp) * dpad;
  uint32_t *buf = reinterpret_cast<uint32_t *>(reinterpret_cast<float *>(fin_sm) + kFinWarps * dpad) +
                  static_cast<size_t>(warp) * kFinBuf;
  const float *qrow = p.q + row * d;
  for (int j = lane; j < d; j += 32) qs[j] = qrow[j];
  __syncwarp();
  const float eps = p.eps[row];
  bool exact_all = !(eps < 1.0f);  // non-finite or useless bound
  const bool cvec = (d & 3) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
  const uint2 *crow = p.cand + row * p.splits * static_cast<size_t>(p.cap);
  const uint32_t *cnt = p.count + row * p.splits;
  for (int s = 0; s < p.splits; ++s)
    if (cnt[s] > static_cast<uint32_t>(p.cap)) exact_all = true;
  const float kInf = __int_as_float(0x7f800000);
  int n = 0;
  if (!exact_all) {
    // the P-th smallest approximate distance over the candidates (which hold
    // every column of the P smallest), then every candidate within 2 eps of it
    WarpTopK<R> tk;
    tk.init();
    for (int s = 0; s < p.splits; ++s) {
      const uint2 *seg = crow + static_cast<size_t>(s) * p.cap;
      const int c = static_cast<int>(cnt[s]);
      for (int i0 = 0; i0 < c; i0 += 32) {
        const int i = i0 + lane;
        uint64_t key = kEmptyKey;
        if (i < c) {
          const uint2 e = seg[i];
          key = pack_key(__fsub_rn(1.0f, __uint_as_float(e.y)), e.x);
        }
        tk.add(key);
      }
    }
    const uint64_t ub = tk.get(p.P - 1);
    const float limit = ub == kEmptyKey ? kInf : __double2float_ru(static_cast<double>(key_dist(ub)) + 2.0 * eps);
    if (ub != kEmptyKey && !(limit < kInf)) exact_all = true;
    for (int s = 0; !exact_all && s < p.splits; ++s) {
      const uint2 *seg = crow + static_cast<size_t>(s) * p.cap;
      const int c = static_cast<int>(cnt[s]);
      for (int i0 = 0; i0 < c; i0 += 32) {
        const int i = i0 + lane;
        uint2 e = make_uint2(0u, 0u);
        bool t = false;
        if (i < c) {
          e = seg[i];
          t = !(__fsub_rn(1.0f, __uint_as_float(e.y)) > limit);
        }
        const unsigned m = __ballot_sync(VG_FULL_MASK, t);
        const int pos = n + __popc(m & ((1u << lane) - 1u));
        if (t && pos < kFinBuf) buf[pos] = e.x;
        n += __popc(m);
      }
    }
    if (n > kFinBuf) exact_all = true;
  }
  __syncwarp();
  auto dist_of = [&](uint32_t c) {
    const float dt = exact_dot(qs, p.x + static_cast<size_t>(c) * d, d, cvec);
    return p.mode == 0 ? __fsub_rn(1.0f, dt) : -dt;
  };
  WarpTopK<R> tk;
  tk.init();
  if (!exact_all) {
    for (int i0 = 0; i0 < n; i0 += 32) {
      uint64_t key = kEmptyKey;
      if (i0 + lane < n) {
        const uint32_t c = buf[i0 + lane];
        key = pack_key(dist_of(c), c);
      }
      tk.add(key);
    }
  } else {
    for (size_t c0 = 0; c0 < p.cols; c0 += 32) {
      const size_t c = c0 + lane;
      tk.add(c < p.cols ? pack_key(dist_of(static_cast<uint32_t>(c)), static_cast<uint32_t>(c)) : kEmptyKey);
    }
  }
  uint32_t real_count = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    const uint64_t key = tk.v[r];
    const bool real = i < p.P && key != kEmptyKey;
    real_count += __popc(__ballot_sync(VG_FULL_MASK, real));
    if (i < p.P) {
      const size_t o = row * p.out_ld + i;
      p.out_ids[o] = real ? key_id(key) : 0xffffffffu;
      p.out_dist[o] = real ? key_dist(key) : kInf;
      if (p.bnd.lb) write_probe_bound(qs, p.x, d, cvec, key_id(key), real, o, p.bnd);
    }
  }
  if (p.out_count && lane == 0) p.out_count[row] = real_count;
}

template <int R>
cudaError_t launch_finish(const FinParams &fp, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(kFinWarps) * (static_cast<size_t>((fp.d + 3) & ~3) * 4 + kFinBuf * 4);
  cudaError_t e = cudaFuncSetAttribute(tc_finish_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>((fp.rows + kFinWarps - 1) / kFinWarps);
  tc_finish_kernel<R><<<grid, kFinWarps * 32, smem, s>>>(fp);
  return cudaGetLastError();
}

}  // namespace

void tc_error_coefs(int d, double *rel, double *abs_coef) {
  const double u = 1.0 / 16777216.0, dd = static_cast<double>(d);
  // 2^-10 + 4u: rounding of both operands to binary16 (and its product term);
  // 2u: the subtractions from 1; 17 d u: accumulation in the tensor core
  // (16 u per add, any order) and the exact sequential dot (u per add)
  *rel = 16384.0 * u + 4.0 * u + 2.0 * u + 17.0 * dd * u;
  // subnormal binary16 operands: each off by at most 2^-25
  *abs_coef = std::sqrt(dd) * u;
}

int umma_kp(int d) { return d <= 0 ? 0 : d <= 64 ? 64 : d <= 128 ? 128 : 0; }

size_t umma_image_bytes(size_t rows, int kp) {
  return (rows + kTile - 1) / kTile * static_cast<size_t>(kTile) * kp * 2;
}

cudaError_t launch_umma_image(const float *x, size_t rows, int d, int kp, void *img, const float *cmax, double rel,
                              double abs_coef, float *eps, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (kp != 64 && kp != 128) return cudaErrorInvalidValue;
  const size_t rows_img = (rows + kTile - 1) / kTile * kTile;
  const size_t threads = rows_img * (kp >> 3);
  umma_image_kernel<<<static_cast<unsigned>(threads / 256), 256, 0, s>>>(
      x, rows, rows_img, d, kp, static_cast<uint4 *>(img), cmax, rel, abs_coef, eps);
  return cudaGetLastError();
}

void tc_select_plan(size_t rows, size_t cols, int P, int num_sms, int *splits, uint32_t *split_cols, int *cap) {
  const size_t rblocks = (rows + kTile - 1) / kTile;
  size_t sp = (cols + kMaxSplitCols - 1) / kMaxSplitCols;
  // few row blocks: more column ranges keep every SM busy, as long as each
  // range stays wide enough for a tight bound on its P-th product
  const size_t bal = rblocks ? static_cast<size_t>(num_sms) / rblocks : 1;
  const size_t wide = std::max<size_t>(1, cols / 8192);
  sp = std::max(sp, std::min(bal, wide));
  if (sp < 1) sp = 1;
  size_t per = (cols + sp - 1) / sp;
  per = (per + kTile - 1) / kTile * kTile;
  if (per == 0) per = kTile;
  sp = (cols + per - 1) / per;
  if (sp < 1) sp = 1;
  *splits = static_cast<int>(sp);
  *split_cols = static_cast<uint32_t>(per);
  *cap = P == 1 ? 32 : std::min(1024, (2 * P + 64 + 31) / 32 * 32);
}

size_t tc_select_workspace_bytes(size_t rows, size_t cols, int P, int num_sms) {
  int sp, cap;
  uint32_t per;
  tc_select_plan(rows, cols, P, num_sms, &sp, &per, &cap);
  return rows * sp * (static_cast<size_t>(cap) * 8 + 4) + 256;
}

cudaError_t launch_tc_select(const TcSelect &t, int num_sms, cudaStream_t s) {
  if (t.rows == 0 || t.P <= 0) return cudaSuccess;
  if (t.P > 256 || (t.kp != 64 && t.kp != 128) || t.cols == 0 || t.cols > 0xfffffffeull) return cudaErrorInvalidValue;
  int sp, cap;
  uint32_t per;
  tc_select_plan(t.rows, t.cols, t.P, num_sms, &sp, &per, &cap);
  uint2 *cand = static_cast<uint2 *>(t.workspace);
  uint32_t *count = reinterpret_cast<uint32_t *>(cand + t.rows * sp * static_cast<size_t>(cap));
  WinParams wp{};
  wp.a_img = static_cast<const uint8_t *>(t.a_img);
  wp.b_img = static_cast<const uint8_t *>(t.b_img);
  wp.rows = t.rows;
  wp.cols = t.cols;
  wp.kp = t.kp;
  wp.P = t.P;
  wp.top1 = t.P == 1;
  wp.splits = sp;
  wp.split_cols = per;
  wp.cap = cap;
  wp.eps = t.eps;
  wp.cand = cand;
  wp.count = count;
  wp.error = t.error;
  const size_t smem = win_smem_bytes(t.kp);
  cudaError_t e = cudaFuncSetAttribute(tc_window_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const size_t units = (t.rows + kTile - 1) / kTile * static_cast<size_t>(sp);
  const unsigned grid = static_cast<unsigned>(std::min<size_t>(units, static_cast<size_t>(num_sms)));
  if (t.marks[0]) cudaEventRecord(t.marks[0], s);
  tc_window_kernel<<<grid, kWinThreads, smem, s>>>(wp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (t.marks[1]) cudaEventRecord(t.marks[1], s);
  FinParams fp{};
  fp.cand = cand;
  fp.count = count;
  fp.splits = sp;
  fp.cap = cap;
  fp.eps = t.eps;
  fp.q = t.q;
  fp.x = t.x;
  fp.rows = t.rows;
  fp.cols = t.cols;
  fp.d = t.d;
  fp.P = t.P;
  fp.mode = t.mode;
  fp.out_ids = t.out_ids;
  fp.out_dist = t.out_dist;
  fp.out_ld = t.out_ld;
  fp.out_count = t.out_count;
  fp.bnd = t.bnd;
  e = t.P <= 32 ? launch_finish<1>(fp, s) : t.P <= 64 ? launch_finish<2>(fp, s)
      : t.P <= 128 ? launch_finish<4>(fp, s) : launch_finish<8>(fp, s);
  if (e == cudaSuccess && t.marks[2]) cudaEventRecord(t.marks[2], s);
  return e;
}

}  // namespace vg
