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
constexpr int kStages = 2;                            // column tiles in flight
constexpr int kBins = 256;                            // histogram bins of 1 - s over [0, 2)
constexpr uint32_t kWarmTiles = 4;                    // tiles of a unit counted before any is gathered
constexpr int kEpiWarps = 8;                          // two epilogue warpgroups, one per accumulator
constexpr int kWinThreads = 64 + kEpiWarps * 32;      // copies, MMA, epilogue
constexpr uint32_t kTmemCols = 2 * kTile;             // two f32 accumulators of 128 columns
constexpr int kFinWarps = 8;
constexpr int kFinBuf = 512;                          // re-scored candidates per row (finisher)

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

struct WinParams {
  const uint8_t *a_img, *b_img;  // operand images (tile = kp * 256 bytes)
  size_t rows, cols;
  int kp, ksteps, P, top1;       // ksteps: MMA K-steps of 16 covering d; top1: running maximum
  int splits;                    // column ranges per row block (work unit = row block x range)
  uint32_t split_cols;           // columns per range, a multiple of 128
  int cap;                       // candidates kept per (row, range, warpgroup)
  const float *eps;              // [rows] error bound of the approximate products
  uint2 *cand;                   // [rows][splits][2][cap] (column, bits of s)
  uint32_t *count;               // [rows][splits][2] candidates found (> cap: overflow)
  uint32_t *gbound;              // [rows] bound shared by every CTA of a row (zeroed before launch)
  int *error;                    // set nonzero when a bounded wait gives up
};

__device__ __forceinline__ void win_fail(const WinParams &p, volatile int *abort_flag, int code) {
  *abort_flag = 1;
  if (p.error) *reinterpret_cast<volatile int *>(p.error) = code;
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t *v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t x;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x) : "r"(a) : "memory");
  return x;
}

// largest of 32 values (tree, no NaN propagation)
__device__ __forceinline__ float max32(const uint32_t *v) {
  float m[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = fmaxf(__uint_as_float(v[i]), __uint_as_float(v[i + 16]));
#pragma unroll
  for (int w = 8; w > 0; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) m[i] = fmaxf(m[i], m[i + w]);
  return m[0];
}

// predicated helpers: no branch per value
__device__ __forceinline__ void red_add_if(bool p, uint32_t addr) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %1, 0;\n\t@q red.shared.add.u32 [%0], 1;\n\t}" ::"r"(addr),
      "r"(static_cast<uint32_t>(p))
      : "memory");
}
__device__ __forceinline__ void st_cand_if(bool p, uint2 *dst, uint32_t col, uint32_t bits) {
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %3, 0;\n\t@q st.global.v2.u32 [%0], {%1, %2};\n\t}" ::"l"(dst),
      "r"(col), "r"(bits), "r"(static_cast<uint32_t>(p))
      : "memory");
}

// Window of one row (thread), a single sweep of the row's columns.  Per tile
// of products (in registers):
//   1. count: histogram mode -- hist[b][row] counts the row's products with
//      bin b = round(128 (1 - s)) clamped to [0, 255] (shared by the row's two
//      epilogue threads, red.shared.add).  h is a bin bound: every value with
//      bin < h is counted exactly, so once the counts below h reach P the P-th
//      smallest 1 - s of the row lies at or below (h - 0.5) / 128; values with
//      bin >= h are skipped (those bins may be undercounted, which only delays
//      the bound).  Top-1 mode -- a running maximum of s.
//   2. refresh the bound (histogram mode: on a schedule): from the exact bins
//      below h, and from the other column ranges of the row through
//      gbound[row] (256 - h, atomicMax; a bound on the P-th smallest of any
//      subset of the row's columns bounds the whole row's).
//   3. gather: every column of the tile with 1 - s within twice the error
//      bound of the current bound is appended to the row's candidates.  The
//      bound only tightens, so every column of the final window has been
//      appended; when the list fills up, candidates below the current window
//      are dropped (compaction).  A list that still overflows marks the row
//      for the exact re-score of every column.
__global__ void __launch_bounds__(kWinThreads, 1) tc_window_kernel(const WinParams p) {
  extern __shared__ uint8_t win_raw[];
  const uint32_t raw = smem_u32(win_raw);
  uint8_t *sm = win_raw + (((raw + 1023u) & ~1023u) - raw);  // swizzled tiles need 1024-byte alignment
  const int nkb = p.kp / kKBlock;
  const uint32_t tile_bytes = static_cast<uint32_t>(nkb) * kBlockBytes;
  uint8_t *sA = sm;
  uint8_t *sB = sm + tile_bytes;
  uint32_t *hist = reinterpret_cast<uint32_t *>(sB + kStages * tile_bytes);  // [kBins][128 rows]
  uint32_t *lowbin = hist + kBins * kTile;  // [128 rows] lowest bin counted in the unit
  uint64_t *bars = reinterpret_cast<uint64_t *>(lowbin + kTile);
  uint64_t *full = bars, *empty = bars + kStages, *afull = bars + 2 * kStages, *aempty = afull + 1;
  uint64_t *accfull = aempty + 1, *accempty = accfull + 2, *drain = accempty + 2, *hzero = drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(hzero + 1);
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
    mbar_init(hzero, kEpiWarps * 32);
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

  // work units range-major: CTAs running at the same time mostly stream the
  // same column range (its tiles shared in L2) for different row blocks
  const size_t rblocks = (p.rows + kTile - 1) / kTile;
  const size_t units = rblocks * static_cast<size_t>(p.splits);
  auto unit_range = [&](size_t u, size_t &rb, int &sp, size_t &c0, uint32_t &ntiles) {
    sp = static_cast<int>(u / rblocks);
    rb = u - static_cast<size_t>(sp) * rblocks;
    c0 = static_cast<size_t>(sp) * p.split_cols;
    const size_t c1 = min(p.cols, c0 + p.split_cols);
    ntiles = static_cast<uint32_t>((c1 - c0 + kTile - 1) / kTile);
  };

  if (warp == 0) {
    // ---- producer: A tile per unit, then the unit's column tiles ----
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
        if (*abort_flag || (ul > 0 && !mbar_wait_sleep(aempty, (ul - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(afull, tile_bytes);
        bulk_copy_g2s(sA, p.a_img + rb * tile_bytes, tile_bytes, afull);
        a_issued = ul;
        const size_t t0 = c0 / kTile;
        const uint32_t nvisit = ntiles + min(ntiles, kWarmTiles);
        for (uint32_t i = 0; i < nvisit; ++i, ++it) {
          const uint32_t t = i < ntiles ? i : i - ntiles;
          const uint32_t stage = it % kStages, ph = (it / kStages) & 1;
          if (*abort_flag || !mbar_wait_sleep(empty + stage, ph ^ 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + stage, tile_bytes);
          bulk_copy_g2s(sB + stage * tile_bytes, p.b_img + (t0 + t) * tile_bytes, tile_bytes, full + stage);
          last_stage_it[stage] = static_cast<int>(it);
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
        if (!mbar_wait_sleep(afull, ul & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA);
        const uint32_t nvisit = ntiles + min(ntiles, kWarmTiles);
        for (uint32_t i = 0; i < nvisit; ++i, ++it, ++tc) {
          const uint32_t stage = it % kStages, ph = (it / kStages) & 1;
          const uint32_t acc = tc & 1, aph = (tc >> 1) & 1;
          if (!mbar_wait_sleep(full + stage, ph) || !mbar_wait_sleep(accempty + acc, aph ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_base = smem_u32(sB + stage * tile_bytes);
          const uint32_t d_tmem = tmem + acc * kTile;
          for (int ks = 0; ks < p.ksteps; ++ks) {
            const uint32_t off = static_cast<uint32_t>(ks >> 2) * kBlockBytes + static_cast<uint32_t>(ks & 3) * 32u;
            umma_f16(d_tmem, umma_desc(a_base + off), umma_desc(b_base + off), ks != 0);
          }
          umma_commit(empty + stage);
          umma_commit(accfull + acc);
        }
        if (ok) umma_commit(aempty);
      }
      if (!ok) win_fail(p, abort_flag, 2);
      // every MMA issued is complete before the accumulators are released
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else {
    // ---- epilogue: warpgroup eg reads accumulator eg (the tiles with tile
    // counter parity eg); warp w reads TMEM lanes 32 (w % 4) .. + 31 ----
    const int eg = (warp - 2) >> 2;
    const int ew = warp & 3;
    const int rloc = ew * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(eg) * kTile;
    const uint32_t hbase = smem_u32(hist) + static_cast<uint32_t>(rloc) * 4u;
    const uint32_t lbase = smem_u32(lowbin) + static_cast<uint32_t>(rloc) * 4u;
    const float kInf = __int_as_float(0x7f800000);
    const uint32_t cap = static_cast<uint32_t>(p.cap);
    uint32_t tc = 0, ul = 0;
    bool ok = true;
    for (size_t u = blockIdx.x; ok && u < units; u += gridDim.x, ++ul) {
      size_t rb, c0;
      int sp;
      uint32_t ntiles;
      unit_range(u, rb, sp, c0, ntiles);
      const size_t row = rb * kTile + rloc;
      const bool rv = row < p.rows;
      const double eps = rv ? static_cast<double>(p.eps[row]) : 0.0;
      const bool bounded = rv && eps < 1.0;  // otherwise the finisher scores the row exactly
      const size_t c1 = min(p.cols, c0 + p.split_cols);
      uint32_t *gb = p.gbound + (rv ? row : 0);
      if (!p.top1) {
        // zero this row's bins (each warpgroup half of them); every epilogue
        // thread arrives, and counting starts once the phase completes
        for (int b = eg * (kBins / 2); b < (eg + 1) * (kBins / 2); ++b) hist[b * kTile + rloc] = 0;
        if (eg == 0) lowbin[rloc] = kBins;
        mbar_arrive(hzero);
        if (!__all_sync(VG_FULL_MASK, mbar_wait_sleep(hzero, ul & 1))) {
          ok = false;
          break;
        }
      }
      uint32_t h = kBins;  // bin bound (kBins: none yet)
      uint32_t gseen = 0;  // largest gbound value seen
      float s_h = -kInf;   // values with s > s_h are counted (1 - h / 128)
      float smax = -kInf;  // top-1 mode: running maximum
      float s_lo = -kInf;  // values with s >= s_lo are gathered
      uint32_t n = 0, tp = 0;
      bool over = false;
      uint2 *cand = p.cand + ((row * p.splits + sp) * 2 + eg) * static_cast<size_t>(p.cap);

      // s_lo of a bound T on the P-th smallest 1 - s: 1 - s <= T + 2 eps
      auto set_window = [&](double T) {
        const double lo = 1.0 - (T + 2.0 * eps) * (1.0 + 9.5367431640625e-7) - 9.5367431640625e-7;
        s_lo = bounded ? __double2float_rd(lo) : -kInf;
      };
      // refresh h from the exact bins below it and from the other ranges
      auto refresh = [&]() {
        uint32_t cum = 0, found = h;
        // bins below the lowest one counted are empty
        for (uint32_t b0 = min(lds_u32(lbase), static_cast<uint32_t>(kBins)) & ~7u; b0 < found; b0 += 8) {
          uint32_t c[8];
#pragma unroll
          for (int uu = 0; uu < 8; ++uu) c[uu] = lds_u32(hbase + ((b0 + uu) << 9));
#pragma unroll
          for (int uu = 0; uu < 8; ++uu) {
            if (b0 + uu < found) {
              cum += c[uu];
              if (cum >= static_cast<uint32_t>(p.P)) found = b0 + uu + 1;
            }
          }
        }
        h = found;
        if (rv) {
          const uint32_t mine = kBins - h;
          if (mine > gseen) atomicMax(gb, mine);
          gseen = max(gseen, max(mine, *reinterpret_cast<volatile uint32_t *>(gb)));
        }
        h = min(h, kBins - gseen);
        s_h = 1.0f - static_cast<float>(h) * (1.0f / 128.0f);
        // bin b holds 128 (1 - s) rounded to nearest: 1 - s <= (b + 0.5) / 128
        if (h < kBins) set_window((h - 0.5) / 128.0);
      };
      // drop candidates below the current window (16 loads in flight)
      auto compact = [&]() {
        const uint32_t m = min(n, cap);
        uint32_t k = 0;
        for (uint32_t i0 = 0; i0 < m; i0 += 16) {
          uint2 e[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) e[j] = i0 + j < m ? cand[i0 + j] : make_uint2(0u, 0x7fc00000u);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const bool keep = __uint_as_float(e[j].y) >= s_lo;
            st_cand_if(keep, cand + k, e[j].x, e[j].y);
            k += keep ? 1u : 0u;
          }
        }
        n = k;
      };

      // The first kWarmTiles tiles are only counted; the sweep then visits
      // them again at its end and gathers them with the final bound.
      const uint32_t warm = min(ntiles, kWarmTiles);
      for (uint32_t i = 0; i < ntiles + warm; ++i, ++tc) {
        const bool revisit = i >= ntiles;
        const uint32_t t = revisit ? i - ntiles : i;
        const uint32_t acc = tc & 1;
        if (acc != static_cast<uint32_t>(eg)) continue;  // the other warpgroup's tile
        const uint32_t aph = (tc >> 1) & 1;
        if (!__all_sync(VG_FULL_MASK, mbar_wait_sleep(accfull + acc, aph))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const size_t col0 = c0 + static_cast<size_t>(t) * kTile;
        const int nval = static_cast<int>(min(static_cast<size_t>(kTile), c1 - col0));
        uint32_t v[kTile];
#pragma unroll
        for (int ch = 0; ch < kTile / 32; ++ch) tmem_ld32_nowait(t_lane + ch * 32, v + ch * 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accempty + acc);  // the values are in registers
        if (nval < kTile) {
#pragma unroll
          for (int j = 0; j < kTile; ++j)
            if (j >= nval) v[j] = 0x7fc00000u;  // NaN: fails every comparison, ignored by fmaxf
        }
        float cmax[kTile / 32];
#pragma unroll
        for (int ch = 0; ch < kTile / 32; ++ch) cmax[ch] = max32(v + ch * 32);
        // 1. count
        if (revisit) {
        } else if (p.top1) {
#pragma unroll
          for (int ch = 0; ch < kTile / 32; ++ch) smax = fmaxf(smax, cmax[ch]);
        } else {
#pragma unroll
          for (int ch = 0; ch < kTile / 32; ++ch) {
            if (cmax[ch] > s_h) {
              uint32_t bmin = kBins;
              const uint32_t *w = v + ch * 32;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float sv = __uint_as_float(w[j]);
                const float tt = fmaf(sv, -128.0f, 8388736.0f);  // 2^23 + 128 (1 - s), rounded
                int b = static_cast<int>(__float_as_uint(tt)) - 0x4B000000;
                b = min(max(b, 0), kBins - 1);
                red_add_if(sv > s_h, hbase + (static_cast<uint32_t>(b) << 9));
                bmin = (sv > s_h) ? min(bmin, static_cast<uint32_t>(b)) : bmin;
              }
              asm volatile("red.shared.min.u32 [%0], %1;" ::"r"(lbase), "r"(bmin) : "memory");
            }
          }
        }
        // 2. refresh the bound
        ++tp;
        if (revisit) {
        } else if (p.top1) {
          if (rv && smax > -kInf) {
            const uint32_t key = order_key(smax);
            if (key > gseen) atomicMax(gb, key);
            gseen = max(gseen, max(key, *reinterpret_cast<volatile uint32_t *>(gb)));
            smax = fmaxf(smax, key_to_float(gseen));
            const double lo = static_cast<double>(smax) - 2.0 * eps * (1.0 + 9.5367431640625e-7) -
                              9.5367431640625e-7 * (1.0 + fabs(static_cast<double>(smax)));
            s_lo = bounded ? __double2float_rd(lo) : -kInf;
          }
        } else if (t + 1 >= warm && ((tp & 1) == 0 || t + 2 >= ntiles || t + 1 == warm)) {
          refresh();
        }
        // 3. gather
        if (bounded && (revisit || t >= warm)) {
#pragma unroll
          for (int ch = 0; ch < kTile / 32; ++ch) {
            if (cmax[ch] >= s_lo) {
              if (n + 32 > cap && !over) {
                compact();
                // a window this wide is scored exactly by the finisher
                if (n > cap / 2) over = true;
              }
              const uint32_t *w = v + ch * 32;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const bool g = __uint_as_float(w[j]) >= s_lo;
                st_cand_if(g && !over, cand + n, static_cast<uint32_t>(col0 + ch * 32 + j), w[j]);
                n += (g && !over) ? 1u : 0u;
              }
            }
          }
        }
      }
      if (rv && ok) p.count[(row * p.splits + sp) * 2 + eg] = over ? cap + 1 : n;
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
  return 1024 + tile * (1 + kStages) + static_cast<size_t>(kBins) * kTile * 4 + kTile * 4 + 16 * 8 + 16;
}

// ---- tensor-core products to memory --------------------------------------

// out[r][c] = binary16(q_r . x_c) for every row and column, rounded to
// nearest from the f32 accumulator: the product matrix the probe shortlist
// (shortlist.cu) ranks.  The same staged-operand pipeline as the window
// kernel (warp 0 bulk copies, warp 1 issues tcgen05.mma into four TMEM
// accumulators, all 512 columns); four epilogue warpgroups, one per
// accumulator, convert theirs 64 columns at a time and store each row's
// products of the tile as whole 128-byte lines.
constexpr int kGemmStages = 4;
constexpr int kGemmAcc = 4;                              // TMEM accumulators (and epilogue warpgroups)
constexpr int kGemmEpiWarps = 4 * kGemmAcc;
constexpr int kGemmThreads = 64 + kGemmEpiWarps * 32;    // copies, MMA, epilogue
constexpr uint32_t kGemmTmemCols = kGemmAcc * kTile;     // 512: the whole TMEM

struct GemmParams {
  const uint8_t *a_img, *b_img;
  size_t rows, cols, ld;
  int kp, ksteps;
  __half *out;    // [rows][ld] binary16 products (nullable: not stored)
  __half *cmax;   // [rows][cstride] largest product of every 32-column chunk (nullable)
  size_t cstride;
  // gather mode (slo set): every column whose f32 product reaches slo[row]
  // is appended to the row's candidates (column + col_base, bits of the
  // product); count[row] may exceed cap, which marks an overflow
  const float *slo;
  uint2 *cand;
  uint32_t *count;
  uint32_t cap, col_base;
  int *error;
};

template <bool kGather>
__global__ void __launch_bounds__(kGemmThreads, 1) tc_gemm_f16_kernel(const GemmParams p) {
  extern __shared__ uint8_t gemm_raw[];
  const uint32_t raw = smem_u32(gemm_raw);
  uint8_t *sm = gemm_raw + (((raw + 1023u) & ~1023u) - raw);
  const int nkb = p.kp / kKBlock;
  const uint32_t tile_bytes = static_cast<uint32_t>(nkb) * kBlockBytes;
  uint8_t *sA = sm;
  uint8_t *sB = sm + tile_bytes;
  uint4 *stage_out = reinterpret_cast<uint4 *>(sB + kGemmStages * tile_bytes);  // [16 warps][32 rows][4 chunks]
  uint64_t *bars = reinterpret_cast<uint64_t *>(stage_out + kGemmEpiWarps * 32 * 4);
  uint64_t *full = bars, *empty = bars + kGemmStages, *afull = bars + 2 * kGemmStages, *aempty = afull + 1;
  uint64_t *accfull = aempty + 1, *accempty = accfull + kGemmAcc, *drain = accempty + kGemmAcc;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(afull, 1);
    mbar_init(aempty, 1);
    for (int a = 0; a < kGemmAcc; ++a) {
      mbar_init(accfull + a, 1);
      mbar_init(accempty + a, 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kGemmTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const size_t rblocks = (p.rows + kTile - 1) / kTile;
  // this CTA's tiles: an equal share of the (row block, column tile) order,
  // in segments of one row block each (the query tile reloads per segment)
  const size_t ctiles = (p.cols + kTile - 1) / kTile, all_tiles = rblocks * ctiles;
  const size_t t_begin = all_tiles * blockIdx.x / gridDim.x, t_end = all_tiles * (blockIdx.x + 1) / gridDim.x;
  const size_t rb_first = t_begin / ctiles;
  const size_t units = t_end > t_begin ? (t_end - 1) / ctiles - rb_first + 1 : 0;  // segments
  auto unit_range = [&](size_t u, size_t &rb, size_t &c0, uint32_t &ntiles) {
    rb = rb_first + u;
    const size_t a = max(t_begin, rb * ctiles) - rb * ctiles, b = min(t_end, (rb + 1) * ctiles) - rb * ctiles;
    c0 = a * kTile;
    ntiles = static_cast<uint32_t>(b - a);
  };
  auto fail = [&](int code) {
    *abort_flag = 1;
    if (p.error) *reinterpret_cast<volatile int *>(p.error) = code;
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0, ul = 0;
      long long a_issued = -1;
      int last_stage_it[kGemmStages];
      for (int s = 0; s < kGemmStages; ++s) last_stage_it[s] = -1;
      bool ok = true;
      for (size_t u = 0; ok && u < units; ++u, ++ul) {
        size_t rb, c0;
        uint32_t ntiles;
        unit_range(u, rb, c0, ntiles);
        if (*abort_flag || (ul > 0 && !mbar_wait_sleep(aempty, (ul - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(afull, tile_bytes);
        bulk_copy_g2s(sA, p.a_img + rb * tile_bytes, tile_bytes, afull);
        a_issued = ul;
        for (uint32_t t = 0; t < ntiles; ++t, ++it) {
          const uint32_t stage = it % kGemmStages, ph = (it / kGemmStages) & 1;
          if (*abort_flag || !mbar_wait_sleep(empty + stage, ph ^ 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + stage, tile_bytes);
          bulk_copy_g2s(sB + stage * tile_bytes, p.b_img + (c0 / kTile + t) * tile_bytes, tile_bytes, full + stage);
          last_stage_it[stage] = static_cast<int>(it);
        }
      }
      if (!ok) {
        fail(1);
        for (int s = 0; s < kGemmStages; ++s)
          if (last_stage_it[s] >= 0) mbar_wait(full + s, (static_cast<uint32_t>(last_stage_it[s]) / kGemmStages) & 1);
        if (a_issued >= 0) mbar_wait(afull, static_cast<uint32_t>(a_issued) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0, tc = 0, ul = 0;
      bool ok = true;
      for (size_t u = 0; ok && u < units; ++u, ++ul) {
        size_t rb, c0;
        uint32_t ntiles;
        unit_range(u, rb, c0, ntiles);
        if (!mbar_wait_sleep(afull, ul & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA);
        for (uint32_t t = 0; t < ntiles; ++t, ++it, ++tc) {
          const uint32_t stage = it % kGemmStages, ph = (it / kGemmStages) & 1;
          const uint32_t acc = tc % kGemmAcc, aph = (tc / kGemmAcc) & 1;
          if (!mbar_wait_sleep(full + stage, ph) || !mbar_wait_sleep(accempty + acc, aph ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_base = smem_u32(sB + stage * tile_bytes);
          for (int ks = 0; ks < p.ksteps; ++ks) {
            const uint32_t off = static_cast<uint32_t>(ks >> 2) * kBlockBytes + static_cast<uint32_t>(ks & 3) * 32u;
            umma_f16(tmem + acc * kTile, umma_desc(a_base + off), umma_desc(b_base + off), ks != 0);
          }
          umma_commit(empty + stage);
          umma_commit(accfull + acc);
        }
        if (ok) umma_commit(aempty);
      }
      if (!ok) fail(2);
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else {
    // epilogue warpgroup eg takes the tiles of accumulator eg; warp ew of it
    // owns TMEM lanes (rows) 32 ew .. 32 ew + 31, lane = row
    const int eg = (warp - 2) >> 2, ew = warp & 3;
    const int rloc = ew * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(eg) * kTile;
    const bool store = p.out != nullptr;
    const bool vec = (p.ld & 7) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
    uint4 *stg = stage_out + static_cast<size_t>(warp - 2) * 32 * 4;  // [32 rows][4 chunks of 16 B]
    uint32_t tc = 0;
    bool ok = true;
    for (size_t u = 0; ok && u < units; ++u) {
      size_t rb, c0;
      uint32_t ntiles;
      unit_range(u, rb, c0, ntiles);
      const size_t row = rb * kTile + rloc;
      const bool rv = row < p.rows;
      const float slo_row = kGather && rv ? p.slo[row] : 0.0f;
      for (uint32_t t = 0; t < ntiles; ++t, ++tc) {
        const uint32_t acc = tc % kGemmAcc;
        if (acc != static_cast<uint32_t>(eg)) continue;
        if (!__all_sync(VG_FULL_MASK, mbar_wait_sleep(accfull + acc, (tc / kGemmAcc) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const size_t col0 = c0 + static_cast<size_t>(t) * kTile;
        const int nval = static_cast<int>(min(static_cast<size_t>(kTile), p.cols - col0));
        uint32_t mpack[2] = {0u, 0u};  // the four chunk maxima as binary16 pairs
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {  // 32 columns (one chunk) at a time
          uint32_t v[32];
          tmem_ld32_nowait(t_lane + h * 32, v);
          tmem_wait_ld();
          if (h == 3) {  // the accumulator is read: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accempty + acc);
          }
          const int nh = min(max(nval - h * 32, 0), 32);  // valid columns in this chunk
          // the largest product of the chunk, rounded as the products are
          // (rounding is monotone: the largest rounded product)
          float m = -__int_as_float(0x7f800000);
          if (nh == 32) {  // a whole chunk (nh is the same for the warp): a tree
            m = max32(v);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nh) m = fmaxf(m, __uint_as_float(v[j]));
          }
          const uint32_t mb = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(m)));
          if (h == 0) mpack[0] = mb;
          if (h == 1) mpack[0] |= mb << 16;
          if (h == 2) mpack[1] = mb;
          if (h == 3) mpack[1] |= mb << 16;
          const size_t colh = col0 + static_cast<size_t>(h) * 32;
          if (kGather && rv && m >= slo_row) {
            // this row's columns of the chunk at or above its threshold
            // (a few hundred per row over every column): the lane parks its
            // values in its own 64-byte row of the staging buffer, 16 at a
            // time, and stores only the columns that pass
            uint32_t take = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              take |= (j < nh && __uint_as_float(v[j]) >= slo_row ? 1u : 0u) << j;
            uint32_t pos = atomicAdd(p.count + row, static_cast<uint32_t>(__popc(take)));
            uint2 *dst = p.cand + row * p.cap;
            const uint32_t cb = p.col_base + static_cast<uint32_t>(colh);
            uint32_t *park = reinterpret_cast<uint32_t *>(stg + lane * 4);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              uint32_t t16 = (take >> (16 * half)) & 0xffffu;
              if (!t16) continue;
#pragma unroll
              for (int c = 0; c < 4; ++c)
                stg[lane * 4 + c] = make_uint4(v[16 * half + 4 * c], v[16 * half + 4 * c + 1],
                                               v[16 * half + 4 * c + 2], v[16 * half + 4 * c + 3]);
              while (t16) {
                const int j = __ffs(t16) - 1;
                t16 &= t16 - 1;
                if (pos < p.cap) dst[pos] = make_uint2(cb + static_cast<uint32_t>(16 * half + j), park[j]);
                ++pos;
              }
            }
          }
          if (!store) {
          } else if (vec && nval == kTile) {
            // the warp's 32 rows x 64 bytes through shared memory (chunk j of
            // row r at r * 4 + (j ^ ((r >> 1) & 3)): conflict-free both ways),
            // then 64-byte row pieces: 4 lanes per row, 8 rows per store
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              __half2 h0 = __floats2half2_rn(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1]));
              __half2 h1 = __floats2half2_rn(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
              __half2 h2 = __floats2half2_rn(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
              __half2 h3 = __floats2half2_rn(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
              uint4 o;
              o.x = *reinterpret_cast<uint32_t *>(&h0);
              o.y = *reinterpret_cast<uint32_t *>(&h1);
              o.z = *reinterpret_cast<uint32_t *>(&h2);
              o.w = *reinterpret_cast<uint32_t *>(&h3);
              stg[lane * 4 + (j ^ ((lane >> 1) & 3))] = o;
            }
            __syncwarp();
            const int rq = lane >> 2, j = lane & 3;
#pragma unroll
            for (int r8 = 0; r8 < 32; r8 += 8) {
              const int r = r8 + rq;
              const size_t grow = rb * kTile + ew * 32 + r;
              const uint4 o = stg[r * 4 + (j ^ ((r >> 1) & 3))];
              if (grow < p.rows) *reinterpret_cast<uint4 *>(p.out + grow * p.ld + colh + 8 * j) = o;
            }
            __syncwarp();
          } else if (rv) {
            __half *dst = p.out + row * p.ld + colh;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nh) dst[j] = __float2half_rn(__uint_as_float(v[j]));
          }
        }
        if (p.cmax && rv) *reinterpret_cast<uint2 *>(p.cmax + row * p.cstride + (col0 / kTile) * 4) =
            make_uint2(mpack[0], mpack[1]);
      }
    }
    if (!ok) fail(3);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kGemmTmemCols) : "memory");
  }
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
  // Column ranges per row block: the split that finishes the work units in
  // the fewest rounds of num_sms CTAs (relative to one whole row block),
  // ranges of at least 512 columns.  The ranges of a row share their bound
  // on the P-th product, so splitting costs little in window width.
  const size_t rblocks = std::max<size_t>(1, (rows + kTile - 1) / kTile);
  const size_t ctiles = (cols + kTile - 1) / kTile;
  const size_t smax = std::max<size_t>(1, std::min<size_t>(64, ctiles / 4));
  size_t best = 1;
  double best_t = 1e30;
  for (size_t sp = 1; sp <= smax; ++sp) {
    const size_t per_tiles = (ctiles + sp - 1) / sp;
    const size_t real_sp = (ctiles + per_tiles - 1) / per_tiles;
    const size_t rounds = (rblocks * real_sp + num_sms - 1) / num_sms;
    const double t = static_cast<double>(rounds) * per_tiles + 2.0 * rounds;  // + per-unit overhead
    if (t < best_t - 1e-9) {
      best_t = t;
      best = sp;
    }
  }
  const size_t per_tiles = (ctiles + best - 1) / best;
  *split_cols = static_cast<uint32_t>(per_tiles * kTile);
  *splits = static_cast<int>((ctiles + per_tiles - 1) / per_tiles);
  *cap = P == 1 ? 32 : std::min(1024, (2 * P + 64 + 31) / 32 * 32);
}

size_t tc_select_workspace_bytes(size_t rows, size_t cols, int P, int num_sms) {
  int sp, cap;
  uint32_t per;
  tc_select_plan(rows, cols, P, num_sms, &sp, &per, &cap);
  return rows * sp * 2 * (static_cast<size_t>(cap) * 8 + 4) + rows * 4 + 256;
}

cudaError_t launch_tc_select(const TcSelect &t, int num_sms, cudaStream_t s) {
  if (t.rows == 0 || t.P <= 0) return cudaSuccess;
  if (t.P > 256 || (t.kp != 64 && t.kp != 128) || t.cols == 0 || t.cols > 0xfffffffeull) return cudaErrorInvalidValue;
  int sp, cap;
  uint32_t per;
  tc_select_plan(t.rows, t.cols, t.P, num_sms, &sp, &per, &cap);
  uint2 *cand = static_cast<uint2 *>(t.workspace);
  uint32_t *count = reinterpret_cast<uint32_t *>(cand + t.rows * sp * 2 * static_cast<size_t>(cap));
  uint32_t *gbound = count + t.rows * sp * 2;
  cudaError_t e = cudaMemsetAsync(gbound, 0, t.rows * 4, s);
  if (e != cudaSuccess) return e;
  WinParams wp{};
  wp.a_img = static_cast<const uint8_t *>(t.a_img);
  wp.b_img = static_cast<const uint8_t *>(t.b_img);
  wp.rows = t.rows;
  wp.cols = t.cols;
  wp.kp = t.kp;
  wp.ksteps = (t.d + 15) / 16;
  wp.P = t.P;
  wp.top1 = t.P == 1;
  wp.splits = sp;
  wp.split_cols = per;
  wp.cap = cap;
  wp.eps = t.eps;
  wp.cand = cand;
  wp.count = count;
  wp.gbound = gbound;
  wp.error = t.error;
  const size_t smem = win_smem_bytes(t.kp);
  e = cudaFuncSetAttribute(tc_window_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
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
  fp.splits = sp * 2;  // a candidate segment per (range, epilogue warpgroup)
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

namespace {

cudaError_t launch_gemm(const GemmParams &gp, int num_sms, cudaStream_t s) {
  const size_t rblocks = (gp.rows + kTile - 1) / kTile, ctiles = (gp.cols + kTile - 1) / kTile;
  const size_t smem = 1024 + static_cast<size_t>(gp.kp / kKBlock) * kBlockBytes * (1 + kGemmStages) +
                      static_cast<size_t>(kGemmEpiWarps) * 32 * 4 * 16 + 32 * 8 + 16;
  auto kern = gp.slo ? tc_gemm_f16_kernel<true> : tc_gemm_f16_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // one CTA per SM, each with an equal share of the tiles
  kern<<<static_cast<unsigned>(std::min<size_t>(rblocks * ctiles, num_sms)), kGemmThreads, smem, s>>>(gp);
  return cudaGetLastError();
}

GemmParams gemm_params(const void *a_img, size_t rows, const void *b_img, size_t cols, int d, int kp, int *error) {
  GemmParams gp{};
  gp.a_img = static_cast<const uint8_t *>(a_img);
  gp.b_img = static_cast<const uint8_t *>(b_img);
  gp.rows = rows;
  gp.cols = cols;
  gp.kp = kp;
  gp.ksteps = (d + 15) / 16;
  gp.error = error;
  return gp;
}

// The P-th largest chunk maximum of each row turned into the row's gather
// threshold (warp per row).  Chunk maxima are binary16 roundings of the f32
// products; m_P, the P-th largest over the lanes' 2R largest values, is
// reached by P distinct chunks, so P distinct columns have products
// s >= S = m_P - 2^-11 |m_P| - 2^-25 (one binary16 rounding) and the row's
// P-th smallest approximate distance is at most fl(1 - S).  Every column
// whose approximate distance is within 2 eps of that -- every column the
// finisher may need -- has s >= slo = S - 2 eps - 2^-20 (1 + |1 - S| + 2 eps)
// (f32 rounding of the distances, with room), rounded down.  Rows with fewer
// than P chunks, a non-finite m_P or eps >= 1 get slo = -inf (every column
// gathered: the finisher then scores the row exactly).
template <int R>
__global__ void __launch_bounds__(256) chunk_threshold_kernel(const __half *__restrict__ cmax, size_t rows,
                                                              size_t nch, size_t cstride, int P,
                                                              const float *__restrict__ eps, float *__restrict__ slo) {
  constexpr int R2 = 2 * R;
  const int lane = lane_id();
  const size_t row = static_cast<size_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float kInf = __int_as_float(0x7f800000);
  float a[R2];  // this lane's 2R largest maxima, descending (-inf: empty)
#pragma unroll
  for (int r = 0; r < R2; ++r) a[r] = -kInf;
  auto insert = [&](float x) {
    if (!(x > a[R2 - 1])) return;  // -inf and NaN never enter
#pragma unroll
    for (int r = 0; r < R2; ++r) {
      const float hi = fmaxf(x, a[r]);
      x = fminf(x, a[r]);
      a[r] = hi;
    }
  };
  const uint2 *src = reinterpret_cast<const uint2 *>(cmax + row * cstride);
  for (size_t i = lane; i < nch / 4; i += 32) {
    const uint2 w = __ldcs(src + i);
    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
    insert(lo.x);
    insert(lo.y);
    insert(hi.x);
    insert(hi.y);
  }
  // the P-th smallest of -a over the warp: bisection on the order key
  uint32_t okey[R2];
  int have = 0;
#pragma unroll
  for (int r = 0; r < R2; ++r) {
    okey[r] = a[r] == -kInf ? 0xffffffffu : order_key(-a[r]);
    have += okey[r] != 0xffffffffu;
  }
  const bool full = __reduce_add_sync(VG_FULL_MASK, static_cast<unsigned>(have)) >= static_cast<unsigned>(P);
  uint32_t klo = 0, khi = 0xfffffffeu;
  while (full && klo < khi) {
    const uint32_t mid = klo + ((khi - klo) >> 1);
    int c = 0;
#pragma unroll
    for (int r = 0; r < R2; ++r) c += okey[r] <= mid;
    if (__reduce_add_sync(VG_FULL_MASK, static_cast<unsigned>(c)) >= static_cast<unsigned>(P))
      khi = mid;
    else
      klo = mid + 1;
  }
  if (lane == 0) {
    const double e = static_cast<double>(eps[row]);
    const double mp = full ? -static_cast<double>(key_to_float(klo)) : 0.0;
    float out = -kInf;
    if (full && e < 1.0 && fabs(mp) < 65536.0) {
      const double S = mp - fabs(mp) * (1.0 / 2048.0) - 2.9802322387695312e-8;
      out = __double2float_rd(S - 2.0 * e - 9.5367431640625e-7 * (1.0 + fabs(1.0 - S) + 2.0 * e));
    }
    slo[row] = out;
  }
}

// candidates per row of the gather pass: about P x (columns / sampled
// columns) lie at or above the sampled threshold
uint32_t sampled_cap(size_t cols, size_t sample_cols, int P) {
  const double ratio = static_cast<double>(cols) / static_cast<double>(std::max<size_t>(sample_cols, 1));
  const double c = 2.0 * P * std::min(ratio, 64.0) + 512.0;
  return static_cast<uint32_t>(std::min(32768.0, std::ceil(c / 32.0) * 32.0));
}

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

}  // namespace

cudaError_t launch_tc_gemm_f16(const void *a_img, size_t rows, const void *b_img, size_t cols, int d, int kp,
                               void *out, size_t ld, void *cmax, size_t cstride, int *error, int num_sms,
                               cudaStream_t s) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  if ((kp != 64 && kp != 128) || d < 1 || d > kp) return cudaErrorInvalidValue;
  GemmParams gp = gemm_params(a_img, rows, b_img, cols, d, kp, error);
  gp.ld = ld;
  gp.out = static_cast<__half *>(out);
  gp.cmax = static_cast<__half *>(cmax);
  gp.cstride = cstride;
  return launch_gemm(gp, num_sms, s);
}

size_t tc_sampled_workspace_bytes(size_t rows, size_t cols, size_t sample_cols, int P) {
  const size_t cap = sampled_cap(cols, sample_cols, P);
  const size_t cstride = 4 * ((sample_cols + kTile - 1) / kTile);
  return align256(rows * cap * 8) + align256(rows * 4) * 2 + align256(rows * cstride * 2) + 256;
}

cudaError_t launch_tc_sampled_select(const TcSampledSelect &t, int num_sms, cudaStream_t s) {
  if (t.rows == 0 || t.P <= 0) return cudaSuccess;
  if (t.P > 256 || (t.kp != 64 && t.kp != 128) || t.cols == 0 || t.cols > 0xfffffffeull || t.sample_cols == 0 ||
      t.d < 1 || t.d > t.kp)
    return cudaErrorInvalidValue;
  const uint32_t cap = sampled_cap(t.cols, t.sample_cols, t.P);
  const size_t cstride = 4 * ((t.sample_cols + kTile - 1) / kTile);
  uint8_t *w = static_cast<uint8_t *>(t.workspace);
  uint2 *cand = reinterpret_cast<uint2 *>(w);
  w += align256(t.rows * cap * 8);
  uint32_t *count = reinterpret_cast<uint32_t *>(w);
  w += align256(t.rows * 4);
  float *slo = reinterpret_cast<float *>(w);
  w += align256(t.rows * 4);
  __half *cm = reinterpret_cast<__half *>(w);
  cudaError_t e = cudaMemsetAsync(count, 0, t.rows * 4, s);
  if (e != cudaSuccess) return e;
  if (t.marks[0]) cudaEventRecord(t.marks[0], s);
  // 1. chunk maxima over the sampled columns, then every row's threshold
  GemmParams gp = gemm_params(t.a_img, t.rows, t.sample_img, t.sample_cols, t.d, t.kp, t.error);
  gp.cmax = cm;
  gp.cstride = cstride;
  if ((e = launch_gemm(gp, num_sms, s)) != cudaSuccess) return e;
  const unsigned tgrid = static_cast<unsigned>((t.rows + 7) / 8);
  if (t.P <= 32)
    chunk_threshold_kernel<1><<<tgrid, 256, 0, s>>>(cm, t.rows, cstride, cstride, t.P, t.eps, slo);
  else if (t.P <= 64)
    chunk_threshold_kernel<2><<<tgrid, 256, 0, s>>>(cm, t.rows, cstride, cstride, t.P, t.eps, slo);
  else if (t.P <= 128)
    chunk_threshold_kernel<4><<<tgrid, 256, 0, s>>>(cm, t.rows, cstride, cstride, t.P, t.eps, slo);
  else
    chunk_threshold_kernel<8><<<tgrid, 256, 0, s>>>(cm, t.rows, cstride, cstride, t.P, t.eps, slo);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // 2. every column, in ranges of 16 MB of operand tiles (shared in L2 by
  // every CTA of a launch): columns at or above the threshold are gathered
  const size_t tile_bytes = static_cast<size_t>(t.kp) * kTile * 2;
  const size_t range = (16u << 20) / tile_bytes * kTile;
  for (size_t c0 = 0; c0 < t.cols; c0 += range) {
    GemmParams g2 = gemm_params(t.a_img, t.rows, static_cast<const uint8_t *>(t.b_img) + c0 / kTile * tile_bytes,
                                std::min(range, t.cols - c0), t.d, t.kp, t.error);
    g2.slo = slo;
    g2.cand = cand;
    g2.count = count;
    g2.cap = cap;
    g2.col_base = static_cast<uint32_t>(c0);
    if ((e = launch_gemm(g2, num_sms, s)) != cudaSuccess) return e;
  }
  if (t.marks[1]) cudaEventRecord(t.marks[1], s);
  // 3. the P-th smallest approximate distance over the candidates, exact
  // re-score of those within 2 eps of it, exact top-P
  FinParams fp{};
  fp.cand = cand;
  fp.count = count;
  fp.splits = 1;
  fp.cap = static_cast<int>(cap);
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
  e = t.P <= 32 ? launch_finish<1>(fp, s) : t.P <= 64 ? launch_finish<2>(fp, s)
      : t.P <= 128 ? launch_finish<4>(fp, s) : launch_finish<8>(fp, s);
  if (e == cudaSuccess && t.marks[2]) cudaEventRecord(t.marks[2], s);
  return e;
}

}  // namespace vg

// ---------------------------------------------------------------------------
// Self-check of the bounded-wait path every pipelined kernel above uses: one
// thread waits, with the given cycle limit, on an mbarrier phase that nothing
// completes, then reports through the error flag exactly as a kernel role
// does when a wait runs out (code 4) and returns.
// ---------------------------------------------------------------------------
namespace vg {
namespace {
__global__ void bounded_wait_check_kernel(long long limit_cycles, int *error) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  if (!mbar_wait_sleep_for(&bar, 0, limit_cycles)) atomicExch(error, 4);
}
}  // namespace

cudaError_t launch_bounded_wait_check(long long limit_cycles, int *error, cudaStream_t s) {
  if (limit_cycles <= 0 || limit_cycles > kWaitCycles) return cudaErrorInvalidValue;
  bounded_wait_check_kernel<<<1, 32, 0, s>>>(limit_cycles, error);
  return cudaGetLastError();
}
}  // namespace vg
