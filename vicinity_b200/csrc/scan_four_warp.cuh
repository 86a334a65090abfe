// Warp-per-query search kernel for 16-entry (4-bit) codebooks.
//
// Same results as ivfpq_four_kernel (search.rs:1175-1391 with the FastScan
// tables of pq_simd.rs:576-769).  Here one warp owns a query for its whole
// search: for each probed list in order it
//   - skips the list when the bound on its quantised distances (known
//     before the table exists) exceeds the warp's current k-th distance;
//   - builds the list's float table (entries e = lane + 32 i, warp-private),
//     reduces its min/max with shuffles and quantises it into a warp-private
//     768-byte u8 table;
//   - checks the exact bound with the table's scale, then scores the
//     candidates with integer sums of nibble lookups, exiting early per 16
//     codes.
// Lists under 16 vectors use the reference's float path: the float entries,
// computed on the fly from the shared-memory codebook, summed in order.
// No block barriers, no merge; the freshest k-th distance prunes every list.
#pragma once

#include <cfloat>

#include "scan_fourbit.cuh"
#include "scan_work.cuh"

namespace vg {

constexpr int kFourWarpThreads = 1024;
constexpr int kFourWarpWarps = kFourWarpThreads / 32;

// shared memory: codebook [M][16][dsub], then per warp the residual [d], the
// float table [M * 16] and the u8 table [M][16]
__host__ __device__ inline size_t four_warp_smem_bytes(int M, int dsub, int d) {
  const size_t cb = (static_cast<size_t>(M) * 16 * dsub + 3) & ~size_t(3);
  const size_t dpad = (static_cast<size_t>(d) + 3) & ~size_t(3);
  return cb * 4 + kFourWarpWarps * ((dpad + four_float_stride(M)) * 4 + four_u8_stride(M));
}

__device__ __forceinline__ void prefetch_l1_4(const void *a) { asm volatile("prefetch.global.L1 [%0];" ::"l"(a)); }

// Float table entry (m, c): sum_j (r_j - w_j)^2 in j order (first square as is).
__device__ __forceinline__ float four_entry(const float *rb, const float *cbs, int dsub, int m, int c) {
  const float *r = rb + m * dsub, *w = cbs + (m * 16 + c) * dsub;
  const float d0 = __fsub_rn(r[0], w[0]);
  float t = __fmul_rn(d0, d0);
  for (int j = 1; j < dsub; ++j) {
    const float dj = __fsub_rn(r[j], w[j]);
    t = __fadd_rn(t, __fmul_rn(dj, dj));
  }
  return t;
}

template <int R>
__global__ void __launch_bounds__(kFourWarpThreads, 1) ivfpq_four_warp_kernel(const ScanParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, d = p.d, P = p.P, k = p.k, dsub = p.dsub;
  const int nent = M * 16;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int dpad = (d + 3) & ~3;
  const int fstride = static_cast<int>(four_float_stride(M));
  float *cbs = reinterpret_cast<float *>(smem);                                     // [M][16][dsub]
  float *rb = cbs + ((nent * dsub + 3) & ~3) + static_cast<size_t>(warp) * (dpad + fstride);  // residual [d]
  float *ft = rb + dpad;                                                            // float table [M * 16]
  uint8_t *qt = reinterpret_cast<uint8_t *>(cbs + ((nent * dsub + 3) & ~3) + kFourWarpWarps * (dpad + fstride)) +
                static_cast<size_t>(warp) * four_u8_stride(M);                      // u8 table [M][16]
  const uint32_t qt_a = smem_u32(qt);

  for (int i = tid; i < nent * dsub; i += kFourWarpThreads) cbs[i] = p.codebooks[i];
  __syncthreads();
  ScanWork work;
  work.init(p);

  for (;;) {
    uint32_t w = 0;
    if (lane == 0) w = atomicAdd(p.counter, 1u);
    w = __shfl_sync(VG_FULL_MASK, w, 0);
    if (w >= work.total) break;
    uint32_t q;
    int first, last;
    size_t orow;
    work.item(p, w, q, first, last, orow);
    const float *qv = p.qn + static_cast<size_t>(q) * d;
    WarpTopK<R> tk;
    tk.init();
    uint32_t n_lists = 0, n_vecs = 0, n_tables = 0, n_groups = 0;  // profiling counters
    // a ceiling key (a bound on the query's k-th key over every shard) keeps
    // only keys at or below it
    uint64_t kth0 = kEmptyKey;
    if (p.key_ceiling) {
      const uint64_t c = p.key_ceiling[static_cast<size_t>(q) * (p.ceiling_stride ? p.ceiling_stride : 1)];
      kth0 = c == kEmptyKey ? kEmptyKey : c + 1;
    }
    if (p.init_keys) {  // keys of probes scanned earlier (a seed pass) start the top-k
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int i = r * 32 + lane;
        tk.add(i < k ? p.init_keys[static_cast<size_t>(q) * k + i] : kEmptyKey);
      }
    }
    uint64_t kth = min(tk.get(k - 1), kth0);
    const bool seed = p.seed_next != nullptr;
    int seed_stop = P;
    bool stopped = false;
    if (seed) {  // a seed pass scores only queries whose nearest list is this rank's
      const uint32_t l0 = p.probes[static_cast<size_t>(q) * P];
      if (l0 == 0xffffffffu || (p.owner && !p.owner[l0])) {
        seed_stop = 1;
        first = last;
      }
    }
    // probes in groups of 32, in order: lane i loads probe c0 + i (list,
    // ownership, bounds, extent) so the warp walks only the live ones with no
    // global load on its serial path; a list the group's starting bound
    // prunes stays pruned (the bound only tightens)
    for (int c0 = first; c0 < last; c0 += 32) {
      if (stopped) break;
      if (seed && tk.get(k - 1) != kEmptyKey) {
        seed_stop = c0;
        break;
      }
      const size_t pr_l = static_cast<size_t>(q) * P + c0 + lane;
      uint32_t l_l = 0xffffffffu, len_l = 0;
      uint64_t lbeg_l = 0, off_l = 0;
      float lbq_l = 0.0f, lb_l = 0.0f;
      if (c0 + lane < last) {
        l_l = p.probes[pr_l];
        if (l_l != 0xffffffffu && p.owner && !p.owner[l_l]) l_l = 0xffffffffu;
        if (l_l != 0xffffffffu) {
          lbeg_l = p.list_off[l_l];
          len_l = static_cast<uint32_t>(p.list_off[l_l + 1] - lbeg_l);
          off_l = len_l >= 16 ? p.pack_off[l_l] : p.code_off[l_l];
          if (p.probe_lbq) lbq_l = p.probe_lbq[pr_l];
          if (p.probe_lb) lb_l = p.probe_lb[pr_l];
        }
      }
      const bool pruned0 = kth != kEmptyKey && p.probe_lbq && lbq_l > key_dist(kth);  // before the table
      unsigned todo = __ballot_sync(VG_FULL_MASK, l_l != 0xffffffffu && len_l > 0 && !pruned0);
      while (todo) {
        const int pj = __ffs(todo) - 1;
        todo &= todo - 1;
        if (seed && tk.get(k - 1) != kEmptyKey) {
          seed_stop = c0 + pj;
          stopped = true;
          break;
        }
        if (kth != kEmptyKey && p.probe_lbq && __shfl_sync(VG_FULL_MASK, lbq_l, pj) > key_dist(kth)) continue;
        const uint32_t l = __shfl_sync(VG_FULL_MASK, l_l, pj);
        const uint64_t lbeg = shfl64(lbeg_l, pj);
        const uint32_t len = __shfl_sync(VG_FULL_MASK, len_l, pj);
        const uint64_t loff = shfl64(off_l, pj);
        const float lb_p = __shfl_sync(VG_FULL_MASK, lb_l, pj);
        const float *cent = p.centroids + static_cast<size_t>(l) * d;
        __syncwarp();
        for (int j = lane; j < d; j += 32) rb[j] = __fsub_rn(qv[j], cent[j]);
        __syncwarp();
        const uint32_t *ids = p.list_ids + lbeg;
        if (len < 16) {  // search.rs:1261: float table, sequential float sum
          ++n_lists;
          n_vecs += len;
          const uint8_t *codes = p.list_codes + loff;
          const bool alive = lane < static_cast<int>(len);
          float dist = 0.0f;
          if (alive)
            for (int m = 0; m < M; ++m)
              dist = __fadd_rn(dist, four_entry(rb, cbs, dsub, m, codes[static_cast<size_t>(lane) * M + m]));
          const uint32_t dk = order_key(dist);
          const bool pass = alive && (kth == kEmptyKey || dk <= static_cast<uint32_t>(kth >> 32));
          const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | ids[lane]) : kEmptyKey;
          tk.add(key < kth ? key : kEmptyKey);
          kth = min(tk.get(k - 1), kth0);
          continue;
        }
        // the first codes of the list come in while the table is built
        const uint8_t *packed = p.packed + loff;
        const int vb = (M + 1) >> 1;  // bytes per vector in the nibble layout
        if (static_cast<uint32_t>(lane) < len) prefetch_l1_4(packed + static_cast<uint64_t>(lane) * vb);
        ++n_tables;
        // float table (warp-private), its min / max (pq_simd.rs:587-598: NaNs
        // skipped as the reference's comparisons do), u8 quantisation
        float lmin = __int_as_float(0x7f800000), lmax = -__int_as_float(0x7f800000);
        for (int e = lane; e < nent; e += 32) {
          const float t = four_entry(rb, cbs, dsub, e >> 4, e & 15);
          ft[e] = t;
          lmin = fminf(lmin, t);
          lmax = fmaxf(lmax, t);
        }
  #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          lmin = fminf(lmin, __shfl_xor_sync(VG_FULL_MASK, lmin, off));
          lmax = fmaxf(lmax, __shfl_xor_sync(VG_FULL_MASK, lmax, off));
        }
        const float range = __fsub_rn(lmax, lmin);
        const bool flat = range < FLT_EPSILON;
        const float inv = flat ? 0.0f : __fdiv_rn(255.0f, range);
        const float scale = flat ? 1.0f : __fdiv_rn(range, 255.0f);
        const float fb = __fmul_rn(lmin, static_cast<float>(M));
        // exact bound with this table's scale (see ivfpq_four_kernel)
        if (kth != kEmptyKey && p.probe_lb) {
          const double lbq = static_cast<double>(lb_p) * (1.0 - 16 * 5.9604644775390625e-8) -
                             0.5 * M * static_cast<double>(scale) * (1.0 + 1e-5);
          if (lbq > static_cast<double>(key_dist(kth))) continue;
        }
        __syncwarp();
        for (int e = lane; e < nent; e += 32) {  // each lane its own entries
          // round half away from zero, clamp; NaN -> 0 (pq_simd.rs:607-609)
          float t = roundf(__fmul_rn(__fsub_rn(ft[e], lmin), inv));
          t = fminf(fmaxf(t, 0.0f), 255.0f);
          qt[e] = static_cast<uint8_t>(t);
        }
        __syncwarp();
        // candidates: integer sums of the u8 entries, checked every 16 codes
        ++n_lists;
        n_vecs += len;
        for (uint32_t x0 = 0; x0 < len; x0 += 32) {
          const uint32_t c = x0 + lane;
          bool live = c < len;
          if (c + 32 < len) prefetch_l1_4(packed + static_cast<uint64_t>(c + 32) * vb);  // next chunk
          const uint32_t tkey = static_cast<uint32_t>(kth >> 32);
          const uint8_t *vp = packed + static_cast<uint64_t>(live ? c : 0u) * vb;
          uint32_t acc = 0;
          if ((M & 15) == 0) {
            for (int m0 = 0; m0 < M; m0 += 16) {
              const unsigned lm = __ballot_sync(VG_FULL_MASK, live);
              if (!lm) break;
              n_groups += __popc(lm);
              if (live) {
                const uint2 w = *reinterpret_cast<const uint2 *>(vp + (m0 >> 1));
                acc += nibble_sum16(w, qt_a + static_cast<uint32_t>(m0 * 16));
                live = order_key(__fadd_rn(__fmul_rn(__uint2float_rn(acc), scale), fb)) <= tkey;
              }
            }
          } else if (live) {
            for (int m = 0; m < M; ++m) acc += qt[m * 16 + ((vp[m >> 1] >> ((m & 1) * 4)) & 15u)];
            live = order_key(__fadd_rn(__fmul_rn(__uint2float_rn(acc), scale), fb)) <= tkey;
          }
          const float dist = __fadd_rn(__fmul_rn(__uint2float_rn(acc), scale), fb);
          const uint32_t dk = order_key(dist);
          const bool pass = live && dk <= tkey;
          unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
          if (!mask) continue;
          const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | ids[c]) : kEmptyKey;
          if (__popc(mask) > 4) {
            tk.add(key < kth ? key : kEmptyKey);
          } else {
            while (mask) {
              const int src = __ffs(mask) - 1;
              mask &= mask - 1;
              const uint64_t kx = shfl64(key, src);
              if (kx < kth) topk_insert_one(tk, kx);
            }
          }
          kth = min(tk.get(k - 1), kth0);
        }
      }
    }

    if (p.out_kth) {
      const uint64_t kk = tk.get(k - 1);
      if (lane == 0) p.out_kth[q] = kk;
    }
    if (seed && lane == 0) p.seed_next[q] = static_cast<uint32_t>(seed_stop);
    uint32_t count = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = r * 32 + lane;
      const uint64_t key = tk.v[r];
      const bool real = i < k && key != kEmptyKey;
      count += __popc(__ballot_sync(VG_FULL_MASK, real));
      if (i < k) {
        const size_t o = orow * k + i;
        if (p.out_keys) p.out_keys[o] = key;
        if (p.out_ids) {
          p.out_ids[o] = real ? p.doc_ids[key_id(key)] : 0xffffffffu;
          p.out_dist[o] = real ? key_dist(key) : __int_as_float(0x7f800000);
        }
      }
    }
    if (p.out_count && lane == 0) p.out_count[q] = count;
    if (p.scored && lane == 0) {
      atomicAdd(p.scored, static_cast<unsigned long long>(n_lists));
      atomicAdd(p.scored + 1, static_cast<unsigned long long>(n_vecs));
      atomicAdd(p.scored + 2, static_cast<unsigned long long>(n_tables));
      atomicAdd(p.scored + 3, static_cast<unsigned long long>(n_groups));
    }
  }
}

}  // namespace vg
