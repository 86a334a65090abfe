// Fused IVF-PQ search for 16-entry (4-bit) codebooks.
//
// Same per-query loop as ivfpq_query_kernel (search.rs:1175-1391) and the
// same results; the work is laid out for what 4-bit tables cost:
//   - a table has only M x 16 entries, so the per-table steps (building,
//     global min/max, u8 quantisation, pq_simd.rs:576-611) are a large share
//     of the work.  Each list of a batch gets its own 128 threads: they build
//     the float table from the shared-memory codebook, reduce min/max among
//     their four warps (named barrier), and quantise their own entries --
//     no integer division and no idle threads in the reductions;
//   - tables are double-buffered, so one block barrier per batch separates
//     building batch b + 1 from scanning batch b;
//   - a candidate's codes are read from the vector-major nibble layout with
//     8-byte loads, and every table lookup is one LOP3 (nibble | 16-byte
//     aligned row address) plus one shared-memory byte load whose subspace
//     offset is an immediate.  All lanes read the same 16-byte row, so the
//     lookups are free of bank conflicts;
//   - lists under 16 vectors use the unquantised float table and the
//     sequential float sum, as the reference does (search.rs:1261);
//   - batches are formed one ahead from the lists whose quantised distances
//     may still come under the block's k-th distance (a bound computed before
//     the table exists, from the residual's per-subspace norms), so pruned
//     lists cost no table; after quantisation the exact scale decides again
//     whether the list is scored.
// The quantised distance is sum * scale + min * M (pq_simd.rs:721-769) with
// the integer sum exact in any order.
#pragma once

#include <cfloat>

#include "pipeline.cuh"
#include "scan_kernel.cuh"

namespace vg {

constexpr int kFourGroup = 128;  // threads that build one list's table

__host__ __device__ inline size_t four_float_stride(int M) { return (static_cast<size_t>(M) * 16 + 3) & ~size_t(3); }
__host__ __device__ inline size_t four_u8_stride(int M) { return (static_cast<size_t>(M) * 16 + 15) & ~size_t(15); }

__host__ __device__ inline size_t four_smem_bytes(int M, int dsub, int R, bool rot = false) {
  const size_t nent = static_cast<size_t>(M) * 16;
  const size_t dpad = (static_cast<size_t>(M) * dsub + 3) & ~size_t(3);
  return static_cast<size_t>(kScanWarps) * 32 * R * 8 + ((nent * dsub + 3) & ~size_t(3)) * 4 +
         2 * kMaxBatch * (four_float_stride(M) * 4 + four_u8_stride(M)) +
         (rot ? kMaxBatch * 2 * dpad * 4 : 0);
}

template <int OFF>
__device__ __forceinline__ uint32_t lds_u8(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(OFF) : "memory");
  return v;
}

// Sum of 16 table entries: codes m0..m0+15 of one vector packed in w (code
// 2j low nibble, 2j + 1 high nibble of byte j), rows of 16 bytes from the
// 16-byte aligned shared address `rows`.
__device__ __forceinline__ uint32_t nibble_sum16(uint2 w, uint32_t rows) {
  uint32_t acc = 0;
#define VG_NIB(W, T) acc += lds_u8<(T) * 16>((((W) >> (4 * ((T) & 7))) & 15u) | rows)
  VG_NIB(w.x, 0);
  VG_NIB(w.x, 1);
  VG_NIB(w.x, 2);
  VG_NIB(w.x, 3);
  VG_NIB(w.x, 4);
  VG_NIB(w.x, 5);
  VG_NIB(w.x, 6);
  VG_NIB(w.x, 7);
  VG_NIB(w.y, 8);
  VG_NIB(w.y, 9);
  VG_NIB(w.y, 10);
  VG_NIB(w.y, 11);
  VG_NIB(w.y, 12);
  VG_NIB(w.y, 13);
  VG_NIB(w.y, 14);
  VG_NIB(w.y, 15);
#undef VG_NIB
  return acc;
}

template <int R>
__global__ void __launch_bounds__(kScanThreads, 2) ivfpq_four_kernel(const ScanParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, d = p.d, P = p.P, k = p.k, dsub = p.dsub;
  const int nent = M * 16;
  const int fstride = static_cast<int>(four_float_stride(M));
  const int qstride = static_cast<int>(four_u8_stride(M));
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(smem);             // [warps][32R]
  float *cbs = reinterpret_cast<float *>(wl + kScanWarps * 32 * R);                   // [nent][dsub]
  float *flut = cbs + ((static_cast<size_t>(nent) * dsub + 3) & ~size_t(3));          // [2][batch][fstride]
  uint8_t *qlut = reinterpret_cast<uint8_t *>(flut + 2 * kMaxBatch * fstride);        // [2][batch][qstride]
  const int dpad = (d + 3) & ~3;
  float *qbuf = reinterpret_cast<float *>(qlut + 2 * kMaxBatch * qstride);           // [batch][2][dpad] (OPQ)

  __shared__ uint32_t s_query;
  __shared__ int s_nvalid;
  __shared__ int s_wcount[kScanWarps];
  __shared__ uint32_t s_list[kScanThreads], s_len[kScanThreads];
  __shared__ uint64_t s_lbeg[kScanThreads];
  __shared__ unsigned long long s_bound;
  __shared__ float s_rmin[kMaxBatch][kFourGroup / 32], s_rmax[kMaxBatch][kFourGroup / 32];
  __shared__ float s_scale[2][kMaxBatch], s_fbase[2][kMaxBatch];
  __shared__ float s_lb[kScanThreads];     // distance lower bound of each compacted probe (float tables)
  __shared__ float s_lbq[kScanThreads];    // bound on its quantised distances, before its table is built
  __shared__ uint16_t s_bat[3][kMaxBatch];  // probe positions of batch j (ring j % 3)
  __shared__ int s_bn[3], s_cur;
  __shared__ uint8_t s_skip[2][kMaxBatch];  // list not scanned (pruned), per table set

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = tid / kFourGroup, gt = tid % kFourGroup;  // list slot of the batch, thread in group

  for (int i = tid; i < nent * dsub; i += kScanThreads) cbs[i] = p.codebooks[i];

  for (;;) {
    if (tid == 0) {
      s_query = atomicAdd(p.counter, 1u);
      s_bound = kEmptyKey;
    }
    __syncthreads();
    const uint32_t q = s_query;
    if (q >= static_cast<uint32_t>(p.nq)) break;
    const float *qv = p.qn + static_cast<size_t>(q) * d;
    WarpTopK<R> tk;
    tk.init();

    // probe metadata of the query, compacted to valid owned lists in order
    {
      uint32_t l = 0xffffffffu;
      bool valid = false;
      if (tid < P) {
        l = p.probes[static_cast<size_t>(q) * P + tid];
        valid = l != 0xffffffffu && (!p.owner || p.owner[l]);
      }
      const unsigned vm = __ballot_sync(VG_FULL_MASK, valid);
      if (lane == 0) s_wcount[warp] = __popc(vm);
      __syncthreads();
      int base = 0, total = 0;
      for (int w = 0; w < kScanWarps; ++w) {
        const int c = s_wcount[w];
        base += w < warp ? c : 0;
        total += c;
      }
      if (valid) {
        const int pos = base + __popc(vm & ((1u << lane) - 1u));
        const uint64_t b = p.list_off[l];
        s_list[pos] = l;
        s_lbeg[pos] = b;
        s_len[pos] = static_cast<uint32_t>(p.list_off[l + 1] - b);
        s_lb[pos] = p.probe_lb ? p.probe_lb[static_cast<size_t>(q) * P + tid] : 0.0f;
        s_lbq[pos] = p.probe_lbq ? p.probe_lbq[static_cast<size_t>(q) * P + tid] : -__int_as_float(0x7f800000);
      }
      if (tid == 0) s_nvalid = total;
      __syncthreads();
    }
    const int nvalid = s_nvalid;

    // Batch j (thread 0, before the barrier that precedes scoring batch j - 1):
    // the next lists in probe order whose quantised distances may still come
    // under the block's k-th distance -- the others get no table at all.
    // Batch j holds at most j + 1 lists: the first are formed before anything
    // has been scored.
    auto form = [&](int j) {
      const uint64_t bnd = s_bound;
      const float bdist = key_dist(bnd);
      const int cap = min(kMaxBatch, j + 1);
      int n = 0, c = s_cur;
      for (; c < nvalid && n < cap; ++c)
        if (bnd == kEmptyKey || !(s_lbq[c] > bdist)) s_bat[j % 3][n++] = static_cast<uint16_t>(c);
      s_bn[j % 3] = n;
      s_cur = c;
    };
    if (tid == 0) {
      s_cur = 0;
      form(0);
    }
    __syncthreads();

    for (int b = 0, set = 0; s_bn[b % 3] > 0; ++b, set ^= 1) {
      const int nb = s_bn[b % 3];
      const uint16_t *bat = s_bat[b % 3];
      float *fset = flut + static_cast<size_t>(set) * kMaxBatch * fstride;
      uint8_t *qset = qlut + static_cast<size_t>(set) * kMaxBatch * qstride;

      // ---- tables: list slot `grp` by its 128 threads --------------------
      if (grp < nb) {
        const float *cent = p.centroids + static_cast<size_t>(s_list[bat[grp]]) * d;
        float *fl = fset + static_cast<size_t>(grp) * fstride;
        // OPQ: the table is built from the rotated residual R r (opq.rs:115-121),
        // kept in shared memory; output i is sum_j R[i][j] r_j from 0.0
        const float *rres = nullptr;
        if (p.rot_t) {
          float *res = qbuf + static_cast<size_t>(grp) * 2 * dpad, *rot = res + dpad;
          for (int j = gt; j < d; j += kFourGroup) res[j] = __fsub_rn(qv[j], cent[j]);
          named_sync(1 + grp, kFourGroup);
          for (int r = gt; r < d; r += kFourGroup) {
            float s = 0.0f;
            for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(p.rot_t[static_cast<size_t>(j) * d + r], res[j]));
            rot[r] = s;
          }
          named_sync(1 + grp, kFourGroup);
          rres = rot;
        }
        float lmin = __int_as_float(0x7f800000), lmax = -__int_as_float(0x7f800000);
        for (int e = gt; e < nent; e += kFourGroup) {
          const int m = e >> 4;
          const float *cw = cbs + static_cast<size_t>(e) * dsub;
          // residual r_j = q_j - c_j (or its rotation), then sum_j (r_j - cw_j)^2 in j order
          float rj = rres ? rres[m * dsub] : __fsub_rn(qv[m * dsub], cent[m * dsub]);
          float diff = __fsub_rn(rj, cw[0]);
          float acc = __fmul_rn(diff, diff);
          for (int j = 1; j < dsub; ++j) {
            rj = rres ? rres[m * dsub + j] : __fsub_rn(qv[m * dsub + j], cent[m * dsub + j]);
            diff = __fsub_rn(rj, cw[j]);
            acc = __fadd_rn(acc, __fmul_rn(diff, diff));
          }
          fl[e] = acc;
          // global min/max of the table (pq_simd.rs:587-598); fminf/fmaxf
          // skip NaNs as the reference's `<` / `>` comparisons do
          lmin = fminf(lmin, acc);
          lmax = fmaxf(lmax, acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          lmin = fminf(lmin, __shfl_xor_sync(VG_FULL_MASK, lmin, off));
          lmax = fmaxf(lmax, __shfl_xor_sync(VG_FULL_MASK, lmax, off));
        }
        if (lane == 0) {
          s_rmin[grp][gt >> 5] = lmin;
          s_rmax[grp][gt >> 5] = lmax;
        }
        named_sync(1 + grp, kFourGroup);
        float gmin = s_rmin[grp][0], gmax = s_rmax[grp][0];
#pragma unroll
        for (int w = 1; w < kFourGroup / 32; ++w) {
          gmin = fminf(gmin, s_rmin[grp][w]);
          gmax = fmaxf(gmax, s_rmax[grp][w]);
        }
        const float range = __fsub_rn(gmax, gmin);
        const bool flat = range < FLT_EPSILON;
        const float inv = flat ? 0.0f : __fdiv_rn(255.0f, range);
        uint8_t *ql = qset + static_cast<size_t>(grp) * qstride;
        for (int e = gt; e < nent; e += kFourGroup) {
          // round half away from zero, clamp; NaN -> 0 (pq_simd.rs:607-609)
          float t = roundf(__fmul_rn(__fsub_rn(fl[e], gmin), inv));
          t = fminf(fmaxf(t, 0.0f), 255.0f);
          ql[e] = static_cast<uint8_t>(t);
        }
        if (gt == 0) {
          const float scale = flat ? 1.0f : __fdiv_rn(range, 255.0f);
          s_scale[set][grp] = scale;
          s_fbase[set][grp] = __fmul_rn(gmin, static_cast<float>(M));
          // List pruning.  s_lb bounds every float-table sum from below; a
          // quantised entry is its float value minus at most scale / 2 (round
          // to nearest, pq_simd.rs:607-609), up to a few more roundings in
          // (v - min) * (255 / range), the sum's scale and + min * M.  So every
          // quantised distance is >= lb (1 - 16 u) - M scale / 2 (1 + 1e-5) for
          // lists of >= 16 vectors, and >= lb for the smaller float-path lists.
          const uint64_t bnd = s_bound;
          double lbq = static_cast<double>(s_lb[bat[grp]]);
          if (s_len[bat[grp]] >= 16)
            lbq = lbq * (1.0 - 16 * 5.9604644775390625e-8) - 0.5 * M * static_cast<double>(scale) * (1.0 + 1e-5);
          s_skip[set][grp] = bnd != kEmptyKey && lbq > static_cast<double>(key_dist(bnd));
        }
      }
      if (tid == 0) form(b + 1);  // built next, while slower warps still score this batch
      __syncthreads();

      // ---- score and select ---------------------------------------------
      // candidates of the batch's lists that are not skipped
      const uint8_t *skip = s_skip[set];
      const uint32_t pre1 = skip[0] ? 0u : s_len[bat[0]];
      const uint32_t pre2 = pre1 + (nb > 1 && !skip[1] ? s_len[bat[1]] : 0u);
      const uint32_t pre3 = pre2 + (nb > 2 && !skip[2] ? s_len[bat[2]] : 0u);
      const uint32_t pre4 = pre3 + (nb > 3 && !skip[3] ? s_len[bat[3]] : 0u);
      const uint32_t qset_a = smem_u32(qset);
      for (uint32_t x0 = warp * 32; x0 < pre4; x0 += kScanThreads) {
        const uint32_t x = x0 + lane;
        // threshold first: candidates whose partial sum already exceeds it stop
        // early (the quantised distance is non-decreasing in the integer sum)
        uint64_t thr = tk.worst();
        const uint64_t bound = s_bound;
        thr = bound < thr ? bound : thr;
        const uint32_t tkey = static_cast<uint32_t>(thr >> 32);
        float dist = 0.0f;
        int g = 0;
        uint32_t c = 0;
        bool alive = x < pre4, quant = false;
        const uint8_t *vp = p.packed;
        uint32_t list = 0;
        if (alive) {
          g = (x >= pre1) + (x >= pre2) + (x >= pre3);
          const uint32_t lo = g == 0 ? 0u : g == 1 ? pre1 : g == 2 ? pre2 : pre3;
          const uint32_t hi = g == 0 ? pre1 : g == 1 ? pre2 : g == 2 ? pre3 : pre4;
          c = x - lo;
          list = s_list[bat[g]];
          quant = hi - lo >= 16;  // search.rs:1261 (SIMD_BATCH_THRESHOLD)
          if (quant) vp = p.packed + p.pack_off[list] + static_cast<uint64_t>(c) * ((M + 1) >> 1);
        }
        // quantised lists: integer sums of the u8 table, checked every 16 codes
        const float sc = s_scale[set][g], fb = s_fbase[set][g];
        bool qlive = alive && quant;
        uint32_t acc = 0;
        if ((M & 15) == 0) {
          const uint32_t qa = qset_a + static_cast<uint32_t>(g * qstride);
          for (int m0 = 0; m0 < M; m0 += 64) {
            if (!__any_sync(VG_FULL_MASK, qlive)) break;
            uint2 w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              w[u] = (qlive && m0 + 16 * u < M) ? *reinterpret_cast<const uint2 *>(vp + (m0 >> 1) + 8 * u)
                                                : make_uint2(0u, 0u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (m0 + 16 * u >= M) break;
              if (u > 0 && !__any_sync(VG_FULL_MASK, qlive)) break;
              if (qlive) {
                acc += nibble_sum16(w[u], qa + static_cast<uint32_t>((m0 + 16 * u) * 16));
                qlive = order_key(__fadd_rn(__fmul_rn(__uint2float_rn(acc), sc), fb)) <= tkey;
              }
            }
          }
        } else if (qlive) {
          const uint8_t *ql = qset + static_cast<size_t>(g) * qstride;
          for (int m = 0; m < M; ++m) acc += ql[m * 16 + ((vp[m >> 1] >> ((m & 1) * 4)) & 15u)];
        }
        if (quant) {
          alive = qlive;
          dist = __fadd_rn(__fmul_rn(__uint2float_rn(acc), sc), fb);
        } else if (alive) {  // lists under 16 vectors: float table, sequential sum
          const uint8_t *cp = p.list_codes + p.code_off[list] + static_cast<uint64_t>(c) * M;
          dist = adc_row_sum<16>(cp, fset + static_cast<size_t>(g) * fstride, M, 16);
        }
        const uint32_t dk = order_key(dist);
        const bool pass = alive && dk <= tkey;
        unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
        if (!mask) continue;
        uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | p.list_ids[s_lbeg[bat[g]] + c]) : kEmptyKey;
        if (p.key_floor && key <= p.key_floor[q]) key = kEmptyKey;  // selected by an earlier pass
        if (__popc(mask) > 4) {
          tk.add(key < thr ? key : kEmptyKey);
        } else {
          while (mask) {
            const int src = __ffs(mask) - 1;
            mask &= mask - 1;
            const uint64_t kx = shfl64(key, src);
            if (kx < thr) topk_insert_one(tk, kx);
          }
        }
        const uint64_t kth = tk.get(k - 1);
        if (lane == 0 && kth < bound) atomicMin(&s_bound, kth);
      }
      // no barrier here: the next batch writes the other table set, and the
      // one after waits behind the next batch's barrier
    }
    __syncthreads();  // all scans done before the warp lists are exchanged

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

}  // namespace vg
