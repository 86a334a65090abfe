// Direct-ADC search kernel for 8-bit codes: one warp per query, no tables.
//
// The reference scores a candidate by summing, over subspaces in order, the
// entry of its code in a per-(query, list) table, each entry being the
// sequential f32 sum sum_j (r_j - w_j)^2 over the subvector
// (search.rs:1175-1391, pq.rs:19-21).  This kernel evaluates exactly those
// entries, in the same order and with the same roundings, for the codes a
// candidate actually has, reading the codewords from a shared-memory copy of
// the codebook -- so it returns the same ids and distances without building a
// table.  What that buys:
//   - a candidate whose partial sum passes the query's k-th distance stops
//     (entries are >= +0 and a rounded add never decreases the sum; checked
//     every 4 subspaces), and the entries it never reaches are never computed;
//   - each warp owns its query: it walks the probes in order, skips a list
//     whose distance lower bound exceeds its current k-th distance (list
//     pruning with the freshest bound), keeps the top-k in registers and
//     writes the result -- no block barrier, no merge.
// Queries are handed out to warps by an atomic counter.
#pragma once

#include "scan_kernel.cuh"
#include "scan_work.cuh"

namespace vg {

constexpr int kDirectThreads = 1024;
constexpr int kDirectWarps = kDirectThreads / 32;

// codeword / subvector stride in shared memory: DSUB rounded up to 1, 2, 4 or 8
__host__ __device__ constexpr int direct_pad(int dsub) { return dsub <= 1 ? 1 : dsub <= 2 ? 2 : dsub <= 4 ? 4 : 8; }

__host__ __device__ inline size_t direct_smem_bytes(int M, int dsub) {
  const size_t dp = static_cast<size_t>(direct_pad(dsub));
  return static_cast<size_t>(M) * 256 * dp * 4 + static_cast<size_t>(kDirectWarps) * M * dp * 4;
}

__device__ __forceinline__ void prefetch_codes(const void *a) { asm volatile("prefetch.global.L1 [%0];" ::"l"(a)); }

template <int DP>
__device__ __forceinline__ void lds_vec(const float *a, float (&v)[DP]) {
  if constexpr (DP == 8) {
    const float4 x = *reinterpret_cast<const float4 *>(a), y = *reinterpret_cast<const float4 *>(a + 4);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
  } else if constexpr (DP == 4) {
    const float4 x = *reinterpret_cast<const float4 *>(a);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  } else if constexpr (DP == 2) {
    const float2 x = *reinterpret_cast<const float2 *>(a);
    v[0] = x.x; v[1] = x.y;
  } else {
    v[0] = a[0];
  }
}

// Table entry (m, code) of the residual in rb: sum_j (r_j - w_j)^2 in j
// order, the first square taken as is (as sq_dist computes it).
template <int DSUB, int DP>
__device__ __forceinline__ float direct_entry(const float *rb, const float *cbk, int m, uint32_t code) {
  float r[DP], w[DP];
  lds_vec<DP>(rb + m * DP, r);
  lds_vec<DP>(cbk + (static_cast<size_t>(m) * 256 + code) * DP, w);
  const float d0 = __fsub_rn(r[0], w[0]);
  float t = __fmul_rn(d0, d0);
#pragma unroll
  for (int j = 1; j < DSUB; ++j) {
    const float dj = __fsub_rn(r[j], w[j]);
    t = __fadd_rn(t, __fmul_rn(dj, dj));
  }
  return t;
}

// Sum over subspaces of the candidate's entries, stopping (alive = false) once
// the partial sum's key exceeds tkey; every lane of the warp calls it.
template <int DSUB, int DP>
__device__ __forceinline__ float direct_row_sum(const uint8_t *cp, const float *cbk, const float *rb, int M,
                                                uint32_t tkey, bool &alive) {
  float acc = 0.0f;
  if ((M & 15) == 0) {
    uint4 wn = alive ? *reinterpret_cast<const uint4 *>(cp) : make_uint4(0u, 0u, 0u, 0u);
    for (int m0 = 0; m0 < M; m0 += 16) {
      if (!__any_sync(VG_FULL_MASK, alive)) break;
      const uint4 w = wn;
      if (alive && m0 + 16 < M) wn = *reinterpret_cast<const uint4 *>(cp + m0 + 16);
      if (alive) {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        // four codes (one word) at a time, the bound checked after each word
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (alive) {
#pragma unroll
            for (int b = 0; b < 4; ++b)
              acc = __fadd_rn(acc, direct_entry<DSUB, DP>(rb, cbk, m0 + 4 * g + b, __byte_perm(ws[g], 0u, 0x4440u + b)));
            alive = order_key(acc) <= tkey;
          }
        }
      }
    }
  } else if (alive) {
    for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, direct_entry<DSUB, DP>(rb, cbk, m, cp[m]));
    alive = order_key(acc) <= tkey;
  }
  return acc;
}

template <int DSUB, int R>
__global__ void __launch_bounds__(kDirectThreads, 1) ivfpq_direct_kernel(const ScanParams p) {
  constexpr int DP = direct_pad(DSUB);
  extern __shared__ __align__(16) float dsm[];
  const int M = p.M, d = p.d, P = p.P, k = p.k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *cbk = dsm;                                                                // [M][256][DP]
  float *rb = dsm + static_cast<size_t>(M) * 256 * DP + static_cast<size_t>(warp) * M * DP;  // [M][DP]

  for (int i = tid; i < M * 256 * DP; i += kDirectThreads) {
    const int e = i / DP, j = i - e * DP;
    cbk[i] = j < DSUB ? p.codebooks[static_cast<size_t>(e) * DSUB + j] : 0.0f;
  }
  for (int i = lane; i < M * DP; i += 32) rb[i] = 0.0f;  // padding lanes of the residual stay 0
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
    uint32_t n_lists = 0, n_vecs = 0;  // scored after pruning (profiling)
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
    const bool seed = p.seed_next != nullptr;
    int seed_stop = P;
    bool stopped = false;
    // a seed pass scores only queries whose nearest list is this rank's (the
    // records of other ranks' lists hold no list)
    if (seed && p.probe_rec[static_cast<size_t>(q) * P].list == 0xffffffffu) {
      seed_stop = 1;
      first = last;
    }
    // probe records in groups of 32, in order: lane i loads record c0 + i so
    // the warp walks only the live ones with no global load on its serial
    // path; a list the group's starting bound prunes stays pruned (the bound
    // only tightens)
    for (int c0 = first; c0 < last; c0 += 32) {
      if (stopped) break;
      if (seed && tk.get(k - 1) != kEmptyKey) {
        seed_stop = c0;
        break;
      }
      ProbeRec rec_l{0xffffffffu, 0u, 0ull, 0ull, 0.0f, 0u};
      if (c0 + lane < last) rec_l = p.probe_rec[static_cast<size_t>(q) * P + c0 + lane];
      const uint64_t kth_g = min(tk.get(k - 1), kth0);
      const bool pruned0 = kth_g != kEmptyKey && rec_l.lb > key_dist(kth_g);
      unsigned todo = __ballot_sync(VG_FULL_MASK, rec_l.list != 0xffffffffu && rec_l.len > 0 && !pruned0);
      while (todo) {
        const int pj = __ffs(todo) - 1;
        todo &= todo - 1;
        if (seed && tk.get(k - 1) != kEmptyKey) {
          seed_stop = c0 + pj;
          stopped = true;
          break;
        }
        ProbeRec rec;
        rec.list = __shfl_sync(VG_FULL_MASK, rec_l.list, pj);
        rec.len = __shfl_sync(VG_FULL_MASK, rec_l.len, pj);
        rec.lbeg = shfl64(rec_l.lbeg, pj);
        rec.coff = shfl64(rec_l.coff, pj);
        rec.lb = __shfl_sync(VG_FULL_MASK, rec_l.lb, pj);
        uint64_t kth = min(tk.get(k - 1), kth0);
        if (kth != kEmptyKey && rec.lb > key_dist(kth)) continue;  // list pruning
        const float *cent = p.centroids + static_cast<size_t>(rec.list) * d;
        const uint8_t *lcodes = p.list_codes + rec.coff;
        if (static_cast<uint32_t>(lane) < rec.len) prefetch_codes(lcodes + static_cast<uint64_t>(lane) * M);
        __syncwarp();
        for (int j = lane; j < d; j += 32) rb[(j / DSUB) * DP + j % DSUB] = __fsub_rn(qv[j], cent[j]);
        __syncwarp();
        ++n_lists;
        n_vecs += rec.len;
        for (uint32_t x0 = 0; x0 < rec.len; x0 += 32) {
          const uint32_t c = x0 + lane;
          bool alive = c < rec.len;
          if (c + 32 < rec.len) prefetch_codes(lcodes + static_cast<uint64_t>(c + 32) * M);  // next chunk
          const uint32_t tkey = static_cast<uint32_t>(kth >> 32);
          const uint8_t *cp = lcodes + static_cast<uint64_t>(alive ? c : 0u) * M;
          const float dist = direct_row_sum<DSUB, DP>(cp, cbk, rb, M, tkey, alive);
          const uint32_t dk = order_key(dist);
          const bool pass = alive && dk <= tkey;
          unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
          if (!mask) continue;
          const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | p.list_ids[rec.lbeg + c]) : kEmptyKey;
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
    }
  }
}

template <int DSUB, int R>
cudaError_t launch_direct_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_direct_kernel<DSUB, R>;
  if (!p.probe_rec || p.ks != 256) return cudaErrorInvalidValue;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t smem = direct_smem_bytes(p.M, DSUB);
  if (smem + 1024 > static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  // one block per SM (queries spread over every SM even when there are fewer
  // than a warp's worth per SM)
  int grid = num_sms < p.nq ? num_sms : p.nq;
  if (grid < 1) grid = 1;
  ScanParams pp = p;
  pp.neg_zero = -0.0f;
  kern<<<grid, kDirectThreads, smem, s>>>(pp);
  return cudaGetLastError();
}

}  // namespace vg
