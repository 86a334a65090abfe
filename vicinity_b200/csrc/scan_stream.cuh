// Query-stream variant of the double-buffered 8-bit search kernel (same
// computation and results as ivfpq_pipe_kernel / ivfpq_query_kernel,
// search.rs:1175-1391).
//
// The double-buffered kernel pipelines table building against scoring
// within one query, but every query still begins with an unhidden table
// build and with a chain of dependent loads for its probe metadata, and ends
// with a phase that builds nothing.  Here batches form one stream across
// the queries a block takes:
//   - phase n scores batch n and builds the tables of batch n + 1, whichever
//     query each belongs to, so the first tables of the next query are built
//     while the last lists of the current one are scored;
//   - a query's probe records (list, length, offsets, pruning bound; one
//     32-byte record per probe, written by the bound kernel) are copied into
//     shared memory with cp.async one phase and waited for the next, several
//     phases before the query's first batch is formed;
//   - thread 0 forms batch n + 2 before the phase barrier from the oldest
//     query with lists left, skipping lists whose bound exceeds that query's
//     k-th distance (list pruning), and fetches the next query index;
//   - after the barrier of the phase that scored a query's last batch, the
//     warps merge their lists and warp 0 writes the results.
// Query slots form a ring: fetched, copied and consumed in order, so a slot
// is free again once its query has been written.
#pragma once

#include "f32x2.cuh"
#include "pipeline.cuh"
#include "scan_kernel.cuh"

namespace vg {

// Shared memory of the per-warp top-k rows and two sets of `batch` tables.
__host__ __device__ inline size_t pipe_smem_bytes(int d, int M, int ks, int batch, int R) {
  const size_t table = static_cast<size_t>((M * ks + 3) & ~3) * 4;
  (void)d;
  return static_cast<size_t>(kScanWarps) * 32 * R * 8 + 2 * static_cast<size_t>(batch) * table;
}

// D floats of row `a` minus row `b` at offset o, each an IEEE subtraction.
template <int D>
__device__ __forceinline__ void load_residual(const float *a, const float *b, int o, bool vec4, float (&r)[D]) {
  if (D % 4 == 0 && vec4) {
#pragma unroll
    for (int j = 0; j < D; j += 4) {
      const float4 x = *reinterpret_cast<const float4 *>(a + o + j);
      const float4 y = *reinterpret_cast<const float4 *>(b + o + j);
      r[j] = __fsub_rn(x.x, y.x);
      r[j + 1] = __fsub_rn(x.y, y.y);
      r[j + 2] = __fsub_rn(x.z, y.z);
      r[j + 3] = __fsub_rn(x.w, y.w);
    }
  } else {
#pragma unroll
    for (int j = 0; j < D; ++j) r[j] = __fsub_rn(a[o + j], b[o + j]);
  }
}

constexpr int kStreamSlots = 8;  // query slots (records in shared memory)
constexpr int kStreamMaxP = 256;  // two 16-byte copies per record, one per thread
constexpr int kStreamAhead = 2;   // queries fetched ahead of the one being formed

__host__ __device__ inline size_t stream_smem_bytes(int M, int ks, int batch, int R, int P, int nslots) {
  return pipe_smem_bytes(0, M, ks, batch, R) + static_cast<size_t>(nslots) * P * sizeof(ProbeRec);
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int DSUB, int GPT, int R, int KS>
__global__ void __launch_bounds__(kScanThreads, 1)
    ivfpq_stream_kernel(const ScanParams p, const int batch, const int nslots) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, d = p.d, P = p.P, k = p.k;
  constexpr int ks = KS;
  const int nent = M * ks;
  const int tstride = (nent + 3) & ~3;
  const bool vec4 = (d & 3) == 0;
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(smem);                  // [warps][32R]
  float *tables = reinterpret_cast<float *>(wl + kScanWarps * 32 * R);                     // [2][batch][tstride]
  ProbeRec *recs = reinterpret_cast<ProbeRec *>(tables + 2 * static_cast<size_t>(batch) * tstride);  // [slots][P]

  __shared__ uint32_t s_q[kStreamSlots];
  __shared__ int s_state[kStreamSlots];   // 0 free, 1 records loading, 2 forming / scoring
  __shared__ int s_ready[kStreamSlots];   // first phase whose batch formation may read the records
  __shared__ int s_cursor[kStreamSlots];  // next probe position to consider
  __shared__ int s_formed[kStreamSlots];  // batches formed
  __shared__ unsigned long long s_bound[kStreamSlots];
  __shared__ uint16_t s_bat[3][kMaxBatch];  // probe positions of batch j (ring j % 3)
  __shared__ int s_bn[3], s_bs[3];          // lists and query slot (-1: no batch) of batch j
  // bookkeeping of warp 0 (written by its lane 0)
  __shared__ int s_form, s_next_form, s_fetch, s_exhausted, s_waiting, s_unformed;
  // read by every thread at the top of phase n, written by thread 0 at the end of
  // phase n - 1: indexed by phase parity so that a late reader never sees the
  // next phase's value
  __shared__ int s_copy[2], s_wait[2], s_stop[2];
  __shared__ uint32_t s_chunk[2];  // next 32-candidate chunk of the phase's batch

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool build_first = (warp & 1) == 0;

  const int ngroups = nent >> 2;
  const f32x2 nz = f2_pack(p.neg_zero, p.neg_zero);
  f32x2 cb[GPT][2][DSUB];
#pragma unroll
  for (int i = 0; i < GPT; ++i) {
    const int G = tid + i * kScanThreads;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < DSUB; ++j) {
        const size_t e = static_cast<size_t>(4 * G + 2 * h);
        cb[i][h][j] = G < ngroups ? f2_pack(p.codebooks[e * DSUB + j], p.codebooks[(e + 1) * DSUB + j]) : 0ull;
      }
  }

  if (tid == 0) {
    for (int s = 0; s < kStreamSlots; ++s) s_state[s] = 0;
    for (int j = 0; j < 3; ++j) {
      s_bn[j] = 0;
      s_bs[j] = -1;
    }
    s_form = -1;
    s_next_form = 0;
    s_fetch = 0;
    s_copy[0] = -1;
    s_wait[0] = -1;
    s_exhausted = 0;
    s_waiting = 0;
    s_unformed = 0;
    s_stop[0] = 0;
    s_chunk[0] = 0;
  }
  WarpTopK<R> tk;
  tk.init();

  // Batch j (warp 0, before a barrier; `n` the current phase): the next
  // lists of the forming query whose bound does not exceed its k-th distance,
  // 32 probe positions per ballot; when that query has none left, the next
  // query whose records are in.  A query without any list gets one empty
  // batch so that it is still written.
  auto form = [&](int j, int n) {
    int cnt = 0, slot = -1;
    for (;;) {
      int F = s_form;
      if (F < 0) {
        const int c = s_next_form;
        if (s_state[c] != 1 || s_ready[c] > n) break;
        F = c;
        __syncwarp();
        if (lane == 0) {
          s_state[F] = 2;
          s_form = F;
          s_next_form = (c + 1) % nslots;
          --s_waiting;
        }
      }
      const uint64_t bnd = s_bound[F];
      const float bdist = key_dist(bnd);
      const ProbeRec *r = recs + static_cast<size_t>(F) * P;
      int c0 = s_cursor[F];
      // a query's first batches are formed before its earlier ones have been
      // scored (no bound yet, nothing pruned): batch j of a query holds at
      // most j + 1 lists, so pruning starts after its nearest list
      const int cap = min(batch, s_formed[F] + 1);
      while (c0 < P && cnt < cap) {
        const int pos = c0 + lane;
        const bool ok = pos < P && r[pos].list != 0xffffffffu && !(bnd != kEmptyKey && r[pos].lb > bdist);
        const unsigned m = __ballot_sync(VG_FULL_MASK, ok);
        const int avail = __popc(m), take = min(avail, cap - cnt);
        const int rank = __popc(m & ((1u << lane) - 1u));
        if (ok && rank < take) s_bat[j % 3][cnt + rank] = static_cast<uint16_t>(pos);
        if (take < avail) {  // batch full: resume after the last list taken
          const unsigned lm = __ballot_sync(VG_FULL_MASK, ok && rank == take - 1);
          c0 = __shfl_sync(VG_FULL_MASK, pos, __ffs(lm) - 1) + 1;
        } else {
          c0 = min(c0 + 32, P);
        }
        cnt += take;
      }
      const bool done = c0 >= P;
      const bool take_batch = cnt > 0 || (done && s_formed[F] == 0);
      __syncwarp();
      if (lane == 0) {
        s_cursor[F] = c0;
        if (done) {
          s_form = -1;
          --s_unformed;
        }
        if (take_batch) ++s_formed[F];
      }
      __syncwarp();
      if (take_batch) {
        slot = F;
        break;
      }
      // the rest of the query was pruned: on to the next query
    }
    if (lane == 0) {
      s_bn[j % 3] = cnt;
      s_bs[j % 3] = slot;
    }
  };

  // tables of batch j into table set `set`
  auto build = [&](int j, int set) {
    const int nb = s_bn[j % 3];
    const int slot = s_bs[j % 3];
    const float *qv = p.qn + static_cast<size_t>(s_q[slot]) * d;
    const ProbeRec *r = recs + static_cast<size_t>(slot) * P;
    float *tset = tables + static_cast<size_t>(set) * batch * tstride;
#pragma unroll 1
    for (int g = 0; g < nb; ++g) {
      const float *cent = p.centroids + static_cast<size_t>(r[s_bat[j % 3][g]].list) * d;
      float *lg = tset + static_cast<size_t>(g) * tstride;
#pragma unroll
      for (int i = 0; i < GPT; ++i) {
        const int G = tid + i * kScanThreads;
        if (G < ngroups) {
          float qs[DSUB];
          load_residual<DSUB>(qv, cent, ((4 * G) / ks) * DSUB, vec4, qs);
          f32x2 qq[DSUB];
#pragma unroll
          for (int jj = 0; jj < DSUB; ++jj) qq[jj] = f2_pack(qs[jj], qs[jj]);
          const float2 e01 = f2_unpack(sq_dist_x2<DSUB>(qq, cb[i][0], nz));
          const float2 e23 = f2_unpack(sq_dist_x2<DSUB>(qq, cb[i][1], nz));
          *reinterpret_cast<float4 *>(lg + 4 * G) = make_float4(e01.x, e01.y, e23.x, e23.y);
        }
      }
    }
  };
  // score and select the candidates of batch j (query slot S) against table set `set`
  auto scan = [&](int j, int set, int S) {
    const int nb = s_bn[j % 3];
    const uint16_t *bat = s_bat[j % 3];
    const ProbeRec *r = recs + static_cast<size_t>(S) * P;
    const float *tset = tables + static_cast<size_t>(set) * batch * tstride;
    const uint32_t pre1 = r[bat[0]].len;
    const uint32_t pre2 = pre1 + (nb > 1 ? r[bat[1]].len : 0u);
    const uint32_t pre3 = pre2 + (nb > 2 ? r[bat[2]].len : 0u);
    const uint32_t pre4 = pre3 + (nb > 3 ? r[bat[3]].len : 0u);
    // chunks of 32 candidates are handed out in order as warps come free, so
    // warps that built first take fewer and the phase ends together
    for (;;) {
      uint32_t chunk = 0;
      if (lane == 0) chunk = atomicAdd(&s_chunk[j & 1], 1u);
      const uint32_t x0 = __shfl_sync(VG_FULL_MASK, chunk, 0) * 32u;
      if (x0 >= pre4) break;
      const uint32_t x = x0 + lane;
      uint64_t thr = tk.worst();
      const uint64_t bound = s_bound[S];
      thr = bound < thr ? bound : thr;
      const uint32_t tkey = static_cast<uint32_t>(thr >> 32);
      int g = 0;
      uint32_t c = 0;
      bool alive = x < pre4;
      const uint8_t *cp = p.list_codes;
      const float *lg = tset;
      if (alive) {
        g = (x >= pre1) + (x >= pre2) + (x >= pre3);
        c = x - (g == 0 ? 0u : g == 1 ? pre1 : g == 2 ? pre2 : pre3);
        cp = p.list_codes + r[bat[g]].coff + static_cast<uint64_t>(c) * M;
        lg = tset + static_cast<size_t>(g) * tstride;
      }
      const float dist = adc_row_sum_bounded<KS>(cp, lg, M, ks, tkey, alive);
      const uint32_t dk = order_key(dist);
      const bool pass = alive && dk <= tkey;
      unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
      if (!mask) continue;
      const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | p.list_ids[r[bat[g]].lbeg + c]) : kEmptyKey;
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
      if (lane == 0 && kth < bound) atomicMin(&s_bound[S], kth);
    }
  };

  bool fetch_go = true;  // thread 0: fetch a query index at the start of the phase
  uint32_t fetch_q = 0;
  __syncthreads();
  for (int n = 0;; ++n) {
    if (s_stop[n & 1]) break;
    const int cur = n % 3, nxt = (n + 1) % 3;
    const int S = s_bs[cur], Sn = s_bs[nxt];
    const int set = n & 1;
    const bool has_scan = S >= 0 && s_bn[cur] > 0;
    const bool has_build = Sn >= 0 && s_bn[nxt] > 0;

    // probe records: the copy issued last phase completes (visible after this
    // phase's barrier), then the copy of a newly fetched query is issued
    const int wslot = s_wait[n & 1], cslot = s_copy[n & 1];
    if (tid == 0 && fetch_go) fetch_q = atomicAdd(p.counter, 1u);
    if (tid < 2 * P) {
      if (wslot >= 0) cp_async_wait_all();
      if (cslot >= 0) {
        const unsigned char *src = reinterpret_cast<const unsigned char *>(p.probe_rec + static_cast<size_t>(s_q[cslot]) * P);
        cp_async16(reinterpret_cast<unsigned char *>(recs + static_cast<size_t>(cslot) * P) + 16 * tid, src + 16 * tid);
        cp_async_commit();
      }
    }

    if (build_first) {
      if (has_build) build(n + 1, set ^ 1);
      if (has_scan) scan(n, set, S);
    } else {
      if (has_scan) scan(n, set, S);
      if (has_build) build(n + 1, set ^ 1);
    }

    if (warp == 0) {
      int ncopy = -1;
      if (lane == 0) {
        if (wslot >= 0) s_ready[wslot] = n + 1;
        if (fetch_go) {  // the query index fetched at the start of this phase
          fetch_go = false;
          const int f = s_fetch;
          if (fetch_q < static_cast<uint32_t>(p.nq)) {
            s_q[f] = fetch_q;
            s_state[f] = 1;
            s_ready[f] = 0x7fffffff;
            s_cursor[f] = 0;
            s_formed[f] = 0;
            s_bound[f] = kEmptyKey;
            ++s_waiting;
            ++s_unformed;
            ncopy = f;
            s_fetch = (f + 1) % nslots;
          } else {
            s_exhausted = 1;
          }
        }
        s_copy[(n + 1) & 1] = ncopy;
        s_wait[(n + 1) & 1] = cslot;
        s_chunk[(n + 1) & 1] = 0;
      }
      __syncwarp();
      form(n + 2, n);
      __syncwarp();
      if (lane == 0) {
        // fetch at the start of the next phase (the atomic's latency hides
        // behind that phase's work) when a slot is free and fewer than
        // kStreamAhead queries wait for their first batch: a deeper queue
        // only holds queries back from blocks that finish early
        fetch_go = !s_exhausted && s_state[s_fetch] == 0 && s_waiting < kStreamAhead;
        const bool pending = fetch_go || ncopy >= 0 || cslot >= 0 || s_waiting > 0 || s_unformed > 0 ||
                             s_bs[(n + 1) % 3] >= 0 || s_bs[(n + 2) % 3] >= 0;
        s_stop[(n + 1) & 1] = s_exhausted && !pending;
      }
    }
    __syncthreads();

    // the query of batch n is complete when batch n + 1 is not its own
    if (S >= 0 && s_bs[nxt] != S) {
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
        const uint32_t q = s_q[S];
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
        if (lane == 0) s_state[S] = 0;
      }
      tk.init();
    }
  }
}

template <int DSUB, int GPT, int R, int KS>
cudaError_t launch_stream_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_stream_kernel<DSUB, GPT, R, KS>;
  if (!p.probe_rec || p.P < 1 || p.P > kStreamMaxP) return cudaErrorInvalidValue;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t reserve = 4096;  // static shared memory of the kernel (< 1 KB) and slack
  int batch = kMaxBatch, nslots = kStreamSlots;
  while (stream_smem_bytes(p.M, KS, batch, R, p.P, nslots) + reserve > static_cast<size_t>(optin)) {
    if (nslots > 6) {
      --nslots;
    } else if (batch > 1) {
      --batch;
      nslots = kStreamSlots;
    } else {
      return cudaErrorInvalidConfiguration;
    }
  }
  const size_t smem = stream_smem_bytes(p.M, KS, batch, R, p.P, nslots);
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int grid = num_sms * per_sm;
  if (grid > p.nq) grid = p.nq;
  ScanParams pp = p;
  pp.neg_zero = -0.0f;
  kern<<<grid, kScanThreads, smem, s>>>(pp, batch, nslots);
  return cudaGetLastError();
}

}  // namespace vg
