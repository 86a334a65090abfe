// Warp-specialised IVF-PQ search kernel (8-bit codes, 256-entry codebooks).
//
// Same computation and results as ivfpq_query_kernel (scan_kernel.cuh) --
// per probed list: residual, ADC table (pq.rs:573-643), sequential table
// sums (pq_simd.rs:314-369), top-k by (distance, id) (search.rs:64-75) --
// but the two halves of the work run concurrently on different warps:
//
//   producers (warps 0-11, 384 threads) walk a query's probes nearest-first
//     and build one ADC table per list into a ring of kWsSlots shared-memory
//     slots.  Each producer keeps EPT codewords of the codebook in registers
//     for the whole kernel, so table building is pure FP32 work;
//   consumers (warps 12-15, 128 threads) take filled slots in order, score
//     the list's candidates against the slot's table (shared-memory lookups)
//     and keep per-warp top-k lists bounded by a per-query block bound, as in
//     the query-major kernel; at the last list of a query they merge and
//     write the result.
//
// Slots are handed over with mbarrier pairs: full[s] completes when all 384
// producers have arrived (table written) and the slot's bulk copy of the
// list's codes into shared memory (cp.async.bulk, issued when the slot is
// claimed, so it lands while the table is being built) has delivered its
// bytes; empty[s] completes when all 128 consumers have arrived (slot read).
// Producers also load the next list's centroid row before building the
// current table, so the residual of the next list is ready without a stall.
// One elected thread per role waits, bounded by kWaitCycles; the role then
// synchronises on its named barrier and leaves together if the wait failed,
// after recording an error code.
#pragma once

#include "pipeline.cuh"
#include "scan_kernel.cuh"

namespace vg {

constexpr int kWsProducerWarps = 12;
constexpr int kWsConsumerWarps = 4;
constexpr int kWsProducers = kWsProducerWarps * 32;
constexpr int kWsConsumers = kWsConsumerWarps * 32;
constexpr int kWsSlots = 4;
constexpr int kWsMaxProbes = kWsProducers;  // probes of one query fit the producer group
constexpr int kWsBarProducers = 1, kWsBarConsumers = 2;

enum : uint32_t { kItemLast = 1u, kItemTerminate = 2u, kItemEmpty = 4u };

struct WsItem {
  uint64_t lbeg;
  uint32_t query, list, len, flags, staged;  // staged: leading candidates whose codes are in the slot buffer
};

// Shared memory without the per-slot code buffers.
__host__ __device__ inline size_t ws_smem_fixed(int d, int M, int ks, int R) {
  size_t table = static_cast<size_t>((M * ks + 3) & ~3) * 4;
  size_t vec = static_cast<size_t>((d + 3) & ~3) * 4;
  return static_cast<size_t>(kWsSlots) * table + 3 * vec + static_cast<size_t>(kWsConsumerWarps) * 32 * R * 8;
}

template <int DSUB, int EPT, int R, int KS>
__global__ void __launch_bounds__(kScanThreads, 1) ivfpq_ws_kernel(const ScanParams p, const uint32_t code_cap) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, d = p.d, P = p.P, k = p.k;
  constexpr int ks = KS;
  const int nent = M * ks;
  const int tstride = (nent + 3) & ~3;
  const int dpad = (d + 3) & ~3;
  float *tables = reinterpret_cast<float *>(smem);                   // [slots][tstride]
  float *qbuf = tables + static_cast<size_t>(kWsSlots) * tstride;    // [2][dpad] residuals
  float *qvec = qbuf + 2 * dpad;                                     // [dpad] query
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(qvec + dpad);  // [cwarps][32R]
  uint8_t *codebuf = reinterpret_cast<uint8_t *>(wl + kWsConsumerWarps * 32 * R);  // [slots][code_cap]

  __shared__ __align__(8) uint64_t full[kWsSlots], empty[kWsSlots];
  __shared__ WsItem items[kWsSlots];
  __shared__ uint32_t p_list[kWsMaxProbes], p_len[kWsMaxProbes];
  __shared__ uint64_t p_beg[kWsMaxProbes];
  __shared__ int p_warp_count[kWsProducerWarps];
  __shared__ uint32_t p_query;
  __shared__ int p_abort, c_abort;
  __shared__ unsigned long long c_bound;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int s = 0; s < kWsSlots; ++s) {
      mbar_init(&full[s], kWsProducers);
      mbar_init(&empty[s], kWsConsumers);
    }
    p_abort = 0;
    c_abort = 0;
    c_bound = kEmptyKey;
  }
  __syncthreads();

  if (warp < kWsProducerWarps) {
    // =========================== producers ===============================
    const int ptid = tid;
    constexpr int kD = DSUB;
    float cb[EPT][kD];
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = ptid + i * kWsProducers;
#pragma unroll
      for (int j = 0; j < kD; ++j) cb[i][j] = e < nent ? p.codebooks[static_cast<size_t>(e) * kD + j] : 0.0f;
    }
    uint32_t t = 0;  // items produced
    // acquire the next slot; false when the wait failed (role leaves)
    auto acquire = [&](int &slot) -> bool {
      slot = static_cast<int>(t % kWsSlots);
      const uint32_t use = t / kWsSlots;
      if (ptid == 0 && !mbar_wait(&empty[slot], (use & 1u) ^ 1u)) {
        p_abort = 1;
        atomicExch(p.error, 1);
      }
      named_sync(kWsBarProducers, kWsProducers);
      return p_abort == 0;
    };
    for (;;) {
      if (ptid == 0) p_query = atomicAdd(p.counter, 1u);
      named_sync(kWsBarProducers, kWsProducers);
      const uint32_t q = p_query;
      if (q >= static_cast<uint32_t>(p.nq)) {
        int slot;
        if (!acquire(slot)) return;
        if (ptid == 0) items[slot] = WsItem{0, q, 0, 0, kItemTerminate, 0};
        mbar_arrive(&full[slot]);
        return;
      }
      // compact this query's valid, owned probes (nearest first)
      uint32_t l = 0xffffffffu;
      bool valid = false;
      if (ptid < P) {
        l = p.probes[static_cast<size_t>(q) * P + ptid];
        valid = l != 0xffffffffu && (!p.owner || p.owner[l]);
      }
      const unsigned vm = __ballot_sync(VG_FULL_MASK, valid);
      if (lane == 0) p_warp_count[warp] = __popc(vm);
      named_sync(kWsBarProducers, kWsProducers);
      int base = 0, total = 0;
      for (int w = 0; w < kWsProducerWarps; ++w) {
        const int c = p_warp_count[w];
        if (w < warp) base += c;
        total += c;
      }
      if (valid) {
        const int pos = base + __popc(vm & ((1u << lane) - 1u));
        const uint64_t b = p.list_off[l];
        p_list[pos] = l;
        p_beg[pos] = b;
        p_len[pos] = static_cast<uint32_t>(p.list_off[l + 1] - b);
      }
      named_sync(kWsBarProducers, kWsProducers);
      if (total == 0) {  // nothing to scan: the consumers still emit an empty row
        int slot;
        if (!acquire(slot)) return;
        if (ptid == 0) items[slot] = WsItem{0, q, 0, 0, kItemLast | kItemEmpty, 0};
        mbar_arrive(&full[slot]);
        ++t;
        continue;
      }
      for (int j = ptid; j < d; j += kWsProducers) qvec[j] = p.qn[static_cast<size_t>(q) * d + j];
      // residual of the first list (later ones are prefetched during the
      // previous table build)
      {
        const float *cv = p.centroids + static_cast<size_t>(p_list[0]) * d;
        named_sync(kWsBarProducers, kWsProducers);
        for (int j = ptid; j < d; j += kWsProducers) qbuf[(t & 1u) * dpad + j] = __fsub_rn(qvec[j], cv[j]);
      }
      for (int it = 0; it < total; ++it) {
        int slot;
        if (!acquire(slot)) return;  // also orders the residual writes above
        const uint32_t list = p_list[it];
        const uint32_t len = p_len[it];
        if (ptid == 0) {
          const uint32_t staged = min(len, code_cap / static_cast<uint32_t>(M));
          const uint32_t bytes = (staged * static_cast<uint32_t>(M) + 15u) & ~15u;
          items[slot] = WsItem{p_beg[it], q, list, len, it + 1 == total ? kItemLast : 0u, staged};
          if (bytes) {
            mbar_expect_tx(&full[slot], bytes);
            bulk_copy_g2s(codebuf + static_cast<size_t>(slot) * code_cap, p.list_codes + p.code_off[list], bytes,
                          &full[slot]);
          }
        }
        // start loading the next list's centroid row; consumed after the build
        const bool has_next = it + 1 < total;
        float next_c = 0.0f;
        if (has_next && ptid < d) next_c = p.centroids[static_cast<size_t>(p_list[it + 1]) * d + ptid];
        const float *qs_cur = qbuf + (t & 1u) * dpad;
        float *tab = tables + static_cast<size_t>(slot) * tstride;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
          const int e = ptid + i * kWsProducers;
          if (e < nent) {
            float qv2[kD];
            load_subvector<kD>(qs_cur + (e / ks) * kD, qv2);
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < kD; ++j) {
              const float diff = __fsub_rn(qv2[j], cb[i][j]);
              acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
            tab[e] = acc;
          }
        }
        for (int j = ptid + kWsProducers; has_next && j < d; j += kWsProducers)  // d > 384 only
          qbuf[((t + 1) & 1u) * dpad + j] =
              __fsub_rn(qvec[j], p.centroids[static_cast<size_t>(p_list[it + 1]) * d + j]);
        if (has_next && ptid < d) qbuf[((t + 1) & 1u) * dpad + ptid] = __fsub_rn(qvec[ptid], next_c);
        mbar_arrive(&full[slot]);
        ++t;
      }
    }
  } else {
    // =========================== consumers ===============================
    const int ctid = tid - kWsProducers;
    const int cwarp = warp - kWsProducerWarps;
    WarpTopK<R> tk;
    tk.init();
    for (uint32_t t = 0;; ++t) {
      const int slot = static_cast<int>(t % kWsSlots);
      const uint32_t use = t / kWsSlots;
      if (ctid == 0 && !mbar_wait(&full[slot], use & 1u)) {
        c_abort = 1;
        atomicExch(p.error, 2);
      }
      named_sync(kWsBarConsumers, kWsConsumers);
      if (c_abort) return;
      const WsItem item = items[slot];
      if (item.flags & kItemTerminate) return;
      if (!(item.flags & kItemEmpty)) {
        const float *tab = tables + static_cast<size_t>(slot) * tstride;
        const uint8_t *scodes = codebuf + static_cast<size_t>(slot) * code_cap;
        const uint8_t *gcodes = p.list_codes + p.code_off[item.list];
        const uint32_t *ids = p.list_ids + item.lbeg;
        for (uint32_t x0 = cwarp * 32; x0 < item.len; x0 += 2 * kWsConsumers) {
          // two candidates per thread: independent sequential sums
          const uint32_t xa = x0 + lane, xb = x0 + kWsConsumers + lane;
          float da = 0.0f, db = 0.0f;
          if (xa < item.len)
            da = adc_row_sum<KS>((xa < item.staged ? scodes : gcodes) + static_cast<size_t>(xa) * M, tab, M, ks);
          if (xb < item.len)
            db = adc_row_sum<KS>((xb < item.staged ? scodes : gcodes) + static_cast<size_t>(xb) * M, tab, M, ks);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t x = h ? xb : xa;
            const float dist = h ? db : da;
            uint64_t thr = tk.worst();
            const uint64_t bound = c_bound;
            thr = bound < thr ? bound : thr;
            const uint32_t dk = order_key(dist);
            const bool pass = x < item.len && dk <= static_cast<uint32_t>(thr >> 32);
            unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
            if (!mask) continue;
            const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | ids[x]) : kEmptyKey;
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
            if (lane == 0 && kth < bound) atomicMin(&c_bound, kth);
          }
        }
      }
      if (item.flags & kItemLast) {
#pragma unroll
        for (int r = 0; r < R; ++r) wl[cwarp * 32 * R + r * 32 + lane] = tk.v[r];
        named_sync(kWsBarConsumers, kWsConsumers);
        if (cwarp == 0) {
          for (int w = 1; w < kWsConsumerWarps; ++w) {
            const unsigned long long *other = wl + w * 32 * R;
            if (other[0] < tk.worst()) {
#pragma unroll
              for (int r = 0; r < R; ++r) tk.merge_sorted_row(other[r * 32 + lane]);
            }
          }
          uint32_t count = 0;
          const uint32_t q = item.query;
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
          if (lane == 0) c_bound = kEmptyKey;
        }
        tk.init();
      }
      mbar_arrive(&empty[slot]);
    }
  }
}

template <int DSUB, int EPT, int R, int KS>
cudaError_t launch_ws_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_ws_kernel<DSUB, EPT, R, KS>;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t fixed = ws_smem_fixed(p.d, p.M, KS, R);
  const size_t reserve = 8192;  // static shared memory of the kernel
  if (fixed + reserve >= static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
  size_t cap = (static_cast<size_t>(optin) - reserve - fixed) / kWsSlots;
  cap = cap > (64u << 10) ? (64u << 10) : cap;
  cap &= ~static_cast<size_t>(15);
  const size_t smem = fixed + kWsSlots * cap;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int grid = num_sms * per_sm;
  if (grid > p.nq) grid = p.nq;
  kern<<<grid, kScanThreads, smem, s>>>(p, static_cast<uint32_t>(cap));
  return cudaGetLastError();
}

}  // namespace vg
