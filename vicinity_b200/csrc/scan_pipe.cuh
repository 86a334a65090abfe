// Double-buffered variant of the fused IVF-PQ search kernel for 8-bit codes
// (same computation and results as ivfpq_query_kernel in scan_kernel.cuh).
//
// Building a list's ADC table is FP32-issue bound and scoring its codes is
// shared-memory bound; done one after the other they leave one of the two
// pipes idle.  This kernel keeps two sets of `batch` tables: in each phase
// every warp builds its share of the NEXT batch's tables and scores its share
// of the CURRENT batch's candidates, even warps in that order and odd warps
// in the other, so at any time half the warps feed the FP32 pipe and half the
// shared-memory pipe.  One block barrier per phase separates the sets.
//
// Batches are formed as the search goes: the next batch takes the next lists
// in probe order whose distance lower bound does not exceed the block's k-th
// distance (list pruning), so pruned lists cost neither a table, a scan nor a
// phase.  Table builders read their residual subvectors straight from the
// query and centroid rows (L1-resident), so no residual buffer has to be
// filled ahead of the batch.
#pragma once

#include "f32x2.cuh"
#include "scan_kernel.cuh"

namespace vg {

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

template <int DSUB, int GPT, int R, int KS>
__global__ void __launch_bounds__(kScanThreads, 1) ivfpq_pipe_kernel(const ScanParams p, const int batch) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, d = p.d, P = p.P, k = p.k;
  constexpr int ks = KS;
  const int nent = M * ks;
  const int tstride = (nent + 3) & ~3;
  const bool vec4 = (d & 3) == 0;  // rows 16-byte aligned: subvectors load as float4
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(smem);     // [warps][32R]
  float *tables = reinterpret_cast<float *>(wl + kScanWarps * 32 * R);        // [2][batch][tstride]

  __shared__ uint32_t s_query;
  __shared__ int s_nvalid;
  __shared__ int s_wcount[kScanWarps];
  __shared__ uint32_t s_list[kScanThreads], s_len[kScanThreads];
  __shared__ uint64_t s_lbeg[kScanThreads], s_coff[kScanThreads];
  __shared__ unsigned long long s_bound;
  __shared__ float s_lb[kScanThreads];           // distance lower bound of each compacted probe
  __shared__ uint16_t s_bat[3][kMaxBatch];       // probe positions of batch j (slot j % 3)
  __shared__ int s_bn[3];                        // lists in batch j (slot j % 3)
  __shared__ int s_cursor;                       // next probe position to consider

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool build_first = (warp & 1) == 0;

  // codewords of this thread's groups, lane-packed as entries (0,1), (2,3)
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
        s_coff[pos] = p.code_off[l];
        s_lb[pos] = p.probe_lb ? p.probe_lb[static_cast<size_t>(q) * P + tid] : 0.0f;
      }
      if (tid == 0) s_nvalid = total;
      __syncthreads();
    }
    const int nvalid = s_nvalid;

    // Batch j: the next `batch` lists from the cursor whose lower bound does
    // not exceed the block's k-th distance (a pruned list holds no candidate
    // that could enter the top-k).  Formed by thread 0 just before a block
    // barrier, read by every thread after it; slot j % 3 is rewritten only
    // after batch j has been built and scanned.
    auto form = [&](int j) {
      const uint64_t bnd = s_bound;
      const float bdist = key_dist(bnd);
      int n = 0, cur = s_cursor;
      for (; cur < nvalid && n < batch; ++cur)
        if (bnd == kEmptyKey || !(s_lb[cur] > bdist)) s_bat[j % 3][n++] = static_cast<uint16_t>(cur);
      s_bn[j % 3] = n;
      s_cursor = cur;
    };

    // tables of batch j into table set `set`
    auto build = [&](int j, int set) {
      const int nb = s_bn[j % 3];
      float *tset = tables + static_cast<size_t>(set) * batch * tstride;
#pragma unroll 1
      for (int g = 0; g < nb; ++g) {
        const float *cent = p.centroids + static_cast<size_t>(s_list[s_bat[j % 3][g]]) * d;
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

    // score and select the candidates of batch j against table set `set`
    auto scan = [&](int j, int set) {
      const int nb = s_bn[j % 3];
      const uint16_t *bat = s_bat[j % 3];
      const float *tset = tables + static_cast<size_t>(set) * batch * tstride;
      const uint32_t pre1 = s_len[bat[0]];
      const uint32_t pre2 = pre1 + (nb > 1 ? s_len[bat[1]] : 0u);
      const uint32_t pre3 = pre2 + (nb > 2 ? s_len[bat[2]] : 0u);
      const uint32_t pre4 = pre3 + (nb > 3 ? s_len[bat[3]] : 0u);
      for (uint32_t x0 = warp * 32; x0 < pre4; x0 += kScanThreads) {
        const uint32_t x = x0 + lane;
        // threshold first: candidates whose partial sum already exceeds it stop early
        uint64_t thr = tk.worst();
        const uint64_t bound = s_bound;
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
          cp = p.list_codes + s_coff[bat[g]] + static_cast<uint64_t>(c) * M;
          lg = tset + static_cast<size_t>(g) * tstride;
        }
        const float dist = adc_row_sum_bounded<KS>(cp, lg, M, ks, tkey, alive);
        const uint32_t dk = order_key(dist);
        const bool pass = alive && dk <= tkey;
        unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
        if (!mask) continue;
        const uint64_t key = pass ? ((static_cast<uint64_t>(dk) << 32) | p.list_ids[s_lbeg[bat[g]] + c]) : kEmptyKey;
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
    };

    if (tid == 0) {
      s_cursor = 0;
      form(0);
      form(1);
    }
    __syncthreads();
    if (s_bn[0] > 0) build(0, 0);
    __syncthreads();
    for (int j = 0; s_bn[j % 3] > 0; ++j) {
      const int set = j & 1;
      const bool has_next = s_bn[(j + 1) % 3] > 0;
      if (build_first) {
        if (has_next) build(j + 1, set ^ 1);
        scan(j, set);
      } else {
        scan(j, set);
        if (has_next) build(j + 1, set ^ 1);
      }
      if (tid == 0) form(j + 2);  // built in phase j + 1, scanned in phase j + 2
      __syncthreads();
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

template <int DSUB, int GPT, int R, int KS>
cudaError_t launch_pipe_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_pipe_kernel<DSUB, GPT, R, KS>;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t reserve = 16384;  // static shared memory of the kernel (~13 KB)
  int batch = kMaxBatch;
  while (batch > 1 && pipe_smem_bytes(p.d, p.M, KS, batch, R) + reserve > static_cast<size_t>(optin)) --batch;
  const size_t smem = pipe_smem_bytes(p.d, p.M, KS, batch, R);
  if (smem + reserve > static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
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
  kern<<<grid, kScanThreads, smem, s>>>(pp, batch);
  return cudaGetLastError();
}

}  // namespace vg
