// Fused IVF-PQ search kernel: one block owns one query at a time and runs
// the reference's per-query loop (search.rs:1175-1391) over its probed lists:
//   1. query residual  q - c_list                      (search.rs:1239-1245)
//   2. ADC table       T[m][c] = sum_j (r_mj - cw_mcj)^2 (pq.rs:196-267)
//   3. code scan       dist = sum_m T[m][code_m]       (pq_simd.rs:314-369)
//      (16-entry codebooks run ivfpq_four_kernel, scan_fourbit.cuh)
//   4. top-k by (distance, vector id)                  (search.rs:64-75)
//
// Persistent blocks (one per SM) take queries from an atomic counter, load
// and compact the query's probe list in parallel, and walk it nearest-first,
// kMaxBatch lists at a time:
//   - every thread builds its fixed share of each list's table; when DSUB > 0
//     a thread owns GPT groups of 4 adjacent entries of one subspace and keeps
//     their codewords in registers for the whole kernel, so a group costs one
//     broadcast load of the residual subvector, 4 x dsub subtract/multiply/add
//     triples and one 16-byte store;
//   - the 512 threads score the batch's candidates, one candidate per thread
//     with the reference's sequential sum over subspaces;
//   - each warp keeps its own sorted top-k for the whole query and admits a
//     candidate only if its key is below min(own k-th key, block bound).  The
//     block bound is the smallest k-th key any warp has reached -- a valid
//     upper bound on the query's final k-th key -- so after the nearest lists
//     almost every candidate is rejected by one comparison;
//   - at the end of the query the warp lists are merged and written out.
// Keys are (total_cmp order of the distance, vector id), unique per vector:
// the result is the reference's exactly, with its arbitrary order of equal
// distances fixed by the id.
#pragma once

#include <float.h>

#include "common.cuh"
#include "kernels.h"
#include "topk.cuh"

namespace vg {

constexpr int kScanThreads = 512;
constexpr int kScanWarps = kScanThreads / 32;
constexpr int kMaxBatch = 4;  // lists per batch (the candidate prefix below is unrolled for 4)

// Per-list shared memory: table (padded to 16 bytes) and residual.
__host__ __device__ inline size_t scan_pair_bytes(int d, int M, int ks) {
  return static_cast<size_t>((M * ks + 3) & ~3) * 4 + static_cast<size_t>((d + 3) & ~3) * 4;
}

__host__ __device__ inline size_t scan_smem_bytes(int d, int M, int ks, int batch, int R, bool rot = false) {
  return static_cast<size_t>(kScanWarps) * 32 * R * 8 + static_cast<size_t>(batch) * scan_pair_bytes(d, M, ks) +
         (rot ? static_cast<size_t>(batch) * ((d + 3) & ~3) * 4 : 0);
}

template <int R>
__device__ __forceinline__ void topk_insert_one(WarpTopK<R> &tk, uint64_t key) {
  if (R == 1) {
    const int lane = lane_id();
    if (key >= shfl64(tk.v[0], 31)) return;
    unsigned below = __ballot_sync(VG_FULL_MASK, tk.v[0] < key);
    int rank = __popc(below);
    uint64_t up = __shfl_up_sync(VG_FULL_MASK, static_cast<unsigned long long>(tk.v[0]), 1);
    tk.v[0] = lane < rank ? tk.v[0] : (lane == rank ? key : up);
  } else {
    tk.add(lane_id() == 0 ? key : kEmptyKey);
  }
}

// Read a subvector of D floats from 16-byte aligned shared memory (the
// start is aligned whenever D is a multiple of the vector width used).
template <int D>
__device__ __forceinline__ void load_subvector(const float *src, float (&v)[D]) {
  if (D % 4 == 0) {
#pragma unroll
    for (int j = 0; j < D; j += 4) {
      float4 t = *reinterpret_cast<const float4 *>(src + j);
      v[j] = t.x;
      v[j + 1] = t.y;
      v[j + 2] = t.z;
      v[j + 3] = t.w;
    }
  } else if (D % 2 == 0) {
#pragma unroll
    for (int j = 0; j < D; j += 2) {
      float2 t = *reinterpret_cast<const float2 *>(src + j);
      v[j] = t.x;
      v[j + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = src[j];
  }
}

// Sequential table sum for one candidate's codes (row layout [m][ks]).
template <int KS>
__device__ __forceinline__ float adc_row_sum(const uint8_t *cp, const float *lg, int M, int ks) {
  const int row_len = KS > 0 ? KS : ks;
  float acc = 0.0f;
  if ((M & 15) == 0) {
    for (int m0 = 0; m0 < M; m0 += 16) {
      uint4 w = *reinterpret_cast<const uint4 *>(cp + m0);
      uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      const float *row = lg + m0 * row_len;
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        uint32_t code = __byte_perm(ws[b >> 2], 0u, 0x4440u + (b & 3));
        acc = __fadd_rn(acc, row[b * row_len + code]);
      }
    }
  } else {
    for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, lg[m * row_len + cp[m]]);
  }
  return acc;
}

// adc_row_sum with early exit against a key threshold.  Table entries are
// >= +0 (squares) and a rounded add of a non-negative term never decreases
// the sum, so once the partial sum's order key exceeds tkey the full sum
// cannot pass `key <= tkey` either: the lane stops (alive = false) and its
// result is discarded by the caller.  The warp leaves the loop when no lane
// is alive.  Every lane of the warp must call this (it votes).
template <int KS>
__device__ __forceinline__ float adc_row_sum_bounded(const uint8_t *cp, const float *lg, int M, int ks,
                                                     uint32_t tkey, bool &alive) {
  const int row_len = KS > 0 ? KS : ks;
  float acc = 0.0f;
  if ((M & 15) == 0) {
    // the next 16 codes are loaded while the current 16 are summed
    uint4 wn = alive ? *reinterpret_cast<const uint4 *>(cp) : make_uint4(0u, 0u, 0u, 0u);
    for (int m0 = 0; m0 < M; m0 += 16) {
      if (!__any_sync(VG_FULL_MASK, alive)) break;
      const uint4 w = wn;
      if (alive && m0 + 16 < M) wn = *reinterpret_cast<const uint4 *>(cp + m0 + 16);
      if (alive) {
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const float *row = lg + m0 * row_len;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const uint32_t code = __byte_perm(ws[b >> 2], 0u, 0x4440u + (b & 3));
          acc = __fadd_rn(acc, row[b * row_len + code]);
        }
        alive = order_key(acc) <= tkey;
        if (alive) {
#pragma unroll
          for (int b = 8; b < 16; ++b) {
            const uint32_t code = __byte_perm(ws[b >> 2], 0u, 0x4440u + (b & 3));
            acc = __fadd_rn(acc, row[b * row_len + code]);
          }
          alive = order_key(acc) <= tkey;
        }
      }
    }
  } else if (alive) {
    for (int m = 0; m < M; ++m) acc = __fadd_rn(acc, lg[m * row_len + cp[m]]);
    alive = order_key(acc) <= tkey;
  }
  return acc;
}

// Squared distance of one residual subvector to one codeword, summed in the
// reference's order.  The first term is taken as is: for s >= +0 the
// reference's 0.0 + s equals s exactly, and a square is never -0.
template <int D>
__device__ __forceinline__ float sq_dist(const float (&q)[D], const float (&c)[D]) {
  float d0 = __fsub_rn(q[0], c[0]);
  float acc = __fmul_rn(d0, d0);
#pragma unroll
  for (int j = 1; j < D; ++j) {
    float dj = __fsub_rn(q[j], c[j]);
    acc = __fadd_rn(acc, __fmul_rn(dj, dj));
  }
  return acc;
}

template <int DSUB, int GPT, int R, int KS>
__global__ void __launch_bounds__(kScanThreads, 1) ivfpq_query_kernel(const ScanParams p, const int batch) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int M = p.M, ks = KS > 0 ? KS : p.ks, d = p.d, P = p.P, k = p.k;
  const int nent = M * ks;
  const int tstride = (nent + 3) & ~3;  // table stride, keeps every region 16-byte aligned
  const int dpad = (d + 3) & ~3;
  unsigned long long *wl = reinterpret_cast<unsigned long long *>(smem);  // [warps][32R]
  float *lut = reinterpret_cast<float *>(wl + kScanWarps * 32 * R);       // [batch][tstride]
  float *qres = lut + static_cast<size_t>(batch) * tstride;                // [batch][dpad]
  float *qrot = qres + static_cast<size_t>(batch) * dpad;                  // [batch][dpad] (OPQ only)

  __shared__ uint32_t s_query;
  __shared__ int s_nvalid;
  __shared__ int s_wcount[kScanWarps];
  __shared__ uint32_t s_list[kScanThreads], s_len[kScanThreads];
  __shared__ uint64_t s_lbeg[kScanThreads];
  __shared__ unsigned long long s_bound;
  __shared__ float s_lb[kScanThreads];      // distance lower bound of each compacted probe
  __shared__ uint8_t s_skip[kMaxBatch];     // list of the current batch skipped (pruned)

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // register-resident codewords: groups G = tid + i*512 cover entries 4G..4G+3
  constexpr int kD = DSUB > 0 ? DSUB : 1;
  constexpr int kG = GPT > 0 ? GPT : 1;
  const int ngroups = nent >> 2;
  float cb[kG][4][kD];
  if (DSUB > 0) {
#pragma unroll
    for (int i = 0; i < kG; ++i) {
      const int G = tid + i * kScanThreads;
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < kD; ++j)
          cb[i][u][j] = G < ngroups ? p.codebooks[(static_cast<size_t>(4 * G + u)) * kD + j] : 0.0f;
    }
  }

  for (;;) {
    if (tid == 0) {
      s_query = atomicAdd(p.counter, 1u);
      s_bound = kEmptyKey;
    }
    __syncthreads();
    if (s_query >= static_cast<uint32_t>(p.nq)) break;
    const uint32_t q = p.qmap ? p.qmap[s_query] : s_query;
    const float *qv = p.qn + static_cast<size_t>(q) * d;
    const uint32_t *prow = p.probes + (p.probes_shared ? 0 : static_cast<size_t>(q) * P);
    WarpTopK<R> tk;
    tk.init();

    // probe lists in chunks of one per thread (P may exceed the block size)
    for (int pc = 0; pc < P; pc += kScanThreads) {
    // probe metadata of the chunk, compacted to valid owned lists in order;
    // a filter also drops lists without its category (search.rs:1502-1505)
    {
      uint32_t l = 0xffffffffu;
      bool valid = false;
      if (pc + tid < P) {
        l = prow[pc + tid];
        valid = l != 0xffffffffu && (!p.owner || p.owner[l]) &&
                (!p.category || ((p.bitmask[l] >> p.want_cat) & 1ull));
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
        s_lb[pos] = p.probe_lb ? p.probe_lb[static_cast<size_t>(q) * P + pc + tid] : 0.0f;
      }
      if (tid == 0) s_nvalid = total;
      __syncthreads();
    }
    const int nvalid = s_nvalid;

    for (int b0 = 0; b0 < nvalid; b0 += batch) {
      const int nb = min(batch, nvalid - b0);
      const uint32_t *blist = s_list + b0;
      for (int i = tid; i < nb * d; i += kScanThreads) {
        int g = i / d, j = i - g * d;
        qres[g * dpad + j] = __fsub_rn(qv[j], p.centroids[static_cast<size_t>(blist[g]) * d + j]);
      }
      // list pruning (bound > block k-th distance: no candidate can enter);
      // decided by one thread, read by all after the barrier
      if (tid == 0) {
        const uint64_t bnd = s_bound;
        const float bdist = key_dist(bnd);
        for (int g = 0; g < kMaxBatch; ++g) s_skip[g] = g < nb && bnd != kEmptyKey && s_lb[b0 + g] > bdist;
      }
      __syncthreads();
      // OPQ: tables are built from the rotated residual R r (opq.rs:115-121);
      // output i is sum_j R[i][j] r_j from 0.0, read through R^T so that a
      // warp's loads of one j are contiguous
      const float *tq = qres;
      if (p.rot_t) {
        for (int i = tid; i < nb * d; i += kScanThreads) {
          const int g = i / d, r = i - g * d;
          const float *res = qres + g * dpad;
          float s = 0.0f;
          for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(p.rot_t[static_cast<size_t>(j) * d + r], res[j]));
          qrot[g * dpad + r] = s;
        }
        __syncthreads();
        tq = qrot;
      }

      // ---- ADC tables: sequential sum over the subvector, no FMA --------
#pragma unroll 1
      for (int g = 0; g < nb; ++g) {
        if (s_skip[g]) continue;
        const float *qg = tq + g * dpad;
        float *lg = lut + static_cast<size_t>(g) * tstride;
        if (DSUB > 0) {
#pragma unroll
          for (int i = 0; i < kG; ++i) {
            const int G = tid + i * kScanThreads;
            if (G < ngroups) {
              float qs[kD];
              load_subvector<kD>(qg + ((4 * G) / ks) * kD, qs);
              float4 out;
              out.x = sq_dist<kD>(qs, cb[i][0]);
              out.y = sq_dist<kD>(qs, cb[i][1]);
              out.z = sq_dist<kD>(qs, cb[i][2]);
              out.w = sq_dist<kD>(qs, cb[i][3]);
              *reinterpret_cast<float4 *>(lg + 4 * G) = out;
            }
          }
        } else {
          for (int e = tid; e < nent; e += kScanThreads) {
            const float *qs = qg + (e / ks) * p.dsub;
            const float *cw = p.codebooks + static_cast<size_t>(e) * p.dsub;
            float acc = 0.0f;
            for (int j = 0; j < p.dsub; ++j) {
              float diff = __fsub_rn(qs[j], __ldg(cw + j));
              acc = __fadd_rn(acc, __fmul_rn(diff, diff));
            }
            lg[e] = acc;
          }
        }
      }
      __syncthreads();

      // candidate prefix over the batch's lists (kMaxBatch == 4)
      const uint32_t pre1 = s_skip[0] ? 0u : s_len[b0];
      const uint32_t pre2 = pre1 + (nb > 1 && !s_skip[1] ? s_len[b0 + 1] : 0u);
      const uint32_t pre3 = pre2 + (nb > 2 && !s_skip[2] ? s_len[b0 + 2] : 0u);
      const uint32_t pre4 = pre3 + (nb > 3 && !s_skip[3] ? s_len[b0 + 3] : 0u);

      // ---- score and select ---------------------------------------------
      const uint32_t ctotal = pre4;
      for (uint32_t x0 = warp * 32; x0 < ctotal; x0 += kScanThreads) {
        const uint32_t x = x0 + lane;
        // threshold first: candidates whose partial sum already exceeds it stop early
        uint64_t thr = tk.worst();
        const uint64_t bound = s_bound;
        thr = bound < thr ? bound : thr;
        const uint32_t tkey = static_cast<uint32_t>(thr >> 32);
        int g = 0;
        uint32_t c = 0, vid = 0;
        bool live = x < ctotal;
        const uint8_t *cp = p.list_codes;
        const float *lg = lut;
        if (live) {
          g = (x >= pre1) + (x >= pre2) + (x >= pre3);
          const uint32_t lo = g == 0 ? 0u : g == 1 ? pre1 : g == 2 ? pre2 : pre3;
          c = x - lo;
          if (p.category) {  // only documents whose metadata matches (search.rs:1515-1520)
            vid = p.list_ids[s_lbeg[b0 + g] + c];
            live = p.category[vid] == static_cast<uint8_t>(p.want_cat);
          }
          cp = p.list_codes + p.code_off[blist[g]] + static_cast<uint64_t>(c) * M;
          lg = lut + static_cast<size_t>(g) * tstride;
        }
        const float dist = adc_row_sum_bounded<KS>(cp, lg, M, ks, tkey, live);
        const uint32_t dk = order_key(dist);
        const bool pass = live && dk <= tkey;
        unsigned mask = __ballot_sync(VG_FULL_MASK, pass);
        if (!mask) continue;
        uint64_t key =
            pass ? ((static_cast<uint64_t>(dk) << 32) | (p.category ? vid : p.list_ids[s_lbeg[b0 + g] + c])) : kEmptyKey;
        if (p.key_floor && key <= p.key_floor[q]) key = kEmptyKey;  // selected by an earlier pass
        if (__popc(mask) > 4) {
          tk.add(key < thr ? key : kEmptyKey);
        } else {
          while (mask) {
            int src = __ffs(mask) - 1;
            mask &= mask - 1;
            uint64_t kx = shfl64(key, src);
            if (kx < thr) topk_insert_one(tk, kx);
          }
        }
        const uint64_t kth = tk.get(k - 1);
        if (lane == 0 && kth < bound) atomicMin(&s_bound, kth);
      }
      __syncthreads();  // tables and batch metadata are rewritten next
    }
    }  // probe chunks

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
cudaError_t launch_scan_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_query_kernel<DSUB, GPT, R, KS>;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t reserve = 12288;  // static shared memory of the kernel (8-9 KB)
  int batch = kMaxBatch;
  while (batch > 1 && scan_smem_bytes(p.d, p.M, p.ks, batch, R, p.rot_t != nullptr) + reserve > static_cast<size_t>(optin)) --batch;
  const size_t smem = scan_smem_bytes(p.d, p.M, p.ks, batch, R, p.rot_t != nullptr);
  if (smem + reserve > static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int grid = num_sms * per_sm;
  if (grid > p.nq) grid = p.nq;
  kern<<<grid, kScanThreads, smem, s>>>(p, batch);
  return cudaGetLastError();
}

}  // namespace vg
