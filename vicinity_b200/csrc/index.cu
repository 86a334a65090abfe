// C ABI of the B200 IVF-PQ engine (include/vicinity_gpu.h): the index object,
// its device-resident layout, build and search orchestration, sharding over
// NCCL, and the exact flat search.
//
// Device layout of a built index (one GPU):
//   vectors    f32 [n][d]          L2-normalised rows (dropped by compact)
//   doc_ids    u32 [n]             caller ids by insertion index
//   centroids  f32 [Lc][d]         coarse centroids (Lc <= num_clusters)
//   codebooks  f32 [M][ks][dsub]   product quantizer (pq.rs:19-21 layout)
//   assign     u32 [n]             list of each insertion index
//   codes      u8  [n][M]          codes in insertion order (codes.bin)
//   list_off   u64 [Lc+1]          CSR offsets of the inverted lists
//   list_ids   u32 [n]             insertion indices, ascending within a list
//   code_off   u64 [Lc]            16-byte aligned byte offset of each list's
//   list_codes u8                  list-contiguous codes (list_codes.bin)
//   pack_off   u64 [Lc]            (ks == 16) 16-byte aligned byte offset of
//   packed     u8                  each list's nibble-packed codes: vector-major,
//                                  ceil(M/2) bytes per vector, lists >= 16 only
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <unordered_map>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "opq.h"
#include "snapshot.h"
#include "vicinity_gpu.h"

using namespace vg;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  int code = e == cudaErrorMemoryAllocation ? VG_ERR_OUT_OF_MEMORY : VG_ERR_CUDA;
  cudaGetLastError();  // clear a sticky launch error so later calls start clean
  return fail(code, std::string(what) + ": " + cudaGetErrorString(e));
}

#define VG_CU(call)                                         \
  do {                                                      \
    cudaError_t vg_e_ = (call);                             \
    if (vg_e_ != cudaSuccess) return cuda_fail(vg_e_, #call); \
  } while (0)

#define VG_TRY(call)            \
  do {                          \
    int vg_s_ = (call);         \
    if (vg_s_ != VG_OK) return vg_s_; \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Owning device buffer with grow-only capacity.  reserve() discards contents.
struct DevBuf {
  void *p = nullptr;
  size_t cap = 0;
  DevBuf() = default;
  DevBuf(const DevBuf &) = delete;
  DevBuf &operator=(const DevBuf &) = delete;
  DevBuf(DevBuf &&o) noexcept : p(o.p), cap(o.cap) {
    o.p = nullptr;
    o.cap = 0;
  }
  DevBuf &operator=(DevBuf &&o) noexcept {
    if (this != &o) {
      release();
      p = o.p;
      cap = o.cap;
      o.p = nullptr;
      o.cap = 0;
    }
    return *this;
  }
  ~DevBuf() { release(); }
  cudaError_t reserve(size_t bytes) {
    if (bytes <= cap) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) cap = bytes;
    else p = nullptr;
    return e;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
  template <class T>
  T *as() const {
    return static_cast<T *>(p);
  }
};

bool is_device_ptr(const void *ptr) {
  if (!ptr) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

uint64_t splitmix64(uint64_t &s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Seeded Fisher-Yates prefix: the first `take` entries of a permutation of
// [0, n).  (The reference shuffles with rand's StdRng, search.rs:808-810;
// training is not bit-reproducible across implementations, so any seeded
// permutation serves.)
std::vector<uint32_t> seeded_prefix(size_t n, size_t take, uint64_t seed) {
  std::vector<uint32_t> idx(n);
  std::iota(idx.begin(), idx.end(), 0u);
  uint64_t s = seed;
  for (size_t i = 0; i < take && i + 1 < n; ++i) {
    size_t j = i + static_cast<size_t>(splitmix64(s) % (n - i));
    std::swap(idx[i], idx[j]);
  }
  idx.resize(take);
  return idx;
}

constexpr size_t kDistBudgetBytes = size_t(1) << 30;  // coarse distance tile
constexpr size_t kAssignChunk = size_t(4) << 20;      // rows per argmin launch
constexpr int kPhaseEvents = 12;
constexpr int kStats = 11;  // profiling counters (vg_index::stats)
// A list-sharded search's main pass runs units of this many probes of one
// query (a query with many unpruned lists spreads over several warps); items
// whose lists hold at least kHeavyVectors vectors are started first.
constexpr int kUnitProbes = 8;
// Host query batches from this many rows on are uploaded in tiles that the
// coarse stage consumes as they arrive.
constexpr size_t kPipeMinRows = 4096;
constexpr uint32_t kHeavyVectors = 1024;

}  // namespace

struct vg_index {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;      // stream in use
  cudaStream_t own_stream = nullptr;  // stream the index created
  size_t d = 0, dsub = 0;
  vg_ivfpq_params params{};
  size_t n = 0, cap = 0;
  size_t num_centroids = 0;
  bool trained = false, built = false, compacted = false;

  DevBuf vectors, doc_ids, centroids, codebooks, assign, codes;
  DevBuf list_off, list_ids, code_off, list_codes, pack_off, packed;
  DevBuf list_radius;  // f32 [Lc]: largest reconstructed-residual norm per list (list pruning)
  DevBuf cent_norm;    // f32 [1]: largest centroid norm (probe shortlist error bound)
  DevBuf sub_radius;   // f32 [M + 1]: largest codeword norm per subspace, then of all (4-bit list pruning)
  DevBuf cent_img;     // binary16 operand image of the centroids (tensor-core coarse products)
  int cent_kp = 0;     // K padding of cent_img (0: no tensor-core path)
  float h_cmax = 0.0f; // largest centroid norm (host copy)
  std::vector<uint64_t> h_list_off;
  std::vector<uint32_t> h_doc_ids;

  // quantizer kind and OPQ rotation (opq.rs): rotation [d][d] row-major when set
  bool optimized = false;
  DevBuf rotation, rotation_t;  // row-major (encode) and transposed (scan kernels)
  std::vector<float> h_rotation;

  // metadata filtering (search.rs:414-470, 626-651): the filter field, every
  // document's metadata in the reference's serialised form, and per list the
  // bitmask of the filter categories present
  bool has_filter_field = false;
  std::string filter_field;
  std::map<uint32_t, std::string> metadata;      // doc id -> metadata object (serde JSON)
  std::unordered_map<uint32_t, int> doc_category;  // doc id -> filter category 0..63 (-1: none)
  std::vector<uint64_t> h_bitmask;                 // [num_clusters], fixed at build
  DevBuf category_d, bitmask_d, cat_counts;        // [n] u8, [num_clusters] u64, [Lc][64] u32
  bool cat_dirty = true;                           // categories changed since the last upload

  // sharding: lists owned by this rank (owner[l] != 0); once sharded, the
  // device list layout (list_off, code_off, pack_off, list_ids, list_codes,
  // packed) holds this rank's lists only (other lists empty) and the
  // insertion-order codes and assignments are dropped
  int rank = 0, world = 1;
  ncclComm_t comm = nullptr;
  int comm_timeout_ms = 60000;
  DevBuf owner;
  bool partitioned = false;
  DevBuf ws_seed;  // [world * nq] u64 seed keys of a sharded search

  // search workspace
  DevBuf ws_q, ws_qn, ws_dist, ws_probes, ws_pdist, ws_scalars,
      ws_keys, ws_all_keys, ws_out_ids, ws_out_dist, ws_out_count, ws_lb, ws_rec, ws_lbq, ws_qimg, ws_eps, ws_tc,
      ws_floor, ws_qall, ws_cmax, ws_units, ws_work;
  DevBuf stats;  // u64 [pairs, vectors, code bytes, scan counters [4], seed scan counters [4]] while profiling

  // error flag of bounded device waits, in mapped pinned host memory
  int *h_err = nullptr, *d_err = nullptr;

  // profiling
  bool profiling = false;
  cudaEvent_t ev[kPhaseEvents] = {};
  size_t coarse_tile_rows = 0;  // query rows per coarse-product tile (0: from kDistBudgetBytes)
  // per-tile (start, coarse done, select done) events of a tiled coarse stage,
  // read after the call's final synchronisation; tile_marks redirects marks 2-4
  std::vector<cudaEvent_t> tile_ev;
  // host queries copied in tiles on their own stream, each tile's coarse
  // stage waiting only for its rows (no timing on these events)
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t copy_start = nullptr;
  std::vector<cudaEvent_t> copy_ev;
  cudaEvent_t *tile_marks = nullptr;
  vg_search_profile prof{};
  uint64_t launches = 0;

  size_t device_bytes() const {
    return vectors.cap + doc_ids.cap + centroids.cap + codebooks.cap + assign.cap + codes.cap +
           list_off.cap + list_ids.cap + code_off.cap + list_codes.cap + pack_off.cap + packed.cap +
           owner.cap + rotation.cap + rotation_t.cap + category_d.cap + bitmask_d.cap + cat_counts.cap +
           list_radius.cap + cent_norm.cap + sub_radius.cap + cent_img.cap;
  }
};

namespace {

int validate_shape(size_t dim, const vg_ivfpq_params &p) {
  if (dim == 0) return fail(VG_ERR_INVALID_CONFIG, "invalid config `dimension`: must be greater than 0");
  if (p.codebook_size > 256)
    return fail(VG_ERR_INVALID_CONFIG,
                "invalid config `codebook_size`: must be at most 256 because PQ codes are stored as u8");
  if (p.num_codebooks == 0 || p.codebook_size == 0 || p.num_clusters == 0)
    return fail(VG_ERR_INVALID_CONFIG,
                "invalid config `num_clusters, num_codebooks, codebook_size`: must all be greater than 0");
  if (dim % p.num_codebooks != 0)
    return fail(VG_ERR_INVALID_CONFIG, "invalid config `dimension`: must be divisible by num_codebooks");
  if (p.codebook_size == 16 && p.num_codebooks > 65535 / 255)
    return fail(VG_ERR_INVALID_PARAMETER,
                "FastScan accumulates LUT terms in u16: at most 257 codebooks are supported");
  if (p.num_clusters > 0x7fffffffull || p.num_codebooks > 4096)
    return fail(VG_ERR_INVALID_CONFIG, "invalid config: num_clusters or num_codebooks out of range");
  return VG_OK;
}

int sync_stream(vg_index *ix) {
  if (!ix->comm) {
    VG_CU(cudaStreamSynchronize(ix->stream));
    return VG_OK;
  }
  // Bounded wait: a peer that never arrives must not hang the caller.
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(ix->comm_timeout_ms);
  for (;;) {
    cudaError_t q = cudaStreamQuery(ix->stream);
    if (q == cudaSuccess) return VG_OK;
    if (q != cudaErrorNotReady) return cuda_fail(q, "cudaStreamQuery");
    ncclResult_t ar = ncclSuccess;
    ncclCommGetAsyncError(ix->comm, &ar);
    if (ar != ncclSuccess && ar != ncclInProgress) {
      ncclCommAbort(ix->comm);
      ix->comm = nullptr;
      return fail(VG_ERR_NCCL, std::string("NCCL async error: ") + ncclGetErrorString(ar));
    }
    if (std::chrono::steady_clock::now() > deadline) {
      ncclCommAbort(ix->comm);
      ix->comm = nullptr;
      return fail(VG_ERR_NCCL, "collective did not complete within the shard timeout; communicator aborted");
    }
    std::this_thread::yield();
  }
}

int nccl_wait_ready(ncclComm_t comm, int timeout_ms) {
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    ncclResult_t r = ncclSuccess;
    ncclCommGetAsyncError(comm, &r);
    if (r == ncclSuccess) return VG_OK;
    if (r != ncclInProgress) return fail(VG_ERR_NCCL, std::string("NCCL: ") + ncclGetErrorString(r));
    if (std::chrono::steady_clock::now() > deadline)
      return fail(VG_ERR_NCCL, "NCCL operation did not complete within the timeout");
    std::this_thread::yield();
  }
}

void mark(vg_index *ix, int i) {
  if (!ix->profiling) return;
  cudaEventRecord(ix->tile_marks && i >= 2 && i <= 4 ? ix->tile_marks[i - 2] : ix->ev[i], ix->stream);
}

cudaError_t reserve_copy_pipeline(vg_index *ix, size_t tiles) {
  if (!ix->copy_stream) {
    cudaError_t e = cudaStreamCreateWithFlags(&ix->copy_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
  }
  if (!ix->copy_start) {
    cudaError_t e = cudaEventCreateWithFlags(&ix->copy_start, cudaEventDisableTiming);
    if (e != cudaSuccess) return e;
  }
  while (ix->copy_ev.size() < tiles) {
    cudaEvent_t e = nullptr;
    cudaError_t err = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (err != cudaSuccess) return err;
    ix->copy_ev.push_back(e);
  }
  return cudaSuccess;
}

cudaError_t reserve_tile_events(vg_index *ix, size_t count) {
  while (ix->tile_ev.size() < count) {
    cudaEvent_t e = nullptr;
    cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) return err;
    ix->tile_ev.push_back(e);
  }
  return cudaSuccess;
}

// ---- training (device Lloyd iterations; not bit-pinned to the reference's
// third-party k-means, see src/partitioning/kmeans.rs:64-90) --------------

int upload_rotation(vg_index *ix);

// The tensor-core path (tc_select.cu) ranks columns by binary16 products and
// re-scores, with the reference's arithmetic, every column its error bound
// cannot rule out.  It applies to rows of up to 128 floats and centroids
// shorter than 100 (beyond that the bound admits most lists); everything else
// takes the exact SIMT tiles.  VICINITY_COARSE=exact forces the exact path.
constexpr size_t kTcMinLists = 512;

bool tc_disabled() {
  static const bool off = [] {
    const char *e = std::getenv("VICINITY_COARSE");
    return e && std::strcmp(e, "exact") == 0;
  }();
  return off;
}

bool coarse_on_tensor_cores(const vg_index *ix, size_t P) {
  return !tc_disabled() && ix->cent_kp && ix->num_centroids >= kTcMinLists && P >= 1 && P <= 256 &&
         std::isfinite(ix->h_cmax) && ix->h_cmax < 100.0f;
}

// Probe selection on the tensor cores: up to 128 probes the binary16 product
// matrix (tile by tile, at most 1 GiB) and the probe shortlist; beyond, the
// fused candidate window.
constexpr size_t kShortlistMaxProbes = 128;
bool coarse_via_products(const vg_index *ix, size_t P) {
  return coarse_on_tensor_cores(ix, P) && P <= kShortlistMaxProbes;
}

// Largest centroid norm (device and host copies) and the binary16 operand
// image of the centroids, after the centroids are final.
int prepare_centroids(vg_index *ix) {
  cudaStream_t s = ix->stream;
  const size_t Lc = ix->num_centroids;
  const int d = static_cast<int>(ix->d);
  VG_CU(ix->cent_norm.reserve(4));
  VG_CU(launch_centroid_norm_max(ix->centroids.as<float>(), Lc, d, ix->cent_norm.as<float>(), s));
  VG_CU(cudaMemcpyAsync(&ix->h_cmax, ix->cent_norm.p, 4, cudaMemcpyDeviceToHost, s));
  ix->cent_kp = umma_kp(d);
  if (ix->cent_kp) {
    VG_CU(ix->cent_img.reserve(umma_image_bytes(std::max<size_t>(Lc, 1), ix->cent_kp)));
    VG_CU(launch_umma_image(ix->centroids.as<float>(), Lc, d, ix->cent_kp, ix->cent_img.p, nullptr, 0.0, 0.0,
                            nullptr, s));
  }
  VG_CU(cudaStreamSynchronize(s));
  return VG_OK;
}

int check_device_error(vg_index *ix, const char *what) {
  if (const int code = *reinterpret_cast<volatile int *>(ix->h_err)) {
    *reinterpret_cast<volatile int *>(ix->h_err) = 0;
    return fail(VG_ERR_CUDA, std::string(what) + " gave up on a bounded device wait (code " + std::to_string(code) + ")");
  }
  return VG_OK;
}

// List of each of the n rows of X (kmeans.rs:97-107, used at search.rs:621):
// argmin over the L centroids of 1 - x.c, ties to the lower list, into out.
// With prev set, the rows whose list differs from prev are added to *changed.
// Rows go through the tensor-core window with P = 1 (re-scored exactly), or
// the exact argmin tiles when that path does not apply.
constexpr size_t kTcAssignChunk = size_t(1) << 20;

int assign_rows_to_lists(vg_index *ix, const float *X, size_t n, const float *cent, size_t L, uint32_t *out,
                         const uint32_t *prev, unsigned int *changed) {
  if (n == 0) return VG_OK;
  cudaStream_t s = ix->stream;
  const int d = static_cast<int>(ix->d), kp = umma_kp(d);
  if (kp && L >= kTcMinLists && !tc_disabled()) {
    DevBuf cn;
    float cmax = 0.0f;
    VG_CU(cn.reserve(4));
    VG_CU(launch_centroid_norm_max(cent, L, d, cn.as<float>(), s));
    VG_CU(cudaMemcpyAsync(&cmax, cn.p, 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaStreamSynchronize(s));
    if (std::isfinite(cmax) && cmax < 100.0f) {
      const size_t chunk = std::min(n, kTcAssignChunk);
      DevBuf cimg, aimg, eps, ws, dist;
      VG_CU(cimg.reserve(umma_image_bytes(L, kp)));
      VG_CU(aimg.reserve(umma_image_bytes(chunk, kp)));
      VG_CU(eps.reserve(chunk * 4));
      VG_CU(ws.reserve(tc_select_workspace_bytes(chunk, L, 1, ix->num_sms)));
      VG_CU(dist.reserve(chunk * 4));
      VG_CU(launch_umma_image(cent, L, d, kp, cimg.p, nullptr, 0.0, 0.0, nullptr, s));
      double rel = 0, abs_coef = 0;
      tc_error_coefs(d, &rel, &abs_coef);
      *reinterpret_cast<volatile int *>(ix->h_err) = 0;
      for (size_t r0 = 0; r0 < n; r0 += chunk) {
        const size_t rows = std::min(chunk, n - r0);
        VG_CU(launch_umma_image(X + r0 * d, rows, d, kp, aimg.p, cn.as<float>(), rel, abs_coef, eps.as<float>(), s));
        TcSelect t{};
        t.a_img = aimg.p;
        t.q = X + r0 * d;
        t.rows = rows;
        t.b_img = cimg.p;
        t.x = cent;
        t.cols = L;
        t.d = d;
        t.kp = kp;
        t.P = 1;
        t.mode = 0;
        t.eps = eps.as<float>();
        t.workspace = ws.p;
        t.out_ids = out + r0;
        t.out_dist = dist.as<float>();
        t.out_ld = 1;
        t.error = ix->d_err;
        VG_CU(launch_tc_select(t, ix->num_sms, s));
      }
      if (prev) VG_CU(launch_count_diff_u32(out, prev, n, changed, s));
      VG_CU(cudaStreamSynchronize(s));
      return check_device_error(ix, "list assignment");
    }
  }
  DevBuf best;
  const size_t chunk = std::min(n, kAssignChunk);
  VG_CU(best.reserve(chunk * 8));
  for (size_t r0 = 0; r0 < n; r0 += chunk) {
    const size_t rows = std::min(chunk, n - r0);
    VG_CU(cudaMemsetAsync(best.p, 0xff, rows * 8, s));
    VG_CU(launch_coarse_argmin(X + r0 * d, rows, cent, L, d, best.as<unsigned long long>(), s));
    VG_CU(launch_keys_to_assign(best.as<unsigned long long>(), rows, out + r0, prev ? prev + r0 : nullptr, changed, s));
  }
  VG_CU(cudaStreamSynchronize(s));
  return VG_OK;
}

int train(vg_index *ix, size_t n_train, size_t max_iter) {
  cudaStream_t s = ix->stream;
  const size_t d = ix->d, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const size_t Lc = std::min<size_t>(ix->params.num_clusters, n_train);

  // training rows (ascending, search.rs:789-814)
  std::vector<uint32_t> rows;
  if (n_train < ix->n) {
    rows = seeded_prefix(ix->n, n_train, ix->params.seed);
    std::sort(rows.begin(), rows.end());
  }
  DevBuf train_x, rows_d, assign_t, assign_prev, keys_sorted, ids_sorted, iota, seg, temp, scal, newc;
  const float *X = ix->vectors.as<float>();
  if (!rows.empty()) {
    VG_CU(rows_d.reserve(n_train * 4));
    VG_CU(cudaMemcpyAsync(rows_d.p, rows.data(), n_train * 4, cudaMemcpyHostToDevice, s));
    VG_CU(train_x.reserve(n_train * d * 4));
    VG_CU(launch_gather_rows(X, static_cast<int>(d), rows_d.as<uint32_t>(), n_train, train_x.as<float>(), s));
    X = train_x.as<float>();
  }

  // coarse: spherical Lloyd from a seeded sample of training rows
  VG_CU(ix->centroids.reserve(Lc * d * 4));
  {
    std::vector<uint32_t> init = seeded_prefix(n_train, Lc, ix->params.seed);
    DevBuf init_d;
    VG_CU(init_d.reserve(Lc * 4));
    VG_CU(cudaMemcpyAsync(init_d.p, init.data(), Lc * 4, cudaMemcpyHostToDevice, s));
    VG_CU(launch_gather_rows(X, static_cast<int>(d), init_d.as<uint32_t>(), Lc, ix->centroids.as<float>(), s));
    VG_CU(cudaStreamSynchronize(s));
  }
  VG_CU(assign_t.reserve(n_train * 4));
  VG_CU(assign_prev.reserve(n_train * 4));
  VG_CU(keys_sorted.reserve(n_train * 4));
  VG_CU(ids_sorted.reserve(n_train * M * 4 > n_train * 4 ? n_train * M * 4 : n_train * 4));
  VG_CU(iota.reserve(n_train * M * 4));
  VG_CU(seg.reserve((std::max(Lc, M * ks) + 1) * 4));
  VG_CU(scal.reserve(16));
  VG_CU(newc.reserve(std::max(Lc * d, M * ks * (d / M)) * 4));
  size_t temp_bytes = 0, tb2 = 0;
  VG_CU(sort_pairs_u32(nullptr, temp_bytes, nullptr, nullptr, nullptr, nullptr, n_train * M, 32, s));
  VG_CU(sort_pairs_u32(nullptr, tb2, nullptr, nullptr, nullptr, nullptr, n_train, 32, s));
  temp_bytes = std::max(temp_bytes, tb2);
  VG_CU(temp.reserve(temp_bytes));
  VG_CU(launch_iota(iota.as<uint32_t>(), n_train, s));

  unsigned int changed = 1;
  for (size_t it = 0; it < max_iter && changed; ++it) {
    VG_CU(cudaMemsetAsync(scal.p, 0, 4, s));
    VG_TRY(assign_rows_to_lists(ix, X, n_train, ix->centroids.as<float>(), Lc, assign_t.as<uint32_t>(),
                                it ? assign_prev.as<uint32_t>() : nullptr, scal.as<unsigned int>()));
    size_t tb = temp_bytes;
    VG_CU(sort_pairs_u32(temp.p, tb, assign_t.as<uint32_t>(), keys_sorted.as<uint32_t>(), iota.as<uint32_t>(),
                         ids_sorted.as<uint32_t>(), n_train, 32, s));
    VG_CU(launch_segments(keys_sorted.as<uint32_t>(), n_train, Lc, seg.as<uint32_t>(), s));
    VG_CU(launch_kmeans_update(X, static_cast<int>(d), ids_sorted.as<uint32_t>(), seg.as<uint32_t>(), Lc,
                               ix->centroids.as<float>(), newc.as<float>(), 1, s));
    VG_CU(cudaMemcpyAsync(ix->centroids.p, newc.p, Lc * d * 4, cudaMemcpyDeviceToDevice, s));
    VG_CU(cudaMemcpyAsync(assign_prev.p, assign_t.p, n_train * 4, cudaMemcpyDeviceToDevice, s));
    VG_CU(cudaMemcpyAsync(&changed, scal.p, 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaStreamSynchronize(s));
    if (it == 0) changed = 1;
  }

  // PQ: Euclidean Lloyd per subspace on training residuals (pq.rs:75-124)
  VG_TRY(assign_rows_to_lists(ix, X, n_train, ix->centroids.as<float>(), Lc, assign_t.as<uint32_t>(), nullptr,
                              nullptr));
  DevBuf resid, codes_t, codes_prev, pkeys;
  VG_CU(resid.reserve(n_train * d * 4));
  VG_CU(launch_residuals(X, n_train, static_cast<int>(d), assign_t.as<uint32_t>(), ix->centroids.as<float>(),
                         resid.as<float>(), s));
  const size_t dsub = d / M;
  VG_CU(ix->codebooks.reserve(M * ks * dsub * 4));
  VG_CU(codes_t.reserve(n_train * M));
  VG_CU(codes_prev.reserve(n_train * M));
  VG_CU(pkeys.reserve(n_train * M * 4));
  DevBuf pvals, pkeys_sorted;
  VG_CU(pvals.reserve(n_train * M * 4));
  VG_CU(pkeys_sorted.reserve(n_train * M * 4));
  int end_bit = 1;
  while ((size_t(1) << end_bit) < M * ks) ++end_bit;

  // Lloyd iterations of the M codebooks on the rows of `data` (training
  // residuals, rotated when OPQ is on), from seeded rows per subspace
  auto fit_pq = [&](const float *data) -> int {
    std::vector<float> cb_init(M * ks * dsub);
    std::vector<float> host_res;  // gather the seeded rows per subspace on the host
    for (size_t m = 0; m < M; ++m) {
      std::vector<uint32_t> pick = seeded_prefix(n_train, ks, ix->params.seed + m);
      DevBuf pick_d, rows_out;
      VG_CU(pick_d.reserve(ks * 4));
      VG_CU(rows_out.reserve(ks * d * 4));
      VG_CU(cudaMemcpyAsync(pick_d.p, pick.data(), ks * 4, cudaMemcpyHostToDevice, s));
      VG_CU(launch_gather_rows(data, static_cast<int>(d), pick_d.as<uint32_t>(), ks, rows_out.as<float>(), s));
      host_res.resize(ks * d);
      VG_CU(cudaMemcpyAsync(host_res.data(), rows_out.p, ks * d * 4, cudaMemcpyDeviceToHost, s));
      VG_CU(cudaStreamSynchronize(s));
      for (size_t c = 0; c < ks; ++c)
        std::memcpy(&cb_init[(m * ks + c) * dsub], &host_res[c * d + m * dsub], dsub * 4);
    }
    VG_CU(cudaMemcpyAsync(ix->codebooks.p, cb_init.data(), cb_init.size() * 4, cudaMemcpyHostToDevice, s));
    changed = 1;
    for (size_t it = 0; it < max_iter && changed; ++it) {
      VG_CU(launch_encode_residuals(data, n_train, static_cast<int>(d), ix->codebooks.as<float>(),
                                    static_cast<int>(M), static_cast<int>(ks), codes_t.as<uint8_t>(), s));
      VG_CU(cudaMemsetAsync(scal.p, 0, 4, s));
      if (it) VG_CU(launch_count_diff_u8(codes_t.as<uint8_t>(), codes_prev.as<uint8_t>(), n_train * M,
                                         scal.as<unsigned int>(), s));
      VG_CU(launch_pq_keys(codes_t.as<uint8_t>(), n_train, static_cast<int>(M), static_cast<int>(ks),
                           pkeys.as<uint32_t>(), pvals.as<uint32_t>(), s));
      size_t tb = temp_bytes;
      VG_CU(sort_pairs_u32(temp.p, tb, pkeys.as<uint32_t>(), pkeys_sorted.as<uint32_t>(), pvals.as<uint32_t>(),
                           ids_sorted.as<uint32_t>(), n_train * M, end_bit, s));
      VG_CU(launch_segments(pkeys_sorted.as<uint32_t>(), n_train * M, M * ks, seg.as<uint32_t>(), s));
      VG_CU(launch_pq_update(data, n_train, static_cast<int>(d), static_cast<int>(M), static_cast<int>(ks),
                             ids_sorted.as<uint32_t>(), seg.as<uint32_t>(), ix->codebooks.as<float>(),
                             newc.as<float>(), s));
      VG_CU(cudaMemcpyAsync(ix->codebooks.p, newc.p, M * ks * dsub * 4, cudaMemcpyDeviceToDevice, s));
      VG_CU(cudaMemcpyAsync(codes_prev.p, codes_t.p, n_train * M, cudaMemcpyDeviceToDevice, s));
      VG_CU(cudaMemcpyAsync(&changed, scal.p, 4, cudaMemcpyDeviceToHost, s));
      VG_CU(cudaStreamSynchronize(s));
      if (it == 0) changed = 1;
    }
    return VG_OK;
  };

  if (!ix->h_rotation.empty()) {
    // a rotation given by the caller: codebooks of the rotated residuals
    DevBuf rot;
    VG_CU(rot.reserve(n_train * d * 4));
    VG_CU(launch_rotate_rows(resid.as<float>(), n_train, static_cast<int>(d), ix->rotation.as<float>(),
                             rot.as<float>(), s));
    VG_TRY(fit_pq(rot.as<float>()));
  } else if (!ix->params.use_opq) {
    VG_TRY(fit_pq(resid.as<float>()));
  } else {
    // OPQ (opq.rs:65-105): ten alternations of fitting the codebooks on the
    // rotated residuals and re-solving the rotation by Procrustes on the
    // first min(n, 5000) residuals (opq.rs:207-290)
    std::vector<float> rmat(d * d, 0.0f);
    for (size_t i = 0; i < d; ++i) rmat[i * d + i] = 1.0f;
    const size_t S = std::min<size_t>(n_train, 5000);
    DevBuf rot, rdev;
    VG_CU(rot.reserve(n_train * d * 4));
    VG_CU(rdev.reserve(d * d * 4));
    std::vector<float> xs(S * d), cbh(M * ks * dsub);
    std::vector<uint8_t> cs(S * M);
    VG_CU(cudaMemcpyAsync(xs.data(), resid.p, S * d * 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaStreamSynchronize(s));
    std::vector<double> cov(d * d), rec(d);
    for (int iter = 0; iter < 10; ++iter) {
      VG_CU(cudaMemcpyAsync(rdev.p, rmat.data(), d * d * 4, cudaMemcpyHostToDevice, s));
      const float *data = resid.as<float>();
      if (iter > 0) {
        VG_CU(launch_rotate_rows(resid.as<float>(), n_train, static_cast<int>(d), rdev.as<float>(),
                                 rot.as<float>(), s));
        data = rot.as<float>();
      }
      VG_TRY(fit_pq(data));
      // M = sum_k recon(quantize(R x_k)) x_k^T over the sample
      VG_CU(launch_rotate_rows(resid.as<float>(), S, static_cast<int>(d), rdev.as<float>(), rot.as<float>(), s));
      VG_CU(launch_encode_residuals(rot.as<float>(), S, static_cast<int>(d), ix->codebooks.as<float>(),
                                    static_cast<int>(M), static_cast<int>(ks), codes_t.as<uint8_t>(), s));
      VG_CU(cudaMemcpyAsync(cs.data(), codes_t.p, S * M, cudaMemcpyDeviceToHost, s));
      VG_CU(cudaMemcpyAsync(cbh.data(), ix->codebooks.p, cbh.size() * 4, cudaMemcpyDeviceToHost, s));
      VG_CU(cudaStreamSynchronize(s));
      std::fill(cov.begin(), cov.end(), 0.0);
      for (size_t k = 0; k < S; ++k) {
        for (size_t m = 0; m < M; ++m)
          for (size_t j = 0; j < dsub; ++j) rec[m * dsub + j] = cbh[(m * ks + cs[k * M + m]) * dsub + j];
        const float *x = &xs[k * d];
        for (size_t i = 0; i < d; ++i) {
          const double ri = rec[i];
          double *row = &cov[i * d];
          for (size_t j = 0; j < d; ++j) row[j] += ri * x[j];
        }
      }
      rmat = procrustes_rotation(cov, d);
    }
    ix->h_rotation = std::move(rmat);
    ix->optimized = true;
    VG_TRY(upload_rotation(ix));
  }
  ix->num_centroids = Lc;
  ix->trained = true;
  return VG_OK;
}

// Device copies of the host rotation: row-major for the encode GEMM and
// transposed for the scan kernels (coalesced loads of one column).
int upload_rotation(vg_index *ix) {
  const size_t d = ix->d;
  if (ix->h_rotation.empty()) {
    ix->rotation.release();
    ix->rotation_t.release();
    return VG_OK;
  }
  std::vector<float> rt(d * d);
  for (size_t i = 0; i < d; ++i)
    for (size_t j = 0; j < d; ++j) rt[j * d + i] = ix->h_rotation[i * d + j];
  VG_CU(ix->rotation.reserve(d * d * 4));
  VG_CU(ix->rotation_t.reserve(d * d * 4));
  VG_CU(cudaMemcpy(ix->rotation.p, ix->h_rotation.data(), d * d * 4, cudaMemcpyHostToDevice));
  VG_CU(cudaMemcpy(ix->rotation_t.p, rt.data(), d * d * 4, cudaMemcpyHostToDevice));
  return VG_OK;
}

// ---- encode and list layout (search.rs:620-848) ---------------------------

int build_list_storage(vg_index *ix, const uint32_t *sorted_lists);

int encode_and_layout(vg_index *ix) {
  cudaStream_t s = ix->stream;
  const size_t n = ix->n, d = ix->d, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const size_t Lc = ix->num_centroids;
  VG_CU(ix->assign.reserve(n * 4));
  VG_TRY(assign_rows_to_lists(ix, ix->vectors.as<float>(), n, ix->centroids.as<float>(), Lc,
                              ix->assign.as<uint32_t>(), nullptr, nullptr));
  VG_CU(ix->codes.reserve(n * M));
  if (ix->h_rotation.empty()) {
    VG_CU(launch_encode(ix->vectors.as<float>(), n, static_cast<int>(d), ix->assign.as<uint32_t>(),
                        ix->centroids.as<float>(), ix->codebooks.as<float>(), static_cast<int>(M),
                        static_cast<int>(ks), ix->codes.as<uint8_t>(), s));
  } else {
    // OPQ (opq.rs:107-113): quantise the rotated residual R (x - c)
    const size_t chunk = std::min(n, size_t(1) << 20);
    DevBuf res, rot;
    VG_CU(res.reserve(chunk * d * 4));
    VG_CU(rot.reserve(chunk * d * 4));
    for (size_t r0 = 0; r0 < n; r0 += chunk) {
      const size_t rows = std::min(chunk, n - r0);
      VG_CU(launch_residuals(ix->vectors.as<float>() + r0 * d, rows, static_cast<int>(d),
                             ix->assign.as<uint32_t>() + r0, ix->centroids.as<float>(), res.as<float>(), s));
      VG_CU(launch_rotate_rows(res.as<float>(), rows, static_cast<int>(d), ix->rotation.as<float>(),
                               rot.as<float>(), s));
      VG_CU(launch_encode_residuals(rot.as<float>(), rows, static_cast<int>(d), ix->codebooks.as<float>(),
                                    static_cast<int>(M), static_cast<int>(ks),
                                    ix->codes.as<uint8_t>() + r0 * M, s));
    }
    VG_CU(cudaStreamSynchronize(s));
  }

  // stable sort by list keeps insertion order inside each list
  DevBuf iota, sorted_lists, temp, seg;
  VG_CU(iota.reserve(n * 4));
  VG_CU(sorted_lists.reserve(n * 4));
  VG_CU(ix->list_ids.reserve(n * 4));
  VG_CU(seg.reserve((Lc + 1) * 4));
  VG_CU(launch_iota(iota.as<uint32_t>(), n, s));
  size_t temp_bytes = 0;
  VG_CU(sort_pairs_u32(nullptr, temp_bytes, nullptr, nullptr, nullptr, nullptr, n, 32, s));
  VG_CU(temp.reserve(temp_bytes));
  VG_CU(sort_pairs_u32(temp.p, temp_bytes, ix->assign.as<uint32_t>(), sorted_lists.as<uint32_t>(),
                       iota.as<uint32_t>(), ix->list_ids.as<uint32_t>(), n, 32, s));
  VG_CU(launch_segments(sorted_lists.as<uint32_t>(), n, Lc, seg.as<uint32_t>(), s));
  std::vector<uint32_t> hseg(Lc + 1);
  VG_CU(cudaMemcpyAsync(hseg.data(), seg.p, (Lc + 1) * 4, cudaMemcpyDeviceToHost, s));
  VG_CU(cudaStreamSynchronize(s));

  ix->h_list_off.assign(hseg.begin(), hseg.end());
  return build_list_storage(ix, sorted_lists.as<uint32_t>());
}

// List-contiguous code storage from the list layout: ix->h_list_off (host
// CSR offsets), ix->list_ids (device, vector ids in list order) and
// sorted_lists (device, the list of every position).  Gathers list_codes and,
// for 16-entry codebooks, the nibble-packed scan copy.
// 16-byte aligned byte offsets of every list's codes (M bytes per vector)
// and, for 16-entry codebooks, of its nibble-packed scan copy (lists of at
// least 16 vectors, ceil(M/2) bytes per vector), from CSR offsets `off`.
void list_layout(const std::vector<uint64_t> &off, size_t Lc, size_t M, size_t ks, std::vector<uint64_t> &code_off,
                 std::vector<uint64_t> &pack_off, uint64_t &code_bytes, uint64_t &pack_bytes) {
  code_off.assign(Lc, 0);
  pack_off.assign(Lc, 0);
  code_bytes = pack_bytes = 0;
  for (size_t l = 0; l < Lc; ++l) {
    const uint64_t len = off[l + 1] - off[l];
    code_off[l] = code_bytes;
    code_bytes += (len * M + 15) & ~uint64_t(15);
    pack_off[l] = pack_bytes;
    if (ks == 16 && len >= 16) pack_bytes += (len * ((M + 1) / 2) + 15) & ~uint64_t(15);
  }
}

int build_list_storage(vg_index *ix, const uint32_t *sorted_lists) {
  cudaStream_t s = ix->stream;
  const size_t n = ix->n, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const size_t Lc = ix->num_centroids;
  std::vector<uint64_t> h_code_off, h_pack_off;
  uint64_t code_bytes = 0, pack_bytes = 0;
  list_layout(ix->h_list_off, Lc, M, ks, h_code_off, h_pack_off, code_bytes, pack_bytes);
  VG_CU(ix->list_off.reserve((Lc + 1) * 8));
  VG_CU(ix->code_off.reserve(Lc * 8));
  VG_CU(ix->pack_off.reserve(Lc * 8));
  VG_CU(ix->list_codes.reserve(std::max<uint64_t>(code_bytes, 16)));
  VG_CU(cudaMemcpyAsync(ix->list_off.p, ix->h_list_off.data(), (Lc + 1) * 8, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->code_off.p, h_code_off.data(), Lc * 8, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->pack_off.p, h_pack_off.data(), Lc * 8, cudaMemcpyHostToDevice, s));
  VG_CU(launch_gather_list_codes(ix->codes.as<uint8_t>(), ix->list_ids.as<uint32_t>(), sorted_lists,
                                 n, static_cast<int>(M), ix->list_off.as<uint64_t>(), ix->code_off.as<uint64_t>(),
                                 ix->list_codes.as<uint8_t>(), s));
  if (ks == 16) {
    VG_CU(ix->packed.reserve(std::max<uint64_t>(pack_bytes, 16)));
    VG_CU(launch_pack_lists_4bit(ix->list_codes.as<uint8_t>(), ix->list_off.as<uint64_t>(),
                                 ix->code_off.as<uint64_t>(), ix->pack_off.as<uint64_t>(), Lc, static_cast<int>(M),
                                 ix->packed.as<uint8_t>(), s));
  }
  VG_CU(ix->list_radius.reserve(std::max<size_t>(Lc, 1) * 4));
  VG_CU(launch_list_radius(ix->list_codes.as<uint8_t>(), ix->code_off.as<uint64_t>(), ix->list_off.as<uint64_t>(), Lc,
                           static_cast<int>(M), static_cast<int>(ks), static_cast<int>(ix->dsub),
                           ix->codebooks.as<float>(), ix->list_radius.as<float>(), s));
  VG_CU(ix->sub_radius.reserve((M + 1) * 4));
  VG_CU(launch_subspace_radius(ix->codebooks.as<float>(), static_cast<int>(M), static_cast<int>(ks),
                               static_cast<int>(ix->dsub), ix->sub_radius.as<float>(), s));
  VG_TRY(prepare_centroids(ix));
  VG_CU(cudaStreamSynchronize(s));
  ix->built = true;
  return VG_OK;
}

// Keep only the lists this rank owns (mine[l] != 0): the device layout is
// rebuilt with every other list empty (list_off, code_off, pack_off) and the
// owned lists' ids, codes and packed codes gathered; the insertion-order codes
// and assignments are released.  Centroids, codebooks, pruning radii and the
// doc-id map stay whole (every rank selects probes and maps ids).
int partition_lists(vg_index *ix, const std::vector<uint8_t> &mine) {
  cudaStream_t s = ix->stream;
  const size_t Lc = ix->num_centroids, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const std::vector<uint64_t> &goff = ix->h_list_off;
  std::vector<uint64_t> gcode, gpack, lcode, lpack, loff(Lc + 1, 0);
  uint64_t gcb = 0, gpb = 0, lcb = 0, lpb = 0;
  list_layout(goff, Lc, M, ks, gcode, gpack, gcb, gpb);
  for (size_t l = 0; l < Lc; ++l) loff[l + 1] = loff[l] + (mine[l] ? goff[l + 1] - goff[l] : 0);
  list_layout(loff, Lc, M, ks, lcode, lpack, lcb, lpb);
  // segments to gather: ids, codes and (4-bit) packed codes of owned lists
  std::vector<uint64_t> seg;  // [3][count] src, dst, bytes per table
  auto build = [&](int table, std::vector<uint64_t> &src, std::vector<uint64_t> &dst, std::vector<uint64_t> &bytes) {
    for (size_t l = 0; l < Lc; ++l) {
      const uint64_t len = goff[l + 1] - goff[l];
      if (!mine[l] || len == 0) continue;
      if (table == 0) {
        src.push_back(goff[l] * 4);
        dst.push_back(loff[l] * 4);
        bytes.push_back(len * 4);
      } else if (table == 1) {
        src.push_back(gcode[l]);
        dst.push_back(lcode[l]);
        bytes.push_back(len * M);
      } else if (len >= 16) {
        src.push_back(gpack[l]);
        dst.push_back(lpack[l]);
        bytes.push_back(len * ((M + 1) / 2));
      }
    }
  };
  DevBuf n_ids, n_codes, n_packed, offs;
  VG_CU(n_ids.reserve(std::max<uint64_t>(loff[Lc] * 4, 16)));
  VG_CU(n_codes.reserve(std::max<uint64_t>(lcb, 16)));
  if (ks == 16) VG_CU(n_packed.reserve(std::max<uint64_t>(lpb, 16)));
  for (int table = 0; table < (ks == 16 ? 3 : 2); ++table) {
    std::vector<uint64_t> src, dst, bytes;
    build(table, src, dst, bytes);
    const size_t cnt = src.size();
    if (!cnt) continue;
    std::vector<uint64_t> h(3 * cnt);
    std::copy(src.begin(), src.end(), h.begin());
    std::copy(dst.begin(), dst.end(), h.begin() + cnt);
    std::copy(bytes.begin(), bytes.end(), h.begin() + 2 * cnt);
    VG_CU(offs.reserve(h.size() * 8));
    VG_CU(cudaMemcpyAsync(offs.p, h.data(), h.size() * 8, cudaMemcpyHostToDevice, s));
    const void *from = table == 0 ? ix->list_ids.p : table == 1 ? ix->list_codes.p : ix->packed.p;
    void *to = table == 0 ? n_ids.p : table == 1 ? n_codes.p : n_packed.p;
    VG_CU(launch_copy_segments(from, to, offs.as<uint64_t>(), offs.as<uint64_t>() + cnt, offs.as<uint64_t>() + 2 * cnt,
                               cnt, s));
    VG_CU(cudaStreamSynchronize(s));  // offs is reused by the next table
  }
  VG_CU(cudaMemcpyAsync(ix->list_off.p, loff.data(), (Lc + 1) * 8, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->code_off.p, lcode.data(), Lc * 8, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->pack_off.p, lpack.data(), Lc * 8, cudaMemcpyHostToDevice, s));
  VG_CU(cudaStreamSynchronize(s));
  ix->list_ids = std::move(n_ids);
  ix->list_codes = std::move(n_codes);
  if (ks == 16) ix->packed = std::move(n_packed);
  ix->codes.release();
  ix->assign.release();
  ix->partitioned = true;
  return VG_OK;
}

// ---- search -------------------------------------------------------------

// The nprobe nearest lists of rows normalised queries qn (search.rs:1602-1617:
// 1 - q.c in sequential f32, ascending, ties by list id) into probes / pdist
// (row stride P).  Many lists: tensor-core products with the fused candidate
// window (tc_select.cu) -- the same probes as the exact path, no product
// matrix in memory.  Few lists, rows beyond 128 floats or centroids too long
// for a useful error bound: the exact distance tile (ws_dist, rows x Lc) and
// a row selection.  Calls mark(3) between the two phases; adds the number of
// this library's kernels launched to *launches.
int coarse_probes(vg_index *ix, const float *qn, size_t rows, size_t P, uint32_t *probes, float *pdist,
                  uint64_t *launches, const ProbeBoundArgs *bounds = nullptr, bool *bounds_done = nullptr) {
  if (bounds_done) *bounds_done = false;
  cudaStream_t s = ix->stream;
  const size_t Lc = ix->num_centroids, d = ix->d;
  if (coarse_via_products(ix, P)) {
    // binary16 products of the tile (f32 accumulation, rounded once more to
    // binary16: 2^-11 of |q| |c| on top of the window's coefficients), then the
    // shortlist re-scores every list the bound cannot rule out
    const int kp = ix->cent_kp;
    double rel = 0, abs_coef = 0;
    tc_error_coefs(static_cast<int>(d), &rel, &abs_coef);
    rel += 1.0 / 2048;
    VG_CU(ix->ws_qimg.reserve(umma_image_bytes(rows, kp)));
    VG_CU(ix->ws_dist.reserve(std::max<size_t>(rows * Lc, 1) * 2));
    const size_t cstride = (Lc + 127) / 128 * 4;  // chunk maxima of 32 products per row
    VG_CU(ix->ws_cmax.reserve(std::max<size_t>(rows * cstride, 1) * 2));
    VG_CU(launch_umma_image(qn, rows, static_cast<int>(d), kp, ix->ws_qimg.p, nullptr, 0.0, 0.0, nullptr, s));
    VG_CU(launch_tc_gemm_f16(ix->ws_qimg.p, rows, ix->cent_img.p, Lc, static_cast<int>(d), kp, ix->ws_dist.p, Lc,
                             ix->ws_cmax.p, cstride, ix->d_err, ix->num_sms, s));
    mark(ix, 3);
    VG_CU(launch_probe_shortlist(ix->ws_dist.p, true, rows, Lc, Lc, qn, static_cast<int>(d),
                                 ix->centroids.as<float>(), ix->cent_norm.as<float>(), rel, abs_coef,
                                 static_cast<int>(P), probes, pdist, P, bounds ? *bounds : ProbeBoundArgs{}, s,
                                 ix->ws_cmax.p, cstride));
    *launches += 3;
    if (bounds_done) *bounds_done = bounds != nullptr;
    return VG_OK;
  }
  if (coarse_on_tensor_cores(ix, P)) {
    const int kp = ix->cent_kp;
    double rel = 0, abs_coef = 0;
    tc_error_coefs(static_cast<int>(d), &rel, &abs_coef);
    VG_CU(ix->ws_qimg.reserve(umma_image_bytes(rows, kp)));
    VG_CU(ix->ws_eps.reserve(rows * 4));
    VG_CU(ix->ws_tc.reserve(tc_select_workspace_bytes(rows, Lc, static_cast<int>(P), ix->num_sms)));
    VG_CU(launch_umma_image(qn, rows, static_cast<int>(d), kp, ix->ws_qimg.p, ix->cent_norm.as<float>(), rel,
                            abs_coef, ix->ws_eps.as<float>(), s));
    mark(ix, 3);
    TcSelect t{};
    t.a_img = ix->ws_qimg.p;
    t.q = qn;
    t.rows = rows;
    t.b_img = ix->cent_img.p;
    t.x = ix->centroids.as<float>();
    t.cols = Lc;
    t.d = static_cast<int>(d);
    t.kp = kp;
    t.P = static_cast<int>(P);
    t.mode = 0;
    t.eps = ix->ws_eps.as<float>();
    t.workspace = ix->ws_tc.p;
    t.out_ids = probes;
    t.out_dist = pdist;
    t.out_ld = P;
    if (bounds) t.bnd = *bounds;
    t.error = ix->d_err;
    VG_CU(launch_tc_select(t, ix->num_sms, s));
    *launches += 3;
    if (bounds_done) *bounds_done = bounds != nullptr;
    return VG_OK;
  }
  VG_CU(ix->ws_dist.reserve(rows * Lc * 4));
  VG_CU(launch_coarse_dist(qn, rows, ix->centroids.as<float>(), Lc, static_cast<int>(d), ix->ws_dist.as<float>(), Lc,
                           s));
  mark(ix, 3);
  VG_CU(launch_select_rows(ix->ws_dist.as<float>(), rows, Lc, Lc, static_cast<int>(P), probes, pdist, P, 0, s));
  *launches += 2;
  return VG_OK;
}

// Query rows per tile of the coarse stage: the exact path holds a tile of f32
// distances (kDistBudgetBytes), the tensor-core path its candidate lists.
size_t coarse_tile(const vg_index *ix, size_t nq, size_t P) {
  const size_t Lc = std::max<size_t>(ix->num_centroids, 1);
  size_t tile;
  if (coarse_via_products(ix, P)) {
    tile = std::max<size_t>(128, kDistBudgetBytes / (Lc * 2));
  } else if (coarse_on_tensor_cores(ix, P)) {
    const size_t est = std::min<size_t>(std::max<size_t>(nq, 1), size_t(1) << 20);
    const size_t per_row = tc_select_workspace_bytes(est, Lc, static_cast<int>(P), ix->num_sms) / est + 1;
    tile = std::max<size_t>(1024, kDistBudgetBytes / per_row);
  } else {
    tile = std::max<size_t>(1, kDistBudgetBytes / (Lc * 4));
  }
  tile = std::min(nq, tile);
  if (ix->coarse_tile_rows) tile = std::min(tile, ix->coarse_tile_rows);
  return std::max<size_t>(tile, 1);
}

int write_padding(vg_index *ix, size_t nq, size_t k, uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  std::vector<uint32_t> ids(nq * k, 0xffffffffu), cnt(nq, 0);
  std::vector<float> dist(nq * k, __builtin_inff());
  if (nq * k) {
    VG_CU(cudaMemcpyAsync(out_ids, ids.data(), nq * k * 4, cudaMemcpyDefault, ix->stream));
    VG_CU(cudaMemcpyAsync(out_dist, dist.data(), nq * k * 4, cudaMemcpyDefault, ix->stream));
  }
  if (out_count && nq) VG_CU(cudaMemcpyAsync(out_count, cnt.data(), nq * 4, cudaMemcpyDefault, ix->stream));
  VG_CU(cudaStreamSynchronize(ix->stream));
  return VG_OK;
}

// Scan-kernel parameters common to every search launch: the device layout
// and the probe workspaces.
vg::ScanParams base_scan_params(vg_index *ix, size_t P, size_t kk, bool prune, bool recs, bool quant) {
  vg::ScanParams sp{};
  sp.qn = ix->ws_qn.as<float>();
  sp.centroids = ix->centroids.as<float>();
  sp.codebooks = ix->codebooks.as<float>();
  sp.probes = ix->ws_probes.as<uint32_t>();
  sp.owner = ix->world > 1 ? ix->owner.as<uint8_t>() : nullptr;  // (the sharded search sets it)
  sp.list_off = ix->list_off.as<uint64_t>();
  sp.code_off = ix->code_off.as<uint64_t>();
  sp.list_codes = ix->list_codes.as<uint8_t>();
  sp.pack_off = ix->pack_off.as<uint64_t>();
  sp.packed = ix->packed.as<uint8_t>();
  sp.list_ids = ix->list_ids.as<uint32_t>();
  sp.doc_ids = ix->doc_ids.as<uint32_t>();
  sp.rot_t = ix->h_rotation.empty() ? nullptr : ix->rotation_t.as<float>();
  sp.probe_lb = prune ? ix->ws_lb.as<float>() : nullptr;
  sp.probe_rec = recs ? ix->ws_rec.as<ProbeRec>() : nullptr;
  sp.probe_lbq = quant ? ix->ws_lbq.as<float>() : nullptr;
  sp.d = static_cast<int>(ix->d);
  sp.M = static_cast<int>(ix->params.num_codebooks);
  sp.ks = static_cast<int>(ix->params.codebook_size);
  sp.dsub = static_cast<int>(ix->dsub);
  sp.P = static_cast<int>(P);
  sp.k = static_cast<int>(kk);
  sp.error = ix->d_err;
  return sp;
}

// Pruning bounds (and probe records) written for probe rows from r0 on.
ProbeBoundArgs bound_args_at(vg_index *ix, size_t P, size_t r0, bool prune, bool recs, bool quant) {
  return ProbeBoundArgs{ix->list_radius.as<float>(), static_cast<int>(ix->params.num_codebooks),
                        static_cast<int>(ix->dsub), ix->list_off.as<uint64_t>(), ix->code_off.as<uint64_t>(),
                        ix->world > 1 ? ix->owner.as<uint8_t>() : nullptr,
                        prune ? ix->ws_lb.as<float>() + r0 * P : nullptr,
                        recs ? ix->ws_rec.as<ProbeRec>() + r0 * P : nullptr, ix->sub_radius.as<float>(),
                        quant ? ix->ws_lbq.as<float>() + r0 * P : nullptr};
}


int nccl_ok(vg_index *ix, ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return VG_OK;
  if (r == ncclInProgress) return nccl_wait_ready(ix->comm, ix->comm_timeout_ms);
  return fail(VG_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

// Search on a list-sharded index (every rank holds the lists it owns).  Each
// rank passes a batch of its own, the same size on every rank, and receives
// the results of its own queries:
//   1. normalise and select the probes of its own queries (with their
//      pruning bounds, valid on every rank);
//   2. all-gather queries, probes and bounds: every rank holds the global
//      batch (world * nq rows, rank r's rows at r * nq);
//   3. seed: the rank owning a query's nearest list scores it (and its own
//      next lists until it keeps k keys); an all-reduce (min) of every
//      query's k-th key gives every rank a bound on the query's k-th key over
//      every list, the one a single GPU has after those lists;
//   4. every rank scans its lists among the remaining probes for the global
//      batch in units of kUnitProbes probes per query, keeping only keys at or
//      below the bound, and merges each query's units with its seed keys;
//   5. an all-to-all returns every query's per-rank top-k to the query's rank,
//      which merges them (the reference's per-shard top-k merge,
//      examples/large_scale.rs:1969-2025).
// Without pruning bounds (an OPQ rotation) the seed is skipped.
int search_sharded(vg_index *ix, const float *queries, size_t nq, size_t k, size_t pool, size_t nprobe,
                   uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  const bool rerank = pool > 0;
  if (rerank && ix->compacted)
    return fail(VG_ERR_UNSUPPORTED,
                "unsupported: search_reranked after compact(); use search() instead, or keep raw vectors");
  const size_t kk = rerank ? std::max(pool, k) : k;
  if (kk > 256) return fail(VG_ERR_UNSUPPORTED, "unsupported: candidate_pool above 256 on a sharded index");
  const size_t Lc = ix->num_centroids, d = ix->d, M = ix->params.num_codebooks;
  const size_t P = std::min(nprobe ? nprobe : static_cast<size_t>(ix->params.nprobe), Lc);
  if (nq == 0 || k == 0 || P == 0) return write_padding(ix, nq, k, out_ids, out_dist, out_count);
  if (!queries || !out_ids || !out_dist) return fail(VG_ERR_INVALID_PARAMETER, "null query or output buffer");
  const size_t W = static_cast<size_t>(ix->world), R = static_cast<size_t>(ix->rank), B = W * nq;
  if (B * P > 0xffffffffull || B > 0x7fffffffull)
    return fail(VG_ERR_INVALID_PARAMETER, "world_size * nq * nprobe must fit in 32 bits");
  cudaStream_t s = ix->stream;
  const bool prof = ix->profiling;
  const uint64_t launches0 = ix->launches;
  ix->tile_marks = nullptr;
  *reinterpret_cast<volatile int *>(ix->h_err) = 0;
  mark(ix, 0);
  const float *dq = queries;
  if (!is_device_ptr(queries)) {
    VG_CU(ix->ws_q.reserve(nq * d * 4));
    VG_CU(cudaMemcpyAsync(ix->ws_q.p, queries, nq * d * 4, cudaMemcpyHostToDevice, s));
    dq = ix->ws_q.as<float>();
  }
  mark(ix, 1);
  const bool prune = ix->h_rotation.empty();
  const bool recs = prune && ix->params.codebook_size == 256;
  const bool quant = prune && ix->params.codebook_size == 16;
  VG_CU(ix->ws_qall.reserve(B * d * 4));
  VG_CU(ix->ws_probes.reserve(B * P * 4));
  VG_CU(ix->ws_pdist.reserve(B * P * 4));
  VG_CU(ix->ws_lb.reserve(B * P * 4));
  if (quant) VG_CU(ix->ws_lbq.reserve(B * P * 4));
  if (recs) VG_CU(ix->ws_rec.reserve(B * P * sizeof(ProbeRec)));
  // every query's k-th key and the probe its main pass starts from; the
  // per-unit keys [1 + U][B][kk] (row 0: the seed's); the work lists
  const size_t U = (P + kUnitProbes - 1) / kUnitProbes;
  VG_CU(ix->ws_seed.reserve(B * 8 + B * 4));
  VG_CU(ix->ws_units.reserve((U + 1) * B * kk * 8));
  VG_CU(ix->ws_work.reserve(B * U * 4));
  VG_CU(ix->ws_keys.reserve(B * kk * 8));
  VG_CU(ix->ws_all_keys.reserve(B * kk * 8));
  float *qall = ix->ws_qall.as<float>(), *qown = qall + R * nq * d;
  uint32_t *pown = ix->ws_probes.as<uint32_t>() + R * nq * P;
  VG_CU(launch_normalize_rows(dq, nq, static_cast<int>(d), qown, s));
  ix->launches += 1;
  mark(ix, 2);

  // 1. probes of this rank's queries, with bounds for every probe
  const size_t tile = coarse_tile(ix, nq, P);
  for (size_t r0 = 0; r0 < nq; r0 += tile) {
    const size_t rows = std::min(tile, nq - r0);
    ProbeBoundArgs ba = bound_args_at(ix, P, R * nq + r0, prune, false, quant);
    ba.owner = nullptr;  // bounds of every probe: other ranks scan with them
    bool done = false;
    VG_TRY(coarse_probes(ix, qown + r0 * d, rows, P, pown + r0 * P, ix->ws_pdist.as<float>() + (R * nq + r0) * P,
                         &ix->launches, prune ? &ba : nullptr, &done));
    if (prune && !done) {
      VG_CU(launch_probe_lb(qown + r0 * d, rows, static_cast<int>(d), pown + r0 * P, static_cast<int>(P),
                            ix->centroids.as<float>(), ba, s));
      ix->launches += 1;
    }
  }
  mark(ix, 4);

  // 2. the global batch on every rank (in place: rank r's block is its own)
  VG_TRY(nccl_ok(ix, ncclGroupStart(), "ncclGroupStart"));
  ncclAllGather(qown, qall, nq * d, ncclFloat32, ix->comm, s);
  ncclAllGather(pown, ix->ws_probes.p, nq * P, ncclUint32, ix->comm, s);
  if (prune) ncclAllGather(ix->ws_lb.as<float>() + R * nq * P, ix->ws_lb.p, nq * P, ncclFloat32, ix->comm, s);
  if (quant) ncclAllGather(ix->ws_lbq.as<float>() + R * nq * P, ix->ws_lbq.p, nq * P, ncclFloat32, ix->comm, s);
  VG_TRY(nccl_ok(ix, ncclGroupEnd(), "ncclAllGather (queries, probes, bounds)"));
  mark(ix, 5);
  if (recs) {
    VG_CU(launch_probe_records(ix->ws_probes.as<uint32_t>(), ix->ws_lb.as<float>(), B * P, ix->owner.as<uint8_t>(),
                               ix->list_off.as<uint64_t>(), ix->code_off.as<uint64_t>(), ix->ws_rec.as<ProbeRec>(),
                               s));
    ix->launches += 1;
  }
  VG_CU(ix->ws_scalars.reserve(64));
  uint32_t *d_counter = ix->ws_scalars.as<uint32_t>();
  uint32_t *d_wcount = d_counter + 2;  // the work list's two counts
  vg::ScanParams sp = base_scan_params(ix, P, kk, prune, recs, quant);
  sp.qn = qall;
  sp.owner = ix->owner.as<uint8_t>();
  sp.counter = d_counter;
  sp.scored = prof ? ix->stats.as<unsigned long long>() + 3 : nullptr;
  sp.nq = static_cast<int>(B);
  sp.force_warp = 1;
  if (prof) {
    VG_CU(launch_probe_stats(ix->ws_probes.as<uint32_t>(), B, static_cast<int>(P), ix->owner.as<uint8_t>(), Lc,
                             ix->list_off.as<uint64_t>(), static_cast<int>(M), ix->params.codebook_size == 16,
                             ix->stats.as<unsigned long long>(), s));
  }

  // 3. seed: the rank that owns a query's nearest list scores it as one GPU
  // would (no bound yet), and its own next lists until it keeps k keys -- any
  // k keys bound the query's k-th key over every list.  The other ranks score
  // nothing here (an unbounded first list on every rank would be work one GPU
  // never does).  The bound travels as a min over ranks of every query's k-th
  // key; each query's main pass resumes after the lists its seed scored.
  const bool seeded = prune && P > 1 && ivfpq_scan_warp_applies(sp);
  unsigned long long *unit_keys = ix->ws_units.as<unsigned long long>();  // [1 + U][B][kk]
  unsigned long long *ceiling = ix->ws_seed.as<unsigned long long>();    // [B]
  uint32_t *resume = reinterpret_cast<uint32_t *>(ceiling + B);          // [B]
  uint32_t *work = ix->ws_work.as<uint32_t>();
  if (seeded) {
    // 3. seed pass over the queries whose nearest list is this rank's
    VG_CU(cudaMemsetAsync(unit_keys, 0xff, (U + 1) * B * kk * 8, s));
    VG_CU(cudaMemsetAsync(ceiling, 0xff, B * 8, s));
    VG_CU(cudaMemsetAsync(d_counter, 0, 16, s));
    VG_CU(launch_order_seed(ix->ws_probes.as<uint32_t>(), static_cast<int>(P), ix->owner.as<uint8_t>(),
                            ix->list_off.as<uint64_t>(), B, kHeavyVectors, work, d_wcount,
                            static_cast<uint32_t>(B * U), resume, s));
    sp.work = work;
    sp.work_count = d_wcount;
    sp.work_cap = static_cast<uint32_t>(B * U);
    sp.seed_next = resume;
    sp.out_keys = unit_keys;
    sp.out_kth = ceiling;
    unsigned long long *main_counters = sp.scored;
    if (prof) sp.scored = ix->stats.as<unsigned long long>() + 7;
    VG_CU(vg::launch_ivfpq_scan(sp, ix->num_sms, s));
    ix->launches += 2;
    mark(ix, 6);
    // one rank holds each query's seed keys (kEmptyKey elsewhere): min over ranks
    VG_TRY(nccl_ok(ix, ncclAllReduce(ceiling, ceiling, B, ncclUint64, ncclMin, ix->comm, s),
                   "ncclAllReduce (seed bounds)"));
    mark(ix, 7);
    // 4. units of this rank's lists for the global batch, bounded by the
    // ceiling, heavy ones first; then every query's keys merged over its units
    VG_CU(cudaMemsetAsync(d_counter, 0, 16, s));
    VG_CU(launch_order_units(ix->ws_probes.as<uint32_t>(), static_cast<int>(P), kUnitProbes,
                             ix->owner.as<uint8_t>(), ix->list_off.as<uint64_t>(),
                             quant ? ix->ws_lbq.as<float>() : ix->ws_lb.as<float>(), ceiling, resume, B,
                             kHeavyVectors, work, d_wcount, static_cast<uint32_t>(B * U), s));
    sp.seed_next = nullptr;
    sp.out_kth = nullptr;
    sp.probe_from = resume;
    sp.unit_probes = kUnitProbes;
    sp.key_ceiling = ceiling;
    sp.scored = main_counters;
    VG_CU(vg::launch_ivfpq_scan(sp, ix->num_sms, s));
    VG_CU(launch_merge_shards(unit_keys, static_cast<int>(U + 1), B, static_cast<int>(kk), nullptr, nullptr,
                              nullptr, nullptr, ix->ws_keys.as<unsigned long long>(), s));
    ix->launches += 3;
  } else {
    mark(ix, 6);
    mark(ix, 7);
    // 4. this rank's lists for the global batch
    sp.out_keys = ix->ws_keys.as<unsigned long long>();
    VG_CU(cudaMemsetAsync(d_counter, 0, 4, s));
    VG_CU(vg::launch_ivfpq_scan(sp, ix->num_sms, s));
    ix->launches += 1;
  }
  mark(ix, 8);

  // 5. every query's per-rank keys to its rank: [W][nq][kk]
  VG_TRY(nccl_ok(ix, ncclGroupStart(), "ncclGroupStart"));
  for (size_t r = 0; r < W; ++r) {
    ncclSend(ix->ws_keys.as<unsigned long long>() + r * nq * kk, nq * kk, ncclUint64, static_cast<int>(r), ix->comm, s);
    ncclRecv(ix->ws_all_keys.as<unsigned long long>() + r * nq * kk, nq * kk, ncclUint64, static_cast<int>(r), ix->comm,
             s);
  }
  VG_TRY(nccl_ok(ix, ncclGroupEnd(), "ncclSend/ncclRecv (per-rank keys)"));
  mark(ix, 9);
  const bool dev_out = is_device_ptr(out_ids) && is_device_ptr(out_dist) && (!out_count || is_device_ptr(out_count));
  uint32_t *o_ids = out_ids, *o_cnt = out_count;
  float *o_dist = out_dist;
  if (!dev_out) {
    VG_CU(ix->ws_out_ids.reserve(nq * k * 4));
    VG_CU(ix->ws_out_dist.reserve(nq * k * 4));
    VG_CU(ix->ws_out_count.reserve(nq * 4));
    o_ids = ix->ws_out_ids.as<uint32_t>();
    o_dist = ix->ws_out_dist.as<float>();
    o_cnt = ix->ws_out_count.as<uint32_t>();
  }
  const uint32_t *doc_map = ix->doc_ids.as<uint32_t>();
  if (rerank) {
    VG_CU(launch_merge_shards(ix->ws_all_keys.as<unsigned long long>(), static_cast<int>(W), nq, static_cast<int>(kk),
                              nullptr, nullptr, nullptr, nullptr, ix->ws_keys.as<unsigned long long>(), s));
    VG_CU(launch_rerank(qown, ix->vectors.as<float>(), static_cast<int>(d), ix->ws_keys.as<unsigned long long>(), nq,
                        static_cast<int>(kk), static_cast<int>(k), doc_map, o_ids, o_dist, o_cnt, s));
    ix->launches += 2;
  } else {
    VG_CU(launch_merge_shards(ix->ws_all_keys.as<unsigned long long>(), static_cast<int>(W), nq, static_cast<int>(k),
                              doc_map, o_ids, o_dist, o_cnt, nullptr, s));
    ix->launches += 1;
  }
  mark(ix, 10);
  if (!dev_out) {
    VG_CU(cudaMemcpyAsync(out_ids, o_ids, nq * k * 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaMemcpyAsync(out_dist, o_dist, nq * k * 4, cudaMemcpyDeviceToHost, s));
    if (out_count) VG_CU(cudaMemcpyAsync(out_count, o_cnt, nq * 4, cudaMemcpyDeviceToHost, s));
  }
  mark(ix, 11);
  VG_TRY(sync_stream(ix));
  VG_TRY(check_device_error(ix, "sharded search"));
  if (prof) {
    auto el = [&](int a, int b) {
      float ms = 0;
      cudaEventElapsedTime(&ms, ix->ev[a], ix->ev[b]);
      return static_cast<double>(ms);
    };
    vg_search_profile &pf = ix->prof;
    pf.h2d_ms += el(0, 1);
    pf.normalize_ms += el(1, 2);
    pf.coarse_ms += el(2, 3);
    pf.select_ms += el(3, 4);
    pf.collective_ms += el(4, 5) + (seeded ? el(6, 7) : 0.0) + el(8, 9);
    pf.pairs_ms += el(5, 6);  // probe records and the seed scan
    pf.scan_ms += el(7, 8);
    pf.merge_ms += el(9, 10);
    pf.d2h_ms += el(10, 11);
    pf.total_ms += el(0, 11);
    pf.calls += 1;
    pf.queries += nq;
    pf.kernel_launches += ix->launches - launches0;
    pf.scan_launches += seeded ? 2 : 1;
  }
  return VG_OK;
}

int search_impl(vg_index *ix, const float *queries, size_t nq, size_t k, size_t pool, size_t nprobe,
                uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  if (!ix->built) return fail(VG_ERR_NOT_BUILT, "IVF-PQ index is not built: cannot search");
  if (k > 256) return fail(VG_ERR_INVALID_PARAMETER, "k must be at most 256");
  if (ix->world > 1) return search_sharded(ix, queries, nq, k, pool, nprobe, out_ids, out_dist, out_count);
  ix->tile_marks = nullptr;  // a call that failed mid-stage may have left it set
  const bool rerank = pool > 0;
  if (rerank && ix->compacted)
    return fail(VG_ERR_UNSUPPORTED,
                "unsupported: search_reranked after compact(); use search() instead, or keep raw vectors");
  const size_t kk = rerank ? std::max(pool, k) : k;
  if (kk > (size_t{1} << 20)) return fail(VG_ERR_INVALID_PARAMETER, "candidate_pool must be at most 1048576");
  if (nq == 0 || k == 0) return write_padding(ix, nq, k, out_ids, out_dist, out_count);
  if ((nq && !queries) || !out_ids || !out_dist)
    return fail(VG_ERR_INVALID_PARAMETER, "null query or output buffer");
  const size_t Lc = ix->num_centroids, d = ix->d, M = ix->params.num_codebooks;
  const size_t P = std::min(nprobe ? nprobe : static_cast<size_t>(ix->params.nprobe), Lc);
  if (P == 0) return write_padding(ix, nq, k, out_ids, out_dist, out_count);
  if (nq * P > 0xffffffffull) return fail(VG_ERR_INVALID_PARAMETER, "nq * nprobe must fit in 32 bits");
  cudaStream_t s = ix->stream;
  const bool prof = ix->profiling;
  uint64_t launches0 = ix->launches;

  *reinterpret_cast<volatile int *>(ix->h_err) = 0;
  // coarse distances + top-nprobe, tiled over queries.  Host queries of a
  // large batch arrive in (at least two) tiles on the copy stream: a tile's
  // coarse stage waits only for its own rows, so the upload of the later
  // rows runs under the products and shortlist of the earlier ones.
  const bool host_q = !is_device_ptr(queries);
  size_t tile = coarse_tile(ix, nq, P);
  const bool pipe = host_q && nq >= kPipeMinRows;
  if (pipe) tile = std::min(tile, ((nq + 1) / 2 + 127) / 128 * 128);
  const size_t ntiles = (nq + tile - 1) / tile;
  mark(ix, 0);
  const float *dq = queries;
  if (host_q) {
    VG_CU(ix->ws_q.reserve(nq * d * 4));
    dq = ix->ws_q.as<float>();
    if (pipe) {
      VG_CU(reserve_copy_pipeline(ix, ntiles));
      // the copies start when the stream reaches this call, not earlier
      VG_CU(cudaEventRecord(ix->copy_start, s));
      VG_CU(cudaStreamWaitEvent(ix->copy_stream, ix->copy_start, 0));
      for (size_t t = 0; t < ntiles; ++t) {
        const size_t r0 = t * tile, rows = std::min(tile, nq - r0);
        VG_CU(cudaMemcpyAsync(ix->ws_q.as<float>() + r0 * d, queries + r0 * d, rows * d * 4, cudaMemcpyHostToDevice,
                              ix->copy_stream));
        VG_CU(cudaEventRecord(ix->copy_ev[t], ix->copy_stream));
      }
    } else {
      VG_CU(cudaMemcpyAsync(ix->ws_q.p, queries, nq * d * 4, cudaMemcpyHostToDevice, s));
    }
  }
  VG_CU(ix->ws_qn.reserve(nq * d * 4));
  if (!pipe) {
    mark(ix, 1);
    VG_CU(launch_normalize_rows(dq, nq, static_cast<int>(d), ix->ws_qn.as<float>(), s));
    ix->launches += 1;
    mark(ix, 2);
  }
  VG_CU(ix->ws_probes.reserve(nq * P * 4));
  VG_CU(ix->ws_pdist.reserve(nq * P * 4));
  // list pruning bounds (tables without a rotation; see launch_probe_lb)
  // and, for 256-entry codebooks, the probe records the streaming kernel
  // copies whole: written by the probe shortlist when it runs, else below
  const bool prune = ix->h_rotation.empty();
  const bool recs = prune && ix->params.codebook_size == 256;
  const bool quant = prune && ix->params.codebook_size == 16;  // bounds of quantised 4-bit distances
  if (prune) {
    VG_CU(ix->ws_lb.reserve(nq * P * 4));
    if (recs) VG_CU(ix->ws_rec.reserve(nq * P * sizeof(ProbeRec)));
    if (quant) VG_CU(ix->ws_lbq.reserve(nq * P * 4));
  }
  auto bound_args = [&](size_t r0) { return bound_args_at(ix, P, r0, prune, recs, quant); };
  bool bounds_done = prune;
  // a profiled tiled stage times each tile on its own events (no host wait
  // between tiles); with the copy pipeline, normalising a later tile's rows
  // falls between those events
  const bool tiled_prof = prof && ntiles > 1;
  if (tiled_prof) VG_CU(reserve_tile_events(ix, 3 * ntiles));
  for (size_t r0 = 0, t = 0; r0 < nq; r0 += tile, ++t) {
    size_t rows = std::min(tile, nq - r0);
    if (pipe) {
      ix->tile_marks = nullptr;
      VG_CU(cudaStreamWaitEvent(s, ix->copy_ev[t], 0));
      if (t == 0) mark(ix, 1);
      VG_CU(launch_normalize_rows(dq + r0 * d, rows, static_cast<int>(d), ix->ws_qn.as<float>() + r0 * d, s));
      ix->launches += 1;
      if (t == 0) mark(ix, 2);
    }
    const ProbeBoundArgs ba = bound_args(r0);
    bool tile_done = false;
    if (tiled_prof) {
      ix->tile_marks = ix->tile_ev.data() + 3 * t;
      mark(ix, 2);
    }
    VG_TRY(coarse_probes(ix, ix->ws_qn.as<float>() + r0 * d, rows, P, ix->ws_probes.as<uint32_t>() + r0 * P,
                         ix->ws_pdist.as<float>() + r0 * P, &ix->launches, prune ? &ba : nullptr, &tile_done));
    bounds_done = bounds_done && tile_done;
    mark(ix, 4);
  }
  ix->tile_marks = nullptr;
  if (tiled_prof) mark(ix, 4);

  // per-query fused scan: probes -> (residual, table, scan, top-k) on chip
  VG_CU(ix->ws_scalars.reserve(64));
  uint32_t *d_counter = ix->ws_scalars.as<uint32_t>();
  VG_CU(cudaMemsetAsync(d_counter, 0, 16, s));  // the kernel's item counter, the work list's counts
  if (prof) {
    VG_CU(launch_probe_stats(ix->ws_probes.as<uint32_t>(), nq, static_cast<int>(P),
                             ix->world > 1 ? ix->owner.as<uint8_t>() : nullptr, Lc, ix->list_off.as<uint64_t>(),
                             static_cast<int>(M), ix->params.codebook_size == 16,
                             ix->stats.as<unsigned long long>(), s));
  }
  if (prune && !bounds_done) {
    VG_CU(launch_probe_lb(ix->ws_qn.as<float>(), nq, static_cast<int>(d), ix->ws_probes.as<uint32_t>(),
                          static_cast<int>(P), ix->centroids.as<float>(), bound_args(0), s));
    ix->launches += 1;
  }
  mark(ix, 5);

  // outputs: device pointers are written in place, host ones via staging
  const bool dev_out = is_device_ptr(out_ids) && is_device_ptr(out_dist) && (!out_count || is_device_ptr(out_count));
  uint32_t *o_ids = out_ids, *o_cnt = out_count;
  float *o_dist = out_dist;
  if (!dev_out) {
    VG_CU(ix->ws_out_ids.reserve(nq * k * 4));
    VG_CU(ix->ws_out_dist.reserve(nq * k * 4));
    VG_CU(ix->ws_out_count.reserve(nq * 4));
    o_ids = ix->ws_out_ids.as<uint32_t>();
    o_dist = ix->ws_out_dist.as<float>();
    o_cnt = ix->ws_out_count.as<uint32_t>();
  }
  const uint32_t *doc_map = ix->doc_ids.as<uint32_t>();
  const bool direct = !rerank;  // the kernel writes final results

  vg::ScanParams sp = base_scan_params(ix, P, kk, prune, recs, quant);
  sp.counter = d_counter;
  sp.scored = prof ? ix->stats.as<unsigned long long>() + 3 : nullptr;
  sp.doc_ids = doc_map;
  sp.nq = static_cast<int>(nq);
  if (direct) {
    sp.out_ids = o_ids;
    sp.out_dist = o_dist;
    sp.out_count = o_cnt;
  } else {
    VG_CU(ix->ws_keys.reserve(nq * kk * 8));
    sp.out_keys = ix->ws_keys.as<unsigned long long>();
  }
  if (kk <= 256) {
    if (prune && ivfpq_scan_warp_applies(sp)) {
      // queries whose nearest list is long (scored with no bound yet) first:
      // a warp that takes one late sets the kernel's end
      VG_CU(ix->ws_work.reserve(nq * 4));
      VG_CU(launch_order_seed(ix->ws_probes.as<uint32_t>(), static_cast<int>(P), nullptr,
                              ix->list_off.as<uint64_t>(), nq, kHeavyVectors, ix->ws_work.as<uint32_t>(),
                              d_counter + 2, static_cast<uint32_t>(nq), nullptr, s));
      sp.work = ix->ws_work.as<uint32_t>();
      sp.work_count = d_counter + 2;
      sp.work_cap = static_cast<uint32_t>(nq);
      ix->launches += 1;
    }
    VG_CU(vg::launch_ivfpq_scan(sp, ix->num_sms, s));
    ix->launches += 1;
  } else {
    // the approximate top-pool in passes of 256: pass i keeps the keys above
    // pass i-1's last one, so the passes concatenate into the sorted top-pool
    constexpr size_t kPass = 256;
    VG_CU(ix->ws_all_keys.reserve(nq * kPass * 8));
    VG_CU(ix->ws_floor.reserve(nq * 8));
    unsigned long long *pass_keys = ix->ws_all_keys.as<unsigned long long>();
    unsigned long long *floor = ix->ws_floor.as<unsigned long long>();
    sp.k = static_cast<int>(kPass);
    sp.out_keys = pass_keys;
    for (size_t c0 = 0; c0 < kk; c0 += kPass) {
      const size_t w = std::min(kPass, kk - c0);
      if (c0) VG_CU(cudaMemsetAsync(d_counter, 0, 4, s));
      sp.key_floor = c0 ? floor : nullptr;
      VG_CU(vg::launch_ivfpq_scan(sp, ix->num_sms, s));
      ix->launches += 1;
      VG_CU(cudaMemcpy2DAsync(ix->ws_keys.as<unsigned long long>() + c0, kk * 8, pass_keys, kPass * 8, w * 8, nq,
                              cudaMemcpyDeviceToDevice, s));
      if (c0 + kPass < kk)
        VG_CU(cudaMemcpy2DAsync(floor, 8, pass_keys + kPass - 1, kPass * 8, 8, nq, cudaMemcpyDeviceToDevice, s));
    }
  }
  mark(ix, 6);

  mark(ix, 7);
  if (rerank) {
    VG_CU(launch_rerank(ix->ws_qn.as<float>(), ix->vectors.as<float>(), static_cast<int>(d),
                        ix->ws_keys.as<unsigned long long>(), nq, static_cast<int>(kk), static_cast<int>(k),
                        doc_map, o_ids, o_dist, o_cnt, s));
    ix->launches += 1;
  }
  mark(ix, 9);
  if (!dev_out) {
    VG_CU(cudaMemcpyAsync(out_ids, o_ids, nq * k * 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaMemcpyAsync(out_dist, o_dist, nq * k * 4, cudaMemcpyDeviceToHost, s));
    if (out_count) VG_CU(cudaMemcpyAsync(out_count, o_cnt, nq * 4, cudaMemcpyDeviceToHost, s));
  }
  mark(ix, 10);
  VG_TRY(sync_stream(ix));
  VG_TRY(check_device_error(ix, "search"));

  if (prof) {
    auto el = [&](int a, int b) {
      float ms = 0;
      cudaEventElapsedTime(&ms, ix->ev[a], ix->ev[b]);
      return static_cast<double>(ms);
    };
    vg_search_profile &p = ix->prof;
    p.h2d_ms += el(0, 1);
    p.normalize_ms += el(1, 2);
    if (tiled_prof) {
      for (size_t t = 0; t < ntiles; ++t) {
        float a = 0, b = 0;
        cudaEventElapsedTime(&a, ix->tile_ev[3 * t], ix->tile_ev[3 * t + 1]);
        cudaEventElapsedTime(&b, ix->tile_ev[3 * t + 1], ix->tile_ev[3 * t + 2]);
        p.coarse_ms += a;
        p.select_ms += b;
      }
    } else {
      p.coarse_ms += el(2, 3);
      p.select_ms += el(3, 4);
    }
    p.pairs_ms += el(4, 5);
    p.scan_ms += el(5, 6);
    p.merge_ms += el(6, 9);
    p.d2h_ms += el(9, 10);
    p.total_ms += el(0, 10);
    p.calls += 1;
    p.queries += nq;
    p.kernel_launches += ix->launches - launches0;
    p.scan_launches += 1;
  }
  return VG_OK;
}

// ---- filtered search (search.rs:1407-1549) --------------------------------

// Device per-vector categories and per-list category counts from the current
// metadata (metadata may change after build; list bitmasks do not).
int refresh_categories(vg_index *ix) {
  if (!ix->cat_dirty) return VG_OK;
  cudaStream_t s = ix->stream;
  const size_t n = ix->n, Lc = ix->num_centroids;
  std::vector<uint8_t> cat(n, 0xff);
  for (size_t i = 0; i < n; ++i) {
    auto it = ix->doc_category.find(ix->h_doc_ids[i]);
    if (it != ix->doc_category.end() && it->second >= 0) cat[i] = static_cast<uint8_t>(it->second);
  }
  VG_CU(ix->category_d.reserve(std::max<size_t>(n, 1)));
  VG_CU(ix->cat_counts.reserve(Lc * 64 * 4));
  VG_CU(cudaMemcpyAsync(ix->category_d.p, cat.data(), n, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemsetAsync(ix->cat_counts.p, 0, Lc * 64 * 4, s));
  VG_CU(launch_category_counts(ix->category_d.as<uint8_t>(), ix->assign.as<uint32_t>(), n,
                               ix->cat_counts.as<uint32_t>(), s));
  VG_CU(cudaStreamSynchronize(s));
  ix->cat_dirty = false;
  return VG_OK;
}

// Per-list category bitmasks at build time (search.rs:626-651).
int build_filter_bitmasks(vg_index *ix) {
  const size_t n = ix->n, L = ix->params.num_clusters;
  std::vector<uint32_t> assign(n);
  VG_CU(cudaMemcpy(assign.data(), ix->assign.p, n * 4, cudaMemcpyDeviceToHost));
  ix->h_bitmask.assign(L, 0);
  for (size_t i = 0; i < n; ++i) {
    auto it = ix->doc_category.find(ix->h_doc_ids[i]);
    if (it != ix->doc_category.end() && it->second >= 0) ix->h_bitmask[assign[i]] |= uint64_t(1) << it->second;
  }
  VG_CU(ix->bitmask_d.reserve(L * 8));
  VG_CU(cudaMemcpy(ix->bitmask_d.p, ix->h_bitmask.data(), L * 8, cudaMemcpyHostToDevice));
  ix->cat_dirty = true;
  return VG_OK;
}

int search_filtered_impl(vg_index *ix, const float *queries, size_t nq, size_t k, const char *field,
                         const char *value_json, uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  if (!ix->built) return fail(VG_ERR_NOT_BUILT, "IVF-PQ index is not built: cannot search");
  if (!field) return fail(VG_ERR_INVALID_PARAMETER, "null filter field");
  if (!ix->has_filter_field || ix->filter_field != field)  // search.rs:1428-1435
    return fail(VG_ERR_INVALID_PARAMETER,
                std::string("filter field '") + field + "' doesn't match index filter field '" +
                    (ix->has_filter_field ? "Some(\"" + ix->filter_field + "\")" : std::string("None")) + "'");
  int want = -1;
  VG_TRY(parse_filter_category(value_json, &want));
  if (k > 256) return fail(VG_ERR_INVALID_PARAMETER, "k must be at most 256");
  if (ix->world > 1) return fail(VG_ERR_UNSUPPORTED, "unsupported: filtered search on a sharded index");
  if (nq == 0 || k == 0) return write_padding(ix, nq, k, out_ids, out_dist, out_count);
  if (!queries || !out_ids || !out_dist) return fail(VG_ERR_INVALID_PARAMETER, "null query or output buffer");
  const size_t Lc = ix->num_centroids, d = ix->d;
  const size_t P = std::min(static_cast<size_t>(ix->params.nprobe), Lc);
  if (P == 0) return write_padding(ix, nq, k, out_ids, out_dist, out_count);
  if (nq * std::max(P, Lc) > 0xffffffffull) return fail(VG_ERR_INVALID_PARAMETER, "too many queries in one call");
  VG_TRY(refresh_categories(ix));
  cudaStream_t s = ix->stream;

  // normalise, coarse distances and the nprobe nearest lists (search.rs:1460-1471)
  const float *dq = queries;
  if (!is_device_ptr(queries)) {
    VG_CU(ix->ws_q.reserve(nq * d * 4));
    VG_CU(cudaMemcpyAsync(ix->ws_q.p, queries, nq * d * 4, cudaMemcpyHostToDevice, s));
    dq = ix->ws_q.as<float>();
  }
  VG_CU(ix->ws_qn.reserve(nq * d * 4));
  VG_CU(launch_normalize_rows(dq, nq, static_cast<int>(d), ix->ws_qn.as<float>(), s));
  const size_t tile = coarse_tile(ix, nq, P);
  VG_CU(ix->ws_probes.reserve(nq * P * 4));
  VG_CU(ix->ws_pdist.reserve(nq * P * 4));
  *reinterpret_cast<volatile int *>(ix->h_err) = 0;
  for (size_t r0 = 0; r0 < nq; r0 += tile) {
    const size_t rows = std::min(tile, nq - r0);
    VG_TRY(coarse_probes(ix, ix->ws_qn.as<float>() + r0 * d, rows, P, ix->ws_probes.as<uint32_t>() + r0 * P,
                         ix->ws_pdist.as<float>() + r0 * P, &ix->launches));
  }

  // which queries find fewer than k matches in their probed lists
  std::vector<uint8_t> widen(nq, 0);
  if (P < Lc) {
    VG_CU(ix->ws_scalars.reserve(std::max<size_t>(64, nq)));
    VG_CU(launch_filter_widen(ix->ws_probes.as<uint32_t>(), nq, static_cast<int>(P), ix->bitmask_d.as<uint64_t>(),
                              ix->cat_counts.as<uint32_t>(), want, k, ix->ws_scalars.as<uint8_t>(), s));
    VG_CU(cudaMemcpyAsync(widen.data(), ix->ws_scalars.p, nq, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaStreamSynchronize(s));
  }
  std::vector<uint32_t> narrow_q, wide_q;
  for (size_t q = 0; q < nq; ++q) (widen[q] ? wide_q : narrow_q).push_back(static_cast<uint32_t>(q));

  const bool dev_out = is_device_ptr(out_ids) && is_device_ptr(out_dist) && (!out_count || is_device_ptr(out_count));
  uint32_t *o_ids = out_ids, *o_cnt = out_count;
  float *o_dist = out_dist;
  if (!dev_out) {
    VG_CU(ix->ws_out_ids.reserve(nq * k * 4));
    VG_CU(ix->ws_out_dist.reserve(nq * k * 4));
    VG_CU(ix->ws_out_count.reserve(nq * 4));
    o_ids = ix->ws_out_ids.as<uint32_t>();
    o_dist = ix->ws_out_dist.as<float>();
    o_cnt = ix->ws_out_count.as<uint32_t>();
  }
  DevBuf qmap, all_lists, counter, cnt_tmp;
  VG_CU(qmap.reserve(nq * 4));
  VG_CU(counter.reserve(16));
  if (!o_cnt) {
    VG_CU(cnt_tmp.reserve(nq * 4));
    o_cnt = cnt_tmp.as<uint32_t>();
  }
  vg::ScanParams sp{};
  sp.qn = ix->ws_qn.as<float>();
  sp.centroids = ix->centroids.as<float>();
  sp.codebooks = ix->codebooks.as<float>();
  sp.counter = counter.as<uint32_t>();
  sp.list_off = ix->list_off.as<uint64_t>();
  sp.code_off = ix->code_off.as<uint64_t>();
  sp.list_codes = ix->list_codes.as<uint8_t>();
  sp.list_ids = ix->list_ids.as<uint32_t>();
  sp.doc_ids = ix->doc_ids.as<uint32_t>();
  sp.rot_t = ix->h_rotation.empty() ? nullptr : ix->rotation_t.as<float>();
  sp.d = static_cast<int>(d);
  sp.M = static_cast<int>(ix->params.num_codebooks);
  sp.ks = static_cast<int>(ix->params.codebook_size);
  sp.dsub = static_cast<int>(ix->dsub);
  sp.k = static_cast<int>(k);
  sp.out_ids = o_ids;
  sp.out_dist = o_dist;
  sp.out_count = o_cnt;
  sp.error = ix->d_err;
  sp.qmap = qmap.as<uint32_t>();
  sp.category = ix->category_d.as<uint8_t>();
  sp.bitmask = ix->bitmask_d.as<uint64_t>();
  sp.want_cat = want;
  // every list scored with the float table, as distance_with_table does
  // (search.rs:1523-1528), also for 16-entry codebooks
  auto run = [&](const std::vector<uint32_t> &qs, const uint32_t *probes, int np, int shared) -> int {
    if (qs.empty()) return VG_OK;
    VG_CU(cudaMemcpyAsync(qmap.p, qs.data(), qs.size() * 4, cudaMemcpyHostToDevice, s));
    VG_CU(cudaMemsetAsync(counter.p, 0, 4, s));
    sp.probes = probes;
    sp.P = np;
    sp.probes_shared = shared;
    sp.nq = static_cast<int>(qs.size());
    VG_CU(launch_ivfpq_scan_generic(sp, ix->num_sms, s));
    VG_CU(cudaStreamSynchronize(s));
    ix->launches += 1;
    return VG_OK;
  };
  VG_TRY(run(narrow_q, ix->ws_probes.as<uint32_t>(), static_cast<int>(P), 0));
  if (!wide_q.empty()) {  // widen: every list, nearest-first order is immaterial to the top-k
    std::vector<uint32_t> iota(Lc);
    std::iota(iota.begin(), iota.end(), 0u);
    VG_CU(all_lists.reserve(Lc * 4));
    VG_CU(cudaMemcpyAsync(all_lists.p, iota.data(), Lc * 4, cudaMemcpyHostToDevice, s));
    VG_TRY(run(wide_q, all_lists.as<uint32_t>(), static_cast<int>(Lc), 1));
  }
  if (!dev_out) {
    VG_CU(cudaMemcpyAsync(out_ids, o_ids, nq * k * 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaMemcpyAsync(out_dist, o_dist, nq * k * 4, cudaMemcpyDeviceToHost, s));
    if (out_count) VG_CU(cudaMemcpyAsync(out_count, o_cnt, nq * 4, cudaMemcpyDeviceToHost, s));
  }
  VG_TRY(sync_stream(ix));
  return check_device_error(ix, "filtered search");
}

}  // namespace

namespace vg {
// Sets the text vg_last_error reports, for entry points defined in other
// translation units.
void set_last_error(const char *msg) { g_last_error = msg; }

// ---- snapshot image (search.rs:945-1084) -----------------------------------

int snapshot_export(const vg_index *ix, SnapshotState &st) {
  if (!ix->built) return fail(VG_ERR_NOT_BUILT, "IVF-PQ index is not built: cannot save");
  if (ix->partitioned)
    return fail(VG_ERR_UNSUPPORTED, "unsupported: saving a list-sharded index (each rank holds its lists only)");
  DeviceGuard g(ix->device);
  const size_t n = ix->n, d = ix->d, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const size_t Lc = ix->num_centroids, L = ix->params.num_clusters;
  st = SnapshotState{};
  st.dim = d;
  st.num_vectors = n;
  st.num_centroids = Lc;
  st.params = ix->params;
  st.centroids.resize(Lc * d);
  st.codebooks.resize(M * ks * ix->dsub);
  st.codes.resize(n * M);
  st.list_ids.resize(n);
  VG_CU(cudaMemcpy(st.centroids.data(), ix->centroids.p, st.centroids.size() * 4, cudaMemcpyDeviceToHost));
  VG_CU(cudaMemcpy(st.codebooks.data(), ix->codebooks.p, st.codebooks.size() * 4, cudaMemcpyDeviceToHost));
  VG_CU(cudaMemcpy(st.codes.data(), ix->codes.p, st.codes.size(), cudaMemcpyDeviceToHost));
  VG_CU(cudaMemcpy(st.list_ids.data(), ix->list_ids.p, n * 4, cudaMemcpyDeviceToHost));
  st.optimized = ix->optimized;
  st.rotation = ix->h_rotation;
  st.doc_ids = ix->h_doc_ids;
  // the reference keeps num_clusters clusters; those past the trained
  // centroids are empty
  st.list_offsets.assign(ix->h_list_off.begin(), ix->h_list_off.end());
  st.list_offsets.resize(L + 1, st.list_offsets.back());
  st.bitmasks = ix->h_bitmask;
  st.bitmasks.resize(L, 0);
  if (!ix->compacted) {
    st.vectors.resize(n * d);
    VG_CU(cudaMemcpy(st.vectors.data(), ix->vectors.p, n * d * 4, cudaMemcpyDeviceToHost));
  }
  st.has_filter_field = ix->has_filter_field;
  st.filter_field = ix->filter_field;
  st.metadata.assign(ix->metadata.begin(), ix->metadata.end());
  return VG_OK;
}

int snapshot_adopt(vg_index *ix, SnapshotState &st) {
  const size_t n = st.num_vectors, d = ix->d, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const size_t L = ix->params.num_clusters, Lc = st.num_centroids;
  auto bad = [](const std::string &what) { return fail(VG_ERR_FORMAT, "IVF-PQ snapshot: " + what); };
  if (st.dim != d) return bad("dimension does not match the index");
  if (n == 0 || n > 0xffffffffull) return bad("vector count out of range");
  if (Lc == 0 || Lc > L) return bad("num_centroids must be in 1..=num_clusters");
  if (st.centroids.size() != Lc * d) return bad("centroid array has the wrong length");
  if (st.codebooks.size() != M * ks * ix->dsub) return bad("codebook array has the wrong length");
  if (!st.rotation.empty() && st.rotation.size() != d * d) return bad("rotation is not dimension x dimension");
  if (st.doc_ids.size() != n || st.codes.size() != n * M) return bad("doc ids or codes have the wrong length");
  if (!st.vectors.empty() && st.vectors.size() != n * d) return bad("raw vectors have the wrong length");
  if (st.list_offsets.size() != L + 1 || st.list_offsets.front() != 0 || st.list_offsets.back() != n ||
      st.list_ids.size() != n || st.bitmasks.size() != L)
    return bad("cluster table does not match num_clusters and num_vectors");
  for (size_t i = 0; i < n * M; ++i)
    if (st.codes[i] >= ks) return bad("code " + std::to_string(st.codes[i]) + " out of range for codebook_size");
  // the clusters must partition the vectors; clusters past the centroids are
  // never probed and must be empty
  std::vector<uint32_t> assign(n, 0xffffffffu), sorted_lists(n);
  for (size_t l = 0; l < L; ++l) {
    if (st.list_offsets[l + 1] < st.list_offsets[l]) return bad("cluster offsets decrease");
    if (l >= Lc && st.list_offsets[l + 1] != st.list_offsets[l]) return bad("a cluster past num_centroids is not empty");
    for (uint64_t p = st.list_offsets[l]; p < st.list_offsets[l + 1]; ++p) {
      const uint32_t id = st.list_ids[p];
      if (id >= n) return bad("cluster id " + std::to_string(id) + " exceeds vector count " + std::to_string(n));
      if (assign[id] != 0xffffffffu) return bad("vector " + std::to_string(id) + " is in more than one cluster");
      assign[id] = static_cast<uint32_t>(l);
      sorted_lists[p] = static_cast<uint32_t>(l);
    }
  }
  DeviceGuard g(ix->device);
  cudaStream_t s = ix->stream;
  VG_CU(ix->centroids.reserve(Lc * d * 4));
  VG_CU(ix->codebooks.reserve(st.codebooks.size() * 4));
  VG_CU(ix->doc_ids.reserve(n * 4));
  VG_CU(ix->codes.reserve(n * M));
  VG_CU(ix->assign.reserve(n * 4));
  VG_CU(ix->list_ids.reserve(n * 4));
  DevBuf d_sorted;
  VG_CU(d_sorted.reserve(n * 4));
  VG_CU(cudaMemcpyAsync(ix->centroids.p, st.centroids.data(), Lc * d * 4, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->codebooks.p, st.codebooks.data(), st.codebooks.size() * 4, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->doc_ids.p, st.doc_ids.data(), n * 4, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->codes.p, st.codes.data(), n * M, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->assign.p, assign.data(), n * 4, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(ix->list_ids.p, st.list_ids.data(), n * 4, cudaMemcpyHostToDevice, s));
  VG_CU(cudaMemcpyAsync(d_sorted.p, sorted_lists.data(), n * 4, cudaMemcpyHostToDevice, s));
  if (!st.vectors.empty()) {
    VG_CU(ix->vectors.reserve(n * d * 4));
    VG_CU(cudaMemcpyAsync(ix->vectors.p, st.vectors.data(), n * d * 4, cudaMemcpyHostToDevice, s));
  }
  VG_CU(cudaStreamSynchronize(s));
  ix->n = ix->cap = n;
  ix->num_centroids = Lc;
  ix->h_doc_ids = std::move(st.doc_ids);
  ix->h_list_off.assign(st.list_offsets.begin(), st.list_offsets.begin() + Lc + 1);
  ix->h_bitmask = std::move(st.bitmasks);
  ix->optimized = st.optimized;
  ix->h_rotation = std::move(st.rotation);
  VG_TRY(upload_rotation(ix));
  ix->compacted = st.vectors.empty();
  ix->has_filter_field = st.has_filter_field;
  ix->filter_field = std::move(st.filter_field);
  for (auto &e : st.metadata) {
    int cat = -1;
    std::string canon;
    if (parse_metadata(e.second.c_str(), ix->filter_field, &cat, &canon) != VG_OK)
      return fail(VG_ERR_FORMAT, "IVF-PQ snapshot: metadata of document " + std::to_string(e.first) + ": " + g_last_error);
    ix->metadata[e.first] = std::move(canon);
    ix->doc_category[e.first] = cat;
  }
  if (ix->has_filter_field) {
    VG_CU(ix->bitmask_d.reserve(ix->h_bitmask.size() * 8));
    VG_CU(cudaMemcpy(ix->bitmask_d.p, ix->h_bitmask.data(), ix->h_bitmask.size() * 8, cudaMemcpyHostToDevice));
  }
  ix->cat_dirty = true;
  ix->trained = true;
  VG_TRY(build_list_storage(ix, d_sorted.as<uint32_t>()));
  return VG_OK;
}
}  // namespace vg

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int vg_last_error(char *buf, size_t len) {
  if (!buf || len == 0) return VG_ERR_INVALID_PARAMETER;
  size_t m = std::min(len - 1, g_last_error.size());
  std::memcpy(buf, g_last_error.data(), m);
  buf[m] = '\0';
  return VG_OK;
}

const char *vg_version(void) { return "vicinity-b200 0.1.0 (sm_100a)"; }

int vg_selftest_bounded_wait(int device, uint32_t limit_us, int *out_expired) {
  if (!out_expired) return fail(VG_ERR_INVALID_PARAMETER, "null output");
  if (limit_us == 0 || limit_us > 1000000u) return fail(VG_ERR_INVALID_PARAMETER, "limit_us must be in 1..1000000");
  DeviceGuard g(device);
  int clock_khz = 0;
  VG_CU(cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, device));
  // the limit in cycles at the part's highest clock: at any lower clock the
  // wait lasts longer, never shorter
  const long long cycles = static_cast<long long>(limit_us) * std::max(clock_khz, 1) / 1000;
  DevBuf flag_d;
  VG_CU(flag_d.reserve(sizeof(int)));
  VG_CU(cudaMemset(flag_d.p, 0, sizeof(int)));
  VG_CU(launch_bounded_wait_check(cycles, flag_d.as<int>(), nullptr));
  int flag = 0;
  VG_CU(cudaMemcpy(&flag, flag_d.p, sizeof(int), cudaMemcpyDeviceToHost));
  *out_expired = flag == 4 ? 1 : 0;
  return VG_OK;
}

int vg_device_count(int *out) {
  if (!out) return fail(VG_ERR_INVALID_PARAMETER, "null output");
  int c = 0;
  cudaError_t e = cudaGetDeviceCount(&c);
  if (e != cudaSuccess) {
    cudaGetLastError();
    c = 0;
  }
  *out = c;
  return VG_OK;
}

int vg_ivfpq_create(size_t dim, const vg_ivfpq_params *params, int device, vg_index **out) {
  if (!params || !out) return fail(VG_ERR_INVALID_PARAMETER, "null params or output");
  *out = nullptr;
  VG_TRY(validate_shape(dim, *params));
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return fail(VG_ERR_CUDA, "no CUDA device " + std::to_string(device) + " (the engine has no CPU path)");
  }
  DeviceGuard g(device);
  auto *ix = new vg_index();
  ix->device = device;
  ix->d = dim;
  ix->params = *params;
  ix->optimized = params->use_opq != 0;
  ix->dsub = dim / params->num_codebooks;
  cudaDeviceGetAttribute(&ix->num_sms, cudaDevAttrMultiProcessorCount, device);
  cudaError_t e = cudaStreamCreateWithFlags(&ix->own_stream, cudaStreamNonBlocking);
  ix->stream = ix->own_stream;
  for (int i = 0; e == cudaSuccess && i < kPhaseEvents; ++i) e = cudaEventCreate(&ix->ev[i]);
  if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void **>(&ix->h_err), sizeof(int), cudaHostAllocMapped);
  if (e == cudaSuccess) {
    *ix->h_err = 0;
    e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&ix->d_err), ix->h_err, 0);
  }
  if (const char *fam = std::getenv("VICINITY_SCAN_KERNEL"))
    vg::set_scan_family(std::strcmp(fam, "query") == 0    ? 1
                        : std::strcmp(fam, "stream") == 0 ? 3
                        : std::strcmp(fam, "direct") == 0 ? 5
                                                          : 4);
  if (e != cudaSuccess) {
    vg_ivfpq_destroy(ix);
    return cuda_fail(e, "stream/event creation");
  }
  *out = ix;
  return VG_OK;
}

int vg_ivfpq_destroy(vg_index *ix) {
  if (!ix) return VG_OK;
  {
    DeviceGuard g(ix->device);
    if (ix->stream) cudaStreamSynchronize(ix->stream);
    if (ix->comm) ncclCommDestroy(ix->comm);
    for (DevBuf *b : {&ix->vectors, &ix->doc_ids, &ix->centroids, &ix->codebooks, &ix->assign, &ix->codes,
                      &ix->list_off, &ix->list_ids, &ix->code_off, &ix->list_codes, &ix->pack_off, &ix->packed,
                      &ix->owner, &ix->ws_q, &ix->ws_qn, &ix->ws_dist, &ix->ws_probes, &ix->ws_pdist,
                      &ix->ws_scalars, &ix->ws_keys, &ix->ws_all_keys, &ix->ws_out_ids, &ix->ws_out_dist,
                      &ix->ws_out_count, &ix->stats, &ix->ws_lb, &ix->ws_rec, &ix->ws_lbq, &ix->ws_qimg,
                      &ix->ws_eps, &ix->ws_tc, &ix->ws_floor, &ix->cent_img, &ix->ws_seed, &ix->ws_qall, &ix->ws_cmax, &ix->ws_units,
                      &ix->ws_work})
      b->release();
    for (int i = 0; i < kPhaseEvents; ++i)
      if (ix->ev[i]) cudaEventDestroy(ix->ev[i]);
    for (cudaEvent_t e : ix->tile_ev) cudaEventDestroy(e);
    for (cudaEvent_t e : ix->copy_ev) cudaEventDestroy(e);
    if (ix->copy_start) cudaEventDestroy(ix->copy_start);
    if (ix->copy_stream) cudaStreamDestroy(ix->copy_stream);
    if (ix->h_err) cudaFreeHost(ix->h_err);
    if (ix->own_stream) cudaStreamDestroy(ix->own_stream);
    delete ix;
  }
  return VG_OK;
}

int vg_ivfpq_add(vg_index *ix, const uint32_t *doc_ids, const float *x, size_t n) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  if (ix->built)
    return fail(VG_ERR_ALREADY_BUILT, "IVF-PQ index is already built: cannot add vectors");
  if (n == 0) return VG_OK;
  if (!doc_ids || !x) return fail(VG_ERR_INVALID_PARAMETER, "null doc_ids or vectors");
  if (ix->n + n > 0xffffffffull) return fail(VG_ERR_INVALID_PARAMETER, "at most 2^32 - 1 vectors per index");
  DeviceGuard g(ix->device);
  cudaStream_t s = ix->stream;
  const size_t d = ix->d;
  if (ix->n + n > ix->cap) {
    size_t cap = std::max(ix->n + n, ix->cap * 2);
    DevBuf nv, nd;
    VG_CU(nv.reserve(cap * d * 4));
    VG_CU(nd.reserve(cap * 4));
    if (ix->n) {
      VG_CU(cudaMemcpyAsync(nv.p, ix->vectors.p, ix->n * d * 4, cudaMemcpyDeviceToDevice, s));
      VG_CU(cudaMemcpyAsync(nd.p, ix->doc_ids.p, ix->n * 4, cudaMemcpyDeviceToDevice, s));
      VG_CU(cudaStreamSynchronize(s));
    }
    ix->vectors = std::move(nv);
    ix->doc_ids = std::move(nd);
    ix->cap = cap;
  }
  const float *src = x;
  DevBuf stage;
  if (!is_device_ptr(x)) {
    VG_CU(stage.reserve(n * d * 4));
    VG_CU(cudaMemcpyAsync(stage.p, x, n * d * 4, cudaMemcpyHostToDevice, s));
    src = stage.as<float>();
  }
  VG_CU(launch_normalize_rows(src, n, static_cast<int>(d), ix->vectors.as<float>() + ix->n * d, s));
  VG_CU(cudaMemcpyAsync(ix->doc_ids.as<uint32_t>() + ix->n, doc_ids, n * 4, cudaMemcpyDefault, s));
  size_t old = ix->h_doc_ids.size();
  ix->h_doc_ids.resize(old + n);
  VG_CU(cudaMemcpyAsync(ix->h_doc_ids.data() + old, doc_ids, n * 4, cudaMemcpyDefault, s));
  VG_CU(cudaStreamSynchronize(s));
  ix->n += n;
  return VG_OK;
}

int vg_ivfpq_set_trained(vg_index *ix, const float *centroids, size_t num_centroids, const float *codebooks) {
  if (!ix || !centroids || !codebooks) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  if (ix->built) return fail(VG_ERR_ALREADY_BUILT, "IVF-PQ index is already built: cannot replace its training");
  if (num_centroids == 0 || num_centroids > ix->params.num_clusters)
    return fail(VG_ERR_INVALID_PARAMETER, "num_centroids must be in 1..=num_clusters");
  DeviceGuard g(ix->device);
  const size_t M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  VG_CU(ix->centroids.reserve(num_centroids * ix->d * 4));
  VG_CU(ix->codebooks.reserve(M * ks * ix->dsub * 4));
  VG_CU(cudaMemcpy(ix->centroids.p, centroids, num_centroids * ix->d * 4, cudaMemcpyDefault));
  VG_CU(cudaMemcpy(ix->codebooks.p, codebooks, M * ks * ix->dsub * 4, cudaMemcpyDefault));
  ix->num_centroids = num_centroids;
  ix->trained = true;
  return VG_OK;
}

int vg_ivfpq_set_rotation(vg_index *ix, const float *rotation) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  if (ix->built) return fail(VG_ERR_ALREADY_BUILT, "IVF-PQ index is already built: cannot replace its rotation");
  DeviceGuard g(ix->device);
  const size_t d = ix->d;
  if (!rotation) {
    ix->h_rotation.clear();
    ix->optimized = ix->params.use_opq != 0;
    return upload_rotation(ix);
  }
  std::vector<float> r(d * d);
  VG_CU(cudaMemcpy(r.data(), rotation, d * d * 4, cudaMemcpyDefault));
  for (float v : r)
    if (!std::isfinite(v)) return fail(VG_ERR_INVALID_PARAMETER, "rotation holds a non-finite value");
  ix->h_rotation = std::move(r);
  ix->optimized = true;
  return upload_rotation(ix);
}

int vg_ivfpq_build(vg_index *ix, size_t training_sample_size, size_t kmeans_max_iter) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  if (ix->built) return VG_OK;  // search.rs:550-552
  if (ix->n == 0) return fail(VG_ERR_EMPTY_INDEX, "index is empty");
  const size_t ks = ix->params.codebook_size, L = ix->params.num_clusters;
  if (ix->n < ks)
    return fail(VG_ERR_INVALID_PARAMETER,
                "invalid parameter: IVF-PQ requires at least codebook_size training vectors (got " +
                    std::to_string(ix->n) + " vectors, codebook_size = " + std::to_string(ks) + ")");
  if (kmeans_max_iter == 0)
    return fail(VG_ERR_INVALID_CONFIG, "invalid config `kmeans_max_iter`: must be greater than 0");
  const size_t n_train = (training_sample_size == 0 || training_sample_size >= ix->n) ? ix->n : training_sample_size;
  const size_t min_train = std::max(std::min(L, ix->n), ks);
  if (n_train < min_train)
    return fail(VG_ERR_INVALID_PARAMETER, "invalid parameter: IVF-PQ training sample is too small (got " +
                                              std::to_string(n_train) + ", need at least " +
                                              std::to_string(min_train) + ")");
  DeviceGuard g(ix->device);
  if (!ix->trained) VG_TRY(train(ix, n_train, kmeans_max_iter));
  VG_TRY(encode_and_layout(ix));
  if (ix->has_filter_field) VG_TRY(build_filter_bitmasks(ix));
  return VG_OK;
}

int vg_ivfpq_set_filter_field(vg_index *ix, const char *field) {
  if (!ix || !field) return fail(VG_ERR_INVALID_PARAMETER, "null index or field");
  if (ix->built) return fail(VG_ERR_ALREADY_BUILT, "IVF-PQ index is already built: cannot enable filtering");
  ix->has_filter_field = true;
  ix->filter_field = field;
  return VG_OK;
}

int vg_ivfpq_add_metadata(vg_index *ix, uint32_t doc_id, const char *metadata_json) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  if (!ix->has_filter_field)  // search.rs:469-474
    return fail(VG_ERR_UNSUPPORTED,
                "unsupported: filtered search; rebuild the index with IVFPQIndex::with_filtering()");
  int cat = -1;
  std::string canon;
  VG_TRY(parse_metadata(metadata_json, ix->filter_field, &cat, &canon));
  ix->metadata[doc_id] = std::move(canon);  // MetadataStore::add replaces (filtering/mod.rs:206-208)
  ix->doc_category[doc_id] = cat;
  ix->cat_dirty = true;
  return VG_OK;
}

int vg_ivfpq_search_filtered_batch(vg_index *ix, const float *queries, size_t nq, size_t k, const char *field,
                                   const char *value_json, uint32_t *out_ids, float *out_dist,
                                   uint32_t *out_count) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  DeviceGuard g(ix->device);
  return search_filtered_impl(ix, queries, nq, k, field, value_json, out_ids, out_dist, out_count);
}

int vg_ivfpq_set_nprobe(vg_index *ix, size_t nprobe) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  ix->params.nprobe = nprobe;
  return VG_OK;
}

int vg_ivfpq_set_stream(vg_index *ix, void *stream) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  DeviceGuard g(ix->device);
  VG_CU(cudaStreamSynchronize(ix->stream));
  ix->stream = stream ? static_cast<cudaStream_t>(stream) : ix->own_stream;
  return VG_OK;
}

int vg_ivfpq_set_coarse_tile_rows(vg_index *ix, size_t rows) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  ix->coarse_tile_rows = rows;
  return VG_OK;
}

int vg_ivfpq_get_info(const vg_index *ix, vg_ivfpq_info *out) {
  if (!ix || !out) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  std::memset(out, 0, sizeof(*out));
  out->dimension = ix->d;
  out->num_vectors = ix->n;
  out->num_clusters = ix->params.num_clusters;
  out->num_centroids = ix->num_centroids;
  out->nprobe = ix->params.nprobe;
  out->num_codebooks = ix->params.num_codebooks;
  out->codebook_size = ix->params.codebook_size;
  out->subvector_dim = ix->dsub;
  out->built = ix->built;
  out->trained = ix->trained;
  out->compacted = ix->compacted;
  out->use_opq = ix->params.use_opq;
  out->device = ix->device;
  out->shard_rank = ix->rank;
  out->shard_world = ix->world;
  out->device_bytes = ix->device_bytes();
  return VG_OK;
}

int vg_ivfpq_search_batch(vg_index *ix, const float *queries, size_t nq, size_t k, size_t nprobe,
                          uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  DeviceGuard g(ix->device);
  return search_impl(ix, queries, nq, k, 0, nprobe, out_ids, out_dist, out_count);
}

int vg_ivfpq_nearest_lists(vg_index *ix, const float *queries, size_t nq, size_t nprobe, uint32_t *out_lists,
                           float *out_dist) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  DeviceGuard g(ix->device);
  if (!ix->built) return fail(VG_ERR_NOT_BUILT, "index not built");
  const size_t Lc = ix->num_centroids, d = ix->d;
  const size_t P = std::min(nprobe ? nprobe : static_cast<size_t>(ix->params.nprobe), Lc);
  if (nq == 0 || P == 0) return VG_OK;
  if (!queries || !out_lists || !out_dist) return fail(VG_ERR_INVALID_PARAMETER, "null query or output buffer");
  if (P > 256) return fail(VG_ERR_INVALID_PARAMETER, "nprobe must be at most 256");
  if (nq * P > 0xffffffffull) return fail(VG_ERR_INVALID_PARAMETER, "nq * nprobe must fit in 32 bits");
  cudaStream_t s = ix->stream;
  const float *dq = queries;
  if (!is_device_ptr(queries)) {
    VG_CU(ix->ws_q.reserve(nq * d * 4));
    VG_CU(cudaMemcpyAsync(ix->ws_q.p, queries, nq * d * 4, cudaMemcpyHostToDevice, s));
    dq = ix->ws_q.as<float>();
  }
  VG_CU(ix->ws_qn.reserve(nq * d * 4));
  VG_CU(launch_normalize_rows(dq, nq, static_cast<int>(d), ix->ws_qn.as<float>(), s));
  const size_t tile = coarse_tile(ix, nq, P);
  VG_CU(ix->ws_probes.reserve(nq * P * 4));
  VG_CU(ix->ws_pdist.reserve(nq * P * 4));
  *reinterpret_cast<volatile int *>(ix->h_err) = 0;
  uint64_t launches = 1;
  for (size_t r0 = 0; r0 < nq; r0 += tile) {
    const size_t rows = std::min(tile, nq - r0);
    VG_TRY(coarse_probes(ix, ix->ws_qn.as<float>() + r0 * d, rows, P, ix->ws_probes.as<uint32_t>() + r0 * P,
                         ix->ws_pdist.as<float>() + r0 * P, &launches));
  }
  VG_CU(cudaMemcpyAsync(out_lists, ix->ws_probes.p, nq * P * 4, cudaMemcpyDefault, s));
  VG_CU(cudaMemcpyAsync(out_dist, ix->ws_pdist.p, nq * P * 4, cudaMemcpyDefault, s));
  VG_CU(cudaStreamSynchronize(s));
  return check_device_error(ix, "nearest_lists");
}

int vg_ivfpq_search_batch_reranked(vg_index *ix, const float *queries, size_t nq, size_t k, size_t candidate_pool,
                                   size_t nprobe, uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  DeviceGuard g(ix->device);
  return search_impl(ix, queries, nq, k, std::max<size_t>(candidate_pool, 1), nprobe, out_ids, out_dist, out_count);
}

int vg_ivfpq_reconstruct(const vg_index *ix, size_t idx, float *out) {
  if (!ix || !out) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  if (!ix->built) return fail(VG_ERR_INVALID_PARAMETER, "invalid parameter: index must be built before reconstruct");
  if (idx >= ix->n)
    return fail(VG_ERR_INVALID_PARAMETER, "invalid parameter: vector index " + std::to_string(idx) +
                                              " out of range (num_vectors = " + std::to_string(ix->n) + ")");
  if (ix->partitioned)
    return fail(VG_ERR_UNSUPPORTED, "unsupported: reconstruct on a list-sharded index (codes are partitioned)");
  DeviceGuard g(ix->device);
  const size_t d = ix->d, M = ix->params.num_codebooks, ks = ix->params.codebook_size, dsub = ix->dsub;
  uint32_t a = 0;
  std::vector<uint8_t> code(M);
  std::vector<float> cent(d), cb(M * ks * dsub);
  VG_CU(cudaMemcpy(&a, ix->assign.as<uint32_t>() + idx, 4, cudaMemcpyDeviceToHost));
  VG_CU(cudaMemcpy(code.data(), ix->codes.as<uint8_t>() + idx * M, M, cudaMemcpyDeviceToHost));
  VG_CU(cudaMemcpy(cent.data(), ix->centroids.as<float>() + static_cast<size_t>(a) * d, d * 4, cudaMemcpyDeviceToHost));
  VG_CU(cudaMemcpy(cb.data(), ix->codebooks.p, cb.size() * 4, cudaMemcpyDeviceToHost));
  std::vector<float> res(d), dec(d);
  for (size_t m = 0; m < M; ++m)
    for (size_t j = 0; j < dsub; ++j) dec[m * dsub + j] = cb[(m * ks + code[m]) * dsub + j];
  if (!ix->h_rotation.empty()) {  // opq.rs:126-136: decode applies R^T
    const std::vector<float> &r = ix->h_rotation;
    std::vector<float> rot(dec);
    for (size_t i = 0; i < d; ++i) {
      float s = 0.0f;
      for (size_t j = 0; j < d; ++j) s += r[j * d + i] * rot[j];
      dec[i] = s;
    }
  }
  for (size_t j = 0; j < d; ++j) res[j] = dec[j] + cent[j];  // search.rs:878-881
  VG_CU(cudaMemcpy(out, res.data(), d * 4, cudaMemcpyDefault));
  return VG_OK;
}

int vg_ivfpq_compact(vg_index *ix) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  if (!ix->built) return fail(VG_ERR_NOT_BUILT, "IVF-PQ index is not built: cannot compact");
  DeviceGuard g(ix->device);
  ix->vectors.release();
  ix->compacted = true;
  return VG_OK;
}

int vg_ivfpq_export(const vg_index *ix, int what, void *dst, size_t bytes) {
  if (!ix || (!dst && bytes)) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  DeviceGuard g(ix->device);
  const size_t n = ix->n, d = ix->d, M = ix->params.num_codebooks, ks = ix->params.codebook_size;
  const void *src = nullptr;
  size_t need = 0;
  bool needs_build = true;
  switch (what) {
    case VG_EXPORT_CENTROIDS: src = ix->centroids.p; need = ix->num_centroids * d * 4; needs_build = false; break;
    case VG_EXPORT_CODEBOOKS: src = ix->codebooks.p; need = ix->trained ? M * ks * ix->dsub * 4 : 0; needs_build = false; break;
    case VG_EXPORT_ASSIGNMENTS: src = ix->assign.p; need = n * 4; break;
    case VG_EXPORT_CODES: src = ix->codes.p; need = n * M; break;
    case VG_EXPORT_LIST_OFFSETS: src = ix->list_off.p; need = (ix->num_centroids + 1) * 8; break;
    case VG_EXPORT_LIST_IDS: src = ix->list_ids.p; need = n * 4; break;
    case VG_EXPORT_DOC_IDS: src = ix->doc_ids.p; need = n * 4; needs_build = false; break;
    case VG_EXPORT_ROTATION:
      src = ix->rotation.p; need = ix->h_rotation.empty() ? 0 : d * d * 4; needs_build = false; break;
    case VG_EXPORT_VECTORS:
      if (ix->compacted) return fail(VG_ERR_UNSUPPORTED, "raw vectors were dropped by compact()");
      src = ix->vectors.p; need = n * d * 4; needs_build = false; break;
    default: return fail(VG_ERR_INVALID_PARAMETER, "unknown export selector");
  }
  if (needs_build && !ix->built) return fail(VG_ERR_NOT_BUILT, "IVF-PQ index is not built: nothing to export");
  if (ix->partitioned && (what == VG_EXPORT_ASSIGNMENTS || what == VG_EXPORT_CODES ||
                          what == VG_EXPORT_LIST_OFFSETS || what == VG_EXPORT_LIST_IDS))
    return fail(VG_ERR_UNSUPPORTED, "unsupported: exporting codes or lists of a list-sharded index");
  if (bytes != need)
    return fail(VG_ERR_INVALID_PARAMETER, "export size mismatch: expected " + std::to_string(need) + " bytes");
  if (need) VG_CU(cudaMemcpy(dst, src, need, cudaMemcpyDefault));
  return VG_OK;
}

int vg_ivfpq_set_profiling(vg_index *ix, int on) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  DeviceGuard g(ix->device);
  if (on && !ix->stats.p) {
    VG_CU(ix->stats.reserve(kStats * 8));
    VG_CU(cudaMemset(ix->stats.p, 0, kStats * 8));
  }
  ix->profiling = on != 0;
  return VG_OK;
}

int vg_ivfpq_get_profile(const vg_index *ix, vg_search_profile *out) {
  if (!ix || !out) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  *out = ix->prof;
  if (ix->stats.p) {
    DeviceGuard g(ix->device);
    unsigned long long st[kStats] = {};
    VG_CU(cudaMemcpy(st, ix->stats.p, sizeof(st), cudaMemcpyDeviceToHost));
    out->probed_pairs = st[0];
    out->scanned_vectors = st[1];
    out->scanned_code_bytes = st[2];
    out->scored_lists = st[3];
    out->scored_vectors = st[4];
    out->tables_built = st[5];
    out->code_groups = st[6];
    out->seed_scored_lists = st[7];
    out->seed_scored_vectors = st[8];
    out->seed_tables_built = st[9];
    out->seed_code_groups = st[10];
  }
  return VG_OK;
}

int vg_ivfpq_reset_profile(vg_index *ix) {
  if (!ix) return fail(VG_ERR_INVALID_PARAMETER, "null index");
  ix->prof = vg_search_profile{};
  if (ix->stats.p) {
    DeviceGuard g(ix->device);
    VG_CU(cudaMemset(ix->stats.p, 0, kStats * 8));
  }
  return VG_OK;
}

int vg_nccl_unique_id(uint8_t out[128]) {
  if (!out) return fail(VG_ERR_INVALID_PARAMETER, "null output");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return fail(VG_ERR_NCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  std::memcpy(out, &id, 128);
  return VG_OK;
}

int vg_shard_assign_lists(const uint64_t *sizes, size_t num_lists, int world_size, int32_t *owner) {
  if ((!sizes || !owner) && num_lists) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  if (world_size < 1) return fail(VG_ERR_INVALID_PARAMETER, "world_size must be at least 1");
  std::vector<size_t> order(num_lists);
  std::iota(order.begin(), order.end(), size_t(0));
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return sizes[a] > sizes[b]; });
  std::vector<uint64_t> load(world_size, 0);
  for (size_t l : order) {
    int best = 0;
    for (int r = 1; r < world_size; ++r)
      if (load[r] < load[best]) best = r;
    owner[l] = best;
    load[best] += sizes[l];
  }
  return VG_OK;
}

int vg_ivfpq_shard(vg_index *ix, int rank, int world_size, const uint8_t nccl_id[128], int timeout_ms) {
  if (!ix || !nccl_id) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  if (!ix->built) return fail(VG_ERR_NOT_BUILT, "IVF-PQ index is not built: cannot shard");
  if (world_size < 1 || rank < 0 || rank >= world_size)
    return fail(VG_ERR_INVALID_PARAMETER, "rank must be in [0, world_size)");
  if (ix->comm) return fail(VG_ERR_ALREADY_BUILT, "index is already sharded");
  DeviceGuard g(ix->device);
  const size_t Lc = ix->num_centroids;
  std::vector<uint64_t> sizes(Lc);
  for (size_t l = 0; l < Lc; ++l) sizes[l] = ix->h_list_off[l + 1] - ix->h_list_off[l];
  std::vector<int32_t> owner(Lc);
  VG_TRY(vg_shard_assign_lists(sizes.data(), Lc, world_size, owner.data()));
  std::vector<uint8_t> mine(Lc);
  for (size_t l = 0; l < Lc; ++l) mine[l] = owner[l] == rank;
  VG_CU(ix->owner.reserve(std::max<size_t>(Lc, 1)));
  VG_CU(cudaMemcpy(ix->owner.p, mine.data(), Lc, cudaMemcpyHostToDevice));
  ix->comm_timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  if (world_size > 1) {
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = ncclCommInitRankConfig(&comm, world_size, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress)
      return fail(VG_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
    int st = nccl_wait_ready(comm, ix->comm_timeout_ms);
    if (st != VG_OK) {
      ncclCommAbort(comm);
      return st;
    }
    ix->comm = comm;
  }
  ix->rank = rank;
  ix->world = world_size;
  if (world_size > 1) VG_TRY(partition_lists(ix, mine));
  return VG_OK;
}

// ---- flat exact search ----------------------------------------------------

}  // extern "C"

// Flat search: every kFlatSampleStride-th operand tile forms the sample of
// the chunk-maxima pre-pass; per-call workspace of the sampled path at most
// kFlatWorkspaceBytes (query rows in tiles beyond it).
constexpr size_t kFlatSampleStride = 4;
constexpr size_t kFlatWorkspaceBytes = size_t(1) << 30;

// An exhaustive inner-product index over f32 rows (distance.rs:125-130; the
// ground truth of evaluation.rs:250-268): the rows (the caller's device rows
// in place, or a device copy of host rows), their largest norm, and the
// binary16 operand image the tensor-core window reads.
struct vg_flat {
  int device = 0, num_sms = 148;
  size_t n = 0, d = 0;
  DevBuf own_rows;
  const float *rows = nullptr;
  DevBuf img, norm_d;
  // every 4th whole 128-row tile of img, contiguous: the sample whose chunk
  // maxima bound each query's k-th product before the gather pass
  DevBuf sample_img;
  size_t sample_cols = 0;
  int kp = 0;
  float xmax = 0.0f;
  bool tc = false;  // tensor-core path usable (rows of <= 128 floats, norms below 2^14)
  cudaStream_t own_stream = nullptr;
  int *h_err = nullptr, *d_err = nullptr;
  std::mutex mu;
  DevBuf q, qimg, eps, ws, dist, chunk, ids, dst, cnt;
  // profiling: events around the query image, the window kernel and the finisher
  bool profiling = false;
  cudaEvent_t ev[4] = {};
  vg_search_profile prof{};
};

namespace {

// Exact path: SIMT tiles of -dot in the reference's order, a top-k per tile
// and a merge (rows beyond 128 floats, or norms too large for binary16).
int flat_exact(vg_flat *f, const float *dq, size_t nq, size_t k, uint32_t *o_ids, float *o_dist, uint32_t *o_cnt,
               cudaStream_t s) {
  const size_t n = f->n, dim = f->d;
  size_t tile = kDistBudgetBytes * 2 / (nq * 4);
  tile = std::max<size_t>(128, tile / 128 * 128);
  tile = std::min(tile, std::max<size_t>(n, 1));
  const size_t chunks = (n + tile - 1) / tile;
  VG_CU(f->dist.reserve(nq * tile * 4));
  VG_CU(f->chunk.reserve(nq * chunks * k * 8));
  for (size_t ci = 0; ci < chunks; ++ci) {
    const size_t c0 = ci * tile, cols = std::min(tile, n - c0);
    VG_CU(launch_neg_dot(dq, nq, f->rows + c0 * dim, cols, static_cast<int>(dim), f->dist.as<float>(), tile, s));
    VG_CU(launch_select_rows_keys(f->dist.as<float>(), nq, cols, tile, static_cast<int>(k),
                                  f->chunk.as<unsigned long long>() + ci * k, chunks * k, static_cast<uint32_t>(c0),
                                  s));
  }
  VG_CU(launch_merge_keys(f->chunk.as<unsigned long long>(), nq, chunks * k, chunks * k, static_cast<int>(k), nullptr,
                          o_ids, o_dist, o_cnt, nullptr, s));
  return VG_OK;
}

}  // namespace

extern "C" {

int vg_flat_create(const float *db, size_t n, size_t dim, int device, vg_flat **out) {
  if (!out) return fail(VG_ERR_INVALID_PARAMETER, "null output");
  *out = nullptr;
  if (dim == 0) return fail(VG_ERR_INVALID_CONFIG, "invalid config `dimension`: must be greater than 0");
  if (n > 0xfffffffeull) return fail(VG_ERR_INVALID_PARAMETER, "at most 2^32 - 2 database rows");
  if (n && !db) return fail(VG_ERR_INVALID_PARAMETER, "null database rows");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return fail(VG_ERR_CUDA, "no CUDA device " + std::to_string(device) + " (the engine has no CPU path)");
  }
  DeviceGuard g(device);
  auto f = std::make_unique<vg_flat>();
  f->device = device;
  f->n = n;
  f->d = dim;
  cudaDeviceGetAttribute(&f->num_sms, cudaDevAttrMultiProcessorCount, device);
  VG_CU(cudaStreamCreateWithFlags(&f->own_stream, cudaStreamNonBlocking));
  VG_CU(cudaHostAlloc(reinterpret_cast<void **>(&f->h_err), sizeof(int), cudaHostAllocMapped));
  *f->h_err = 0;
  VG_CU(cudaHostGetDevicePointer(reinterpret_cast<void **>(&f->d_err), f->h_err, 0));
  cudaStream_t s = f->own_stream;
  if (n && !is_device_ptr(db)) {
    VG_CU(f->own_rows.reserve(n * dim * 4));
    VG_CU(cudaMemcpyAsync(f->own_rows.p, db, n * dim * 4, cudaMemcpyHostToDevice, s));
    f->rows = f->own_rows.as<float>();
  } else {
    f->rows = db;
  }
  f->kp = umma_kp(static_cast<int>(dim));
  if (n && f->kp && !tc_disabled()) {
    VG_CU(f->norm_d.reserve(4));
    VG_CU(launch_centroid_norm_max(f->rows, n, static_cast<int>(dim), f->norm_d.as<float>(), s));
    VG_CU(cudaMemcpyAsync(&f->xmax, f->norm_d.p, 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaStreamSynchronize(s));
    f->tc = std::isfinite(f->xmax) && f->xmax < 16384.0f;
    if (f->tc) {
      VG_CU(f->img.reserve(umma_image_bytes(n, f->kp)));
      VG_CU(launch_umma_image(f->rows, n, static_cast<int>(dim), f->kp, f->img.p, nullptr, 0.0, 0.0, nullptr, s));
      const size_t full_tiles = n / 128, tile_bytes = static_cast<size_t>(f->kp) * 256;
      if (full_tiles >= 64) {
        const size_t st = (full_tiles + kFlatSampleStride - 1) / kFlatSampleStride;
        VG_CU(f->sample_img.reserve(st * tile_bytes));
        VG_CU(cudaMemcpy2DAsync(f->sample_img.p, tile_bytes, f->img.p, tile_bytes * kFlatSampleStride, tile_bytes,
                                st, cudaMemcpyDeviceToDevice, s));
        f->sample_cols = st * 128;
      }
    }
  }
  VG_CU(cudaStreamSynchronize(s));
  *out = f.release();
  return VG_OK;
}

int vg_flat_destroy(vg_flat *f) {
  if (!f) return VG_OK;
  {
    DeviceGuard g(f->device);
    if (f->own_stream) cudaStreamSynchronize(f->own_stream);
    for (DevBuf *b : {&f->own_rows, &f->img, &f->sample_img, &f->norm_d, &f->q, &f->qimg, &f->eps, &f->ws, &f->dist, &f->chunk,
                      &f->ids, &f->dst, &f->cnt})
      b->release();
    if (f->h_err) cudaFreeHost(f->h_err);
    for (cudaEvent_t e : f->ev)
      if (e) cudaEventDestroy(e);
    if (f->own_stream) cudaStreamDestroy(f->own_stream);
  }
  delete f;
  return VG_OK;
}

int vg_flat_search(vg_flat *f, const float *queries, size_t nq, size_t k, void *stream, uint32_t *out_ids,
                   float *out_dist, uint32_t *out_count) {
  if (!f) return fail(VG_ERR_INVALID_PARAMETER, "null flat index");
  if (k > 256) return fail(VG_ERR_INVALID_PARAMETER, "k must be at most 256");
  if (nq == 0 || k == 0) return VG_OK;
  if (!queries || !out_ids || !out_dist) return fail(VG_ERR_INVALID_PARAMETER, "null query or output buffer");
  DeviceGuard g(f->device);
  std::lock_guard<std::mutex> lock(f->mu);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : f->own_stream;
  const size_t n = f->n, dim = f->d;
  const float *dq = queries;
  if (!is_device_ptr(queries)) {
    VG_CU(f->q.reserve(nq * dim * 4));
    VG_CU(cudaMemcpyAsync(f->q.p, queries, nq * dim * 4, cudaMemcpyHostToDevice, s));
    dq = f->q.as<float>();
  }
  const bool dev_out = is_device_ptr(out_ids) && is_device_ptr(out_dist) && (!out_count || is_device_ptr(out_count));
  uint32_t *o_ids = out_ids, *o_cnt = out_count;
  float *o_dist = out_dist;
  if (!dev_out) {
    VG_CU(f->ids.reserve(nq * k * 4));
    VG_CU(f->dst.reserve(nq * k * 4));
    VG_CU(f->cnt.reserve(nq * 4));
    o_ids = f->ids.as<uint32_t>();
    o_dist = f->dst.as<float>();
    o_cnt = f->cnt.as<uint32_t>();
  }
  *reinterpret_cast<volatile int *>(f->h_err) = 0;
  size_t launches = 3, scan_launches = 1;  // profiling counts of this call's kernels
  if (n == 0) {
    VG_CU(cudaMemsetAsync(o_ids, 0xff, nq * k * 4, s));
    std::vector<float> inf(nq * k, __builtin_inff());
    VG_CU(cudaMemcpyAsync(o_dist, inf.data(), nq * k * 4, cudaMemcpyHostToDevice, s));
    if (o_cnt) VG_CU(cudaMemsetAsync(o_cnt, 0, nq * 4, s));
    VG_CU(cudaStreamSynchronize(s));
  } else if (f->tc) {
    double rel = 0, abs_coef = 0;
    tc_error_coefs(static_cast<int>(dim), &rel, &abs_coef);
    VG_CU(f->qimg.reserve(umma_image_bytes(nq, f->kp)));
    VG_CU(f->eps.reserve(nq * 4));
    // the sampled path when the sample holds at least 4k chunk maxima
    const bool sampled = f->sample_cols / 32 >= 4 * k;
    size_t tile_rows = nq;
    if (sampled) {
      const size_t per_row = tc_sampled_workspace_bytes(1, n, f->sample_cols, static_cast<int>(k));
      tile_rows = std::min(nq, std::max<size_t>(128, kFlatWorkspaceBytes / per_row / 128 * 128));
      VG_CU(f->ws.reserve(tc_sampled_workspace_bytes(tile_rows, n, f->sample_cols, static_cast<int>(k))));
      // per row tile: sampled GEMM, thresholds, gather GEMMs, finisher
      const size_t range = (size_t(16) << 20) / (static_cast<size_t>(f->kp) * 256) * 128;
      const size_t tiles = (nq + tile_rows - 1) / tile_rows;
      scan_launches = tiles * (2 + (n + range - 1) / range);
      launches = 1 + tiles * (3 + (n + range - 1) / range);
    } else {
      VG_CU(f->ws.reserve(tc_select_workspace_bytes(nq, n, static_cast<int>(k), f->num_sms)));
    }
    if (f->profiling) VG_CU(cudaEventRecord(f->ev[0], s));
    VG_CU(launch_umma_image(dq, nq, static_cast<int>(dim), f->kp, f->qimg.p, f->norm_d.as<float>(), rel, abs_coef,
                            f->eps.as<float>(), s));
    for (size_t r0 = 0; sampled && r0 < nq; r0 += tile_rows) {
      const size_t rows = std::min(tile_rows, nq - r0);
      TcSampledSelect t{};
      if (f->profiling) {
        if (r0 == 0) t.marks[0] = f->ev[1];
        if (r0 + rows == nq) {
          t.marks[1] = f->ev[2];
          t.marks[2] = f->ev[3];
        }
      }
      t.a_img = static_cast<const uint8_t *>(f->qimg.p) + r0 / 128 * static_cast<size_t>(f->kp) * 256;
      t.q = dq + r0 * dim;
      t.rows = rows;
      t.b_img = f->img.p;
      t.x = f->rows;
      t.cols = n;
      t.sample_img = f->sample_img.p;
      t.sample_cols = f->sample_cols;
      t.d = static_cast<int>(dim);
      t.kp = f->kp;
      t.P = static_cast<int>(k);
      t.mode = 1;
      t.eps = f->eps.as<float>() + r0;
      t.workspace = f->ws.p;
      t.out_ids = o_ids + r0 * k;
      t.out_dist = o_dist + r0 * k;
      t.out_ld = k;
      t.out_count = o_cnt ? o_cnt + r0 : nullptr;
      t.error = f->d_err;
      VG_CU(launch_tc_sampled_select(t, f->num_sms, s));
    }
    TcSelect t{};
    if (f->profiling) {
      t.marks[0] = f->ev[1];
      t.marks[1] = f->ev[2];
      t.marks[2] = f->ev[3];
    }
    t.a_img = f->qimg.p;
    t.q = dq;
    t.rows = nq;
    t.b_img = f->img.p;
    t.x = f->rows;
    t.cols = n;
    t.d = static_cast<int>(dim);
    t.kp = f->kp;
    t.P = static_cast<int>(k);
    t.mode = 1;
    t.eps = f->eps.as<float>();
    t.workspace = f->ws.p;
    t.out_ids = o_ids;
    t.out_dist = o_dist;
    t.out_ld = k;
    t.out_count = o_cnt;
    t.error = f->d_err;
    if (!sampled) VG_CU(launch_tc_select(t, f->num_sms, s));
  } else {
    VG_TRY(flat_exact(f, dq, nq, k, o_ids, o_dist, o_cnt, s));
  }
  if (!dev_out) {
    VG_CU(cudaMemcpyAsync(out_ids, o_ids, nq * k * 4, cudaMemcpyDeviceToHost, s));
    VG_CU(cudaMemcpyAsync(out_dist, o_dist, nq * k * 4, cudaMemcpyDeviceToHost, s));
    if (out_count) VG_CU(cudaMemcpyAsync(out_count, o_cnt, nq * 4, cudaMemcpyDeviceToHost, s));
  }
  VG_CU(cudaStreamSynchronize(s));
  if (const int code = *reinterpret_cast<volatile int *>(f->h_err))
    return fail(VG_ERR_CUDA, "flat search gave up on a bounded device wait (code " + std::to_string(code) + ")");
  if (f->profiling && f->tc && n) {
    float a = 0, b = 0, c = 0;
    cudaEventElapsedTime(&a, f->ev[0], f->ev[1]);
    cudaEventElapsedTime(&b, f->ev[1], f->ev[2]);
    cudaEventElapsedTime(&c, f->ev[2], f->ev[3]);
    f->prof.normalize_ms += a;  // query image
    f->prof.scan_ms += b;       // tensor-core window kernel
    f->prof.merge_ms += c;      // exact re-score of the windows
    f->prof.total_ms += a + b + c;
    f->prof.calls += 1;
    f->prof.queries += nq;
    f->prof.kernel_launches += launches;
    f->prof.scan_launches += scan_launches;
  }
  return VG_OK;
}

int vg_flat_set_profiling(vg_flat *f, int on) {
  if (!f) return fail(VG_ERR_INVALID_PARAMETER, "null flat index");
  DeviceGuard g(f->device);
  for (cudaEvent_t &e : f->ev)
    if (!e) VG_CU(cudaEventCreate(&e));
  f->profiling = on != 0;
  f->prof = vg_search_profile{};
  return VG_OK;
}

int vg_flat_get_profile(const vg_flat *f, vg_search_profile *out) {
  if (!f || !out) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  *out = f->prof;
  return VG_OK;
}

int vg_flat_search_ip(const float *db, size_t n, const float *queries, size_t nq, size_t dim, size_t k, int device,
                      uint32_t *out_ids, float *out_dist, uint32_t *out_count) {
  if (dim == 0) return fail(VG_ERR_INVALID_CONFIG, "invalid config `dimension`: must be greater than 0");
  if (k > 256) return fail(VG_ERR_INVALID_PARAMETER, "k must be at most 256");
  if (n > 0xfffffffeull) return fail(VG_ERR_INVALID_PARAMETER, "at most 2^32 - 2 database rows");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return fail(VG_ERR_CUDA, "no CUDA device " + std::to_string(device) + " (the engine has no CPU path)");
  }
  if (nq == 0 || k == 0) return VG_OK;
  if (!db || !queries || !out_ids || !out_dist) return fail(VG_ERR_INVALID_PARAMETER, "null argument");
  vg_flat *f = nullptr;
  VG_TRY(vg_flat_create(db, n, dim, device, &f));
  const int st = vg_flat_search(f, queries, nq, k, nullptr, out_ids, out_dist, out_count);
  vg_flat_destroy(f);
  return st;
}

}  // extern "C"
