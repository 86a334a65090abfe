// Exact flat inner-product search that allocates nothing
// (vg_flat_search_ip_noalloc).
//
// Who needs it: callers that cannot allocate device memory at search time --
// serving processes whose device memory is handed out up front to another
// allocator (a framework's caching pool, a per-process memory budget), loops
// where cudaMalloc/cudaFree's implicit device synchronisation and latency are
// not acceptable, and embedders that forbid driver allocations after
// start-up.  vg_flat_search_ip grows a per-device workspace with cudaMalloc
// and stages host buffers; this entry point computes the same result but
// takes every byte of scratch -- the distance tile and the per-tile top-k
// keys -- from one fixed device array defined in this file, and accepts only
// device memory for its inputs and outputs.
//
// What a caller must know:
//   - The scratch is a file-scope `static __device__` array of
//     kFlatScratchBytes (32 MiB).  A GPU holds it, for the life of the
//     process, from the first call on that GPU.  A request whose scratch would
//     exceed it returns VG_ERR_INVALID_PARAMETER with a message saying so:
//     split the query batch (the scratch grows with nq) instead.
//   - Host code cannot hand the array's name to a kernel (on the host it is a
//     shadow symbol, not a device address).  The first call on each device
//     resolves the address with cudaGetSymbolAddress while that device is
//     current, checks the result and caches it; later calls reuse it.
//   - Every call shares the one array and the array keeps whatever the last
//     call left there.  Each scratch element a call reads was written earlier
//     in the same call, so nothing has to start at zero and nothing is
//     cleared.  Calls whose GPU work overlaps (two host threads, or two
//     streams, at the same time) race on the scratch and give wrong results:
//     serialise them.
//   - The call allocates nothing: no cudaMalloc, cudaFree, stream or event
//     creation, and no host allocation on the success path (a failure stores
//     its message for vg_last_error).  Work is enqueued on the caller's
//     stream, and the call returns after that stream has finished it.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>

#include "kernels.h"
#include "vicinity_gpu.h"

namespace vg {
void set_last_error(const char *msg);
}

namespace {

constexpr size_t kFlatScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_flat_scratch[kFlatScratchBytes];

// Device address of g_flat_scratch per device ordinal, resolved once.
std::atomic<void *> g_scratch_addr[kMaxDevices];

int noalloc_fail(int code, const char *msg) {
  vg::set_last_error(msg);
  return code;
}

int noalloc_cuda_fail(cudaError_t e, const char *what) {
  cudaGetLastError();  // clear a sticky launch error so later calls start clean
  char buf[256];
  std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  vg::set_last_error(buf);
  return VG_ERR_CUDA;
}

// True when p is device (or managed) memory usable from `device`.
bool device_memory_on(const void *p, int device) {
  cudaPointerAttributes a;
  if (!p || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type == cudaMemoryTypeManaged) return true;
  return a.type == cudaMemoryTypeDevice && a.device == device;
}

}  // namespace

extern "C" int vg_flat_search_ip_noalloc(const float *db, size_t n, const float *queries, size_t nq, size_t dim,
                                         size_t k, int device, void *stream, uint32_t *out_ids, float *out_dist,
                                         uint32_t *out_count) {
  if (dim == 0) return noalloc_fail(VG_ERR_INVALID_CONFIG, "invalid config `dimension`: must be greater than 0");
  if (k > 256) return noalloc_fail(VG_ERR_INVALID_PARAMETER, "k must be at most 256");
  if (n > 0xfffffffeull) return noalloc_fail(VG_ERR_INVALID_PARAMETER, "at most 2^32 - 2 database rows");
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count || device >= kMaxDevices) {
    cudaGetLastError();
    return noalloc_fail(VG_ERR_CUDA, "no such CUDA device (the engine has no CPU path)");
  }
  if (nq == 0 || k == 0) return VG_OK;

  // Scratch layout: distance tile [nq][tile] f32 (at most half the array),
  // then 256-aligned per-tile keys [nq][chunks][k] u64.  The tile is the
  // widest multiple of 128 columns that fits, capped at n rounded up to 128.
  size_t tile = (kFlatScratchBytes / 2) / (nq * sizeof(float));
  tile = tile / 128 * 128;
  if (tile == 0)
    return noalloc_fail(VG_ERR_INVALID_PARAMETER,
                        "vg_flat_search_ip_noalloc: nq above 32768 does not fit the fixed 32 MiB scratch; "
                        "split the query batch");
  if (n > 0 && tile > n) tile = (n + 127) / 128 * 128;
  const size_t chunks = (n + tile - 1) / tile;
  const size_t dist_bytes = (nq * tile * sizeof(float) + 255) & ~size_t(255);
  const size_t key_bytes = nq * chunks * k * sizeof(unsigned long long);
  if (dist_bytes + key_bytes > kFlatScratchBytes)
    return noalloc_fail(VG_ERR_INVALID_PARAMETER,
                        "vg_flat_search_ip_noalloc: nq * k * (n / tile) top-k keys exceed the fixed 32 MiB "
                        "scratch; split the query batch");

  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return noalloc_cuda_fail(e, "cudaSetDevice");
  struct Restore {
    int dev;
    ~Restore() {
      if (dev >= 0) cudaSetDevice(dev);
    }
  } restore{prev};

  if ((n > 0 && !device_memory_on(db, device)) || !device_memory_on(queries, device) ||
      !device_memory_on(out_ids, device) || !device_memory_on(out_dist, device) ||
      (out_count && !device_memory_on(out_count, device)))
    return noalloc_fail(VG_ERR_INVALID_PARAMETER,
                        "vg_flat_search_ip_noalloc takes device memory of `device` only, for inputs and outputs");

  void *base = g_scratch_addr[device].load(std::memory_order_acquire);
  if (!base) {
    e = cudaGetSymbolAddress(&base, g_flat_scratch);
    if (e != cudaSuccess || !base) return noalloc_cuda_fail(e, "cudaGetSymbolAddress(g_flat_scratch)");
    g_scratch_addr[device].store(base, std::memory_order_release);
  }
  float *dist = static_cast<float *>(base);
  unsigned long long *keys = reinterpret_cast<unsigned long long *>(static_cast<unsigned char *>(base) + dist_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // A launch that fails part way leaves earlier kernels of this call queued
  // on the stream, still using the shared scratch: wait for them (whatever
  // the outcome) before returning, so a failed call has also finished with
  // the scratch when it returns.
  auto fail_after_launches = [&](cudaError_t err, const char *what) {
    const int code = noalloc_cuda_fail(err, what);
    cudaStreamSynchronize(s);
    cudaGetLastError();
    return code;
  };
  for (size_t ci = 0; ci < chunks; ++ci) {
    const size_t c0 = ci * tile, cols = (n - c0) < tile ? (n - c0) : tile;
    e = vg::launch_neg_dot(queries, nq, db + c0 * dim, cols, static_cast<int>(dim), dist, tile, s);
    if (e != cudaSuccess) return fail_after_launches(e, "distance tile");
    e = vg::launch_select_rows_keys(dist, nq, cols, tile, static_cast<int>(k), keys + ci * k, chunks * k,
                                    static_cast<uint32_t>(c0), s);
    if (e != cudaSuccess) return fail_after_launches(e, "tile top-k");
  }
  // With n == 0 the merge reads nothing and writes the padding (id
  // 0xffffffff, +inf, count 0), as vg_flat_search_ip does.
  e = vg::launch_merge_keys(keys, nq, chunks * k, chunks * k, static_cast<int>(k), nullptr, out_ids, out_dist,
                            out_count, nullptr, s);
  if (e != cudaSuccess) return fail_after_launches(e, "merge");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return noalloc_cuda_fail(e, "cudaStreamSynchronize");
  return VG_OK;
}
