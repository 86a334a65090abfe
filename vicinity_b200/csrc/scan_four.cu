// Launchers of the 4-bit (16-entry codebook) search kernels: block per query
// (scan_fourbit.cuh) and warp per query (scan_four_warp.cuh).
#include "scan_four_warp.cuh"

namespace vg {

namespace {
template <int R>
cudaError_t launch_four_variant(const ScanParams &p, int num_sms, cudaStream_t s) {
  auto kern = ivfpq_four_kernel<R>;
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  const size_t reserve = 14336;  // static shared memory of the kernel (~12.3 KB)
  const size_t smem = four_smem_bytes(p.M, p.dsub, R, p.rot_t != nullptr);
  if (smem + reserve > static_cast<size_t>(optin)) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int grid = num_sms * per_sm;
  if (grid > p.nq) grid = p.nq;
  kern<<<grid, kScanThreads, smem, s>>>(p);
  return cudaGetLastError();
}
}  // namespace

bool scan_four_warp_fits(const ScanParams &p) {
  return p.ks == 16 && !p.rot_t && !p.qmap && !p.category && p.k <= 64 && p.dsub >= 1 &&
         four_warp_smem_bytes(p.M, p.dsub, p.d) <= 200 * 1024;
}

cudaError_t launch_scan_four_warp(const ScanParams &p, int num_sms, cudaStream_t s) {
  if (!scan_four_warp_fits(p)) return cudaErrorInvalidValue;
  const size_t smem = four_warp_smem_bytes(p.M, p.dsub, p.d);
  auto kern1 = ivfpq_four_warp_kernel<1>;
  auto kern2 = ivfpq_four_warp_kernel<2>;
  auto kern = p.k <= 32 ? kern1 : kern2;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int grid = num_sms < p.nq ? num_sms : p.nq;  // one block per SM, a warp per query at a time
  if (grid < 1) grid = 1;
  kern<<<grid, kFourWarpThreads, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_scan_four(const ScanParams &p, int, int, int num_sms, cudaStream_t s) {
  if (p.ks != 16) return cudaErrorInvalidValue;
  if (p.k <= 32) return launch_four_variant<1>(p, num_sms, s);
  if (p.k <= 64) return launch_four_variant<2>(p, num_sms, s);
  if (p.k <= 128) return launch_four_variant<4>(p, num_sms, s);
  return launch_four_variant<8>(p, num_sms, s);
}

}  // namespace vg
