// Launcher of the 4-bit (16-entry codebook) search kernel, scan_fourbit.cuh.
#include "scan_fourbit.cuh"

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

cudaError_t launch_scan_four(const ScanParams &p, int, int, int num_sms, cudaStream_t s) {
  if (p.ks != 16) return cudaErrorInvalidValue;
  if (p.k <= 32) return launch_four_variant<1>(p, num_sms, s);
  if (p.k <= 64) return launch_four_variant<2>(p, num_sms, s);
  if (p.k <= 128) return launch_four_variant<4>(p, num_sms, s);
  return launch_four_variant<8>(p, num_sms, s);
}

}  // namespace vg
