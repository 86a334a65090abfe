// Variant selection for the fused search kernel (scan_kernel.cuh).
//
// Register-resident codebooks are used when the subvector has at most 8
// dimensions and the whole codebook fits in EPT entries per thread with at
// most 64 codebook floats per thread; k <= 32 keeps one top-k row per lane.
// Everything else (longer subvectors, huge codebooks, k up to 256) runs the
// general variant.
#include <stdio.h>

#include "scan_kernel.cuh"

namespace vg {

cudaError_t launch_scan_four(const ScanParams &p, int dsub, int ept, int num_sms, cudaStream_t s);
cudaError_t launch_scan_eight(const ScanParams &p, int dsub, int ept, int num_sms, cudaStream_t s);

namespace {
int pick_ept(const ScanParams &p) {
  if (p.dsub < 1 || p.dsub > 8 || p.k > 32) return 0;
  const int nent = p.M * p.ks;
  const int max_ept = p.ks == 16 ? 4 : 16;
  for (int ept = 1; ept <= max_ept; ept <<= 1)
    if (ept * kScanThreads >= nent && ept * p.dsub <= 64) return ept;
  return 0;
}
}  // namespace

cudaError_t launch_ivfpq_scan(const ScanParams &p, int num_sms, cudaStream_t s) {
  if (p.k < 1 || p.k > 256) return cudaErrorInvalidValue;
  const int ept = pick_ept(p);
  if (p.ks == 16) return launch_scan_four(p, ept ? p.dsub : 0, ept, num_sms, s);
  return launch_scan_eight(p, ept ? p.dsub : 0, ept, num_sms, s);
}

int ivfpq_scan_variant_name(const ScanParams &p, char *buf, size_t len) {
  const int ept = pick_ept(p);
  return snprintf(buf, len, "ivfpq_query_kernel<%d,%d,%d,%s>", ept ? p.dsub : 0, ept,
                  p.k <= 32 ? 1 : p.k <= 64 ? 2 : p.k <= 128 ? 4 : 8, p.ks == 16 ? "4bit" : "8bit");
}

}  // namespace vg
