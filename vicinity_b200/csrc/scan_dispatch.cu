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
cudaError_t launch_scan_stream(const ScanParams &p, int dsub, int gpt, int num_sms, cudaStream_t s);
cudaError_t launch_scan_direct(const ScanParams &p, int num_sms, cudaStream_t s);
cudaError_t launch_scan_four_warp(const ScanParams &p, int num_sms, cudaStream_t s);
bool scan_four_warp_fits(const ScanParams &p);
bool scan_direct_fits(const ScanParams &p);

namespace {
// 1 query-major, 3 query-stream, 4 warp-per-query kernels (direct ADC, 4-bit
// warp) for large batches else the block kernels (default), 5 warp-per-query
// wherever they apply
int g_family = 4;
}  // namespace

void set_scan_family(int family) { g_family = family; }

namespace {
// The direct kernel gives each query one warp for its whole search: it needs
// a batch that keeps every warp busy (16 queries per SM here); smaller
// batches go to the query-stream kernel, whose blocks share a query.
bool use_direct(const ScanParams &p, int num_sms) {
  return scan_direct_fits(p) && (g_family == 5 || p.force_warp || p.nq >= 16 * num_sms);
}
bool use_four_warp(const ScanParams &p, int num_sms) {
  return (g_family >= 4 || p.force_warp) && scan_four_warp_fits(p) &&
         (g_family == 5 || p.force_warp || p.nq >= 16 * num_sms);
}
}  // namespace

namespace {
int pick_gpt(const ScanParams &p) {
  if (p.dsub < 1 || p.dsub > 8 || p.k > 32 || p.ks % 4 != 0) return 0;
  const int ngroups = p.M * p.ks / 4;
  for (int gpt = 1; gpt <= 4; gpt <<= 1)
    if (gpt * kScanThreads >= ngroups && gpt * 4 * p.dsub <= 64) return gpt;
  return 0;
}
}  // namespace

cudaError_t launch_ivfpq_scan(const ScanParams &p, int num_sms, cudaStream_t s) {
  if (p.k < 1 || p.k > 256) return cudaErrorInvalidValue;
  if (p.key_floor) {  // a key floor is applied by the query-major and 4-bit block kernels only
    const int gpt = pick_gpt(p);
    if (p.ks == 16) return launch_scan_four(p, gpt ? p.dsub : 0, gpt, num_sms, s);
    return launch_scan_eight(p, gpt ? p.dsub : 0, gpt, num_sms, s);
  }
  // an OPQ rotation is applied by the query-major and 4-bit kernels only
  if ((g_family >= 4 || p.force_warp) && use_direct(p, num_sms)) return launch_scan_direct(p, num_sms, s);
  const int gpt = pick_gpt(p);
  if (g_family >= 3 && gpt && p.ks == 256 && !p.rot_t && p.probe_rec && p.P <= 256)
    return launch_scan_stream(p, p.dsub, gpt, num_sms, s);
  if (p.ks == 16) {
    if (use_four_warp(p, num_sms)) return launch_scan_four_warp(p, num_sms, s);
    return launch_scan_four(p, gpt ? p.dsub : 0, gpt, num_sms, s);
  }
  return launch_scan_eight(p, gpt ? p.dsub : 0, gpt, num_sms, s);
}

bool ivfpq_scan_warp_applies(const ScanParams &p) {
  return p.k >= 1 && p.k <= 64 && !p.key_floor && (scan_direct_fits(p) || (p.ks == 16 && scan_four_warp_fits(p)));
}

cudaError_t launch_ivfpq_scan_generic(const ScanParams &p, int num_sms, cudaStream_t s) {
  if (p.k < 1 || p.k > 256) return cudaErrorInvalidValue;
  const int gpt = p.ks == 256 ? pick_gpt(p) : 0;
  return launch_scan_eight(p, gpt ? p.dsub : 0, gpt, num_sms, s);
}

int ivfpq_scan_variant_name(const ScanParams &p, int num_sms, char *buf, size_t len) {
  if ((g_family >= 4 || p.force_warp) && !p.key_floor && use_direct(p, num_sms))
    return snprintf(buf, len, "ivfpq_direct_kernel<%d,%d>", p.dsub, p.k <= 32 ? 1 : 2);
  const int gpt = pick_gpt(p);
  if (g_family >= 3 && gpt && p.ks == 256 && !p.rot_t && !p.key_floor && p.probe_rec && p.P <= 256)
    return snprintf(buf, len, "ivfpq_stream_kernel<%d,%d,1,256>", p.dsub, gpt);
  if (!p.key_floor && use_four_warp(p, num_sms)) return snprintf(buf, len, "ivfpq_four_warp_kernel<%d>", p.k <= 32 ? 1 : 2);
  if (p.ks == 16) return snprintf(buf, len, "ivfpq_four_kernel<%d>", p.k <= 32 ? 1 : p.k <= 64 ? 2 : p.k <= 128 ? 4 : 8);
  return snprintf(buf, len, "ivfpq_query_kernel<%d,%d,%d,%s>", gpt ? p.dsub : 0, gpt,
                  p.k <= 32 ? 1 : p.k <= 64 ? 2 : p.k <= 128 ? 4 : 8, p.ks == 16 ? "4bit" : "8bit");
}

}  // namespace vg
