// Instantiations of the fused search kernel for general (8-bit) codebooks.
// One case per (subvector dimensions, 4-entry groups per thread) the dispatcher can pick.
#include "scan_kernel.cuh"

namespace vg {

cudaError_t launch_scan_eight(const ScanParams &p, int dsub, int gpt, int num_sms, cudaStream_t s) {
  if (gpt == 0) {
    if (p.k <= 32) return launch_scan_variant<0, 0, 1, 0>(p, num_sms, s);
    if (p.k <= 64) return launch_scan_variant<0, 0, 2, 0>(p, num_sms, s);
    if (p.k <= 128) return launch_scan_variant<0, 0, 4, 0>(p, num_sms, s);
    return launch_scan_variant<0, 0, 8, 0>(p, num_sms, s);
  }
  if (p.ks == 256) {
    switch (dsub * 100 + gpt) {
      case 101: return launch_scan_variant<1, 1, 1, 256>(p, num_sms, s);
      case 102: return launch_scan_variant<1, 2, 1, 256>(p, num_sms, s);
      case 104: return launch_scan_variant<1, 4, 1, 256>(p, num_sms, s);
      case 201: return launch_scan_variant<2, 1, 1, 256>(p, num_sms, s);
      case 202: return launch_scan_variant<2, 2, 1, 256>(p, num_sms, s);
      case 204: return launch_scan_variant<2, 4, 1, 256>(p, num_sms, s);
      case 301: return launch_scan_variant<3, 1, 1, 256>(p, num_sms, s);
      case 302: return launch_scan_variant<3, 2, 1, 256>(p, num_sms, s);
      case 304: return launch_scan_variant<3, 4, 1, 256>(p, num_sms, s);
      case 401: return launch_scan_variant<4, 1, 1, 256>(p, num_sms, s);
      case 402: return launch_scan_variant<4, 2, 1, 256>(p, num_sms, s);
      case 404: return launch_scan_variant<4, 4, 1, 256>(p, num_sms, s);
      case 501: return launch_scan_variant<5, 1, 1, 256>(p, num_sms, s);
      case 502: return launch_scan_variant<5, 2, 1, 256>(p, num_sms, s);
      case 601: return launch_scan_variant<6, 1, 1, 256>(p, num_sms, s);
      case 602: return launch_scan_variant<6, 2, 1, 256>(p, num_sms, s);
      case 701: return launch_scan_variant<7, 1, 1, 256>(p, num_sms, s);
      case 702: return launch_scan_variant<7, 2, 1, 256>(p, num_sms, s);
      case 801: return launch_scan_variant<8, 1, 1, 256>(p, num_sms, s);
      case 802: return launch_scan_variant<8, 2, 1, 256>(p, num_sms, s);
      default: break;
    }
  }
  {
    switch (dsub * 100 + gpt) {
      case 101: return launch_scan_variant<1, 1, 1, 0>(p, num_sms, s);
      case 102: return launch_scan_variant<1, 2, 1, 0>(p, num_sms, s);
      case 104: return launch_scan_variant<1, 4, 1, 0>(p, num_sms, s);
      case 201: return launch_scan_variant<2, 1, 1, 0>(p, num_sms, s);
      case 202: return launch_scan_variant<2, 2, 1, 0>(p, num_sms, s);
      case 204: return launch_scan_variant<2, 4, 1, 0>(p, num_sms, s);
      case 301: return launch_scan_variant<3, 1, 1, 0>(p, num_sms, s);
      case 302: return launch_scan_variant<3, 2, 1, 0>(p, num_sms, s);
      case 304: return launch_scan_variant<3, 4, 1, 0>(p, num_sms, s);
      case 401: return launch_scan_variant<4, 1, 1, 0>(p, num_sms, s);
      case 402: return launch_scan_variant<4, 2, 1, 0>(p, num_sms, s);
      case 404: return launch_scan_variant<4, 4, 1, 0>(p, num_sms, s);
      case 501: return launch_scan_variant<5, 1, 1, 0>(p, num_sms, s);
      case 502: return launch_scan_variant<5, 2, 1, 0>(p, num_sms, s);
      case 601: return launch_scan_variant<6, 1, 1, 0>(p, num_sms, s);
      case 602: return launch_scan_variant<6, 2, 1, 0>(p, num_sms, s);
      case 701: return launch_scan_variant<7, 1, 1, 0>(p, num_sms, s);
      case 702: return launch_scan_variant<7, 2, 1, 0>(p, num_sms, s);
      case 801: return launch_scan_variant<8, 1, 1, 0>(p, num_sms, s);
      case 802: return launch_scan_variant<8, 2, 1, 0>(p, num_sms, s);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace vg
