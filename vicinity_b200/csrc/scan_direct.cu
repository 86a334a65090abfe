// Instantiations of the direct-ADC search kernel (256-entry codebooks): one
// case per (subvector dimensions, top-k rows).
#include "scan_direct.cuh"

namespace vg {

cudaError_t launch_scan_direct(const ScanParams &p, int num_sms, cudaStream_t s) {
  const int R = p.k <= 32 ? 1 : p.k <= 64 ? 2 : 0;
  switch (p.dsub * 10 + R) {
    case 11: return launch_direct_variant<1, 1>(p, num_sms, s);
    case 12: return launch_direct_variant<1, 2>(p, num_sms, s);
    case 21: return launch_direct_variant<2, 1>(p, num_sms, s);
    case 22: return launch_direct_variant<2, 2>(p, num_sms, s);
    case 31: return launch_direct_variant<3, 1>(p, num_sms, s);
    case 32: return launch_direct_variant<3, 2>(p, num_sms, s);
    case 41: return launch_direct_variant<4, 1>(p, num_sms, s);
    case 42: return launch_direct_variant<4, 2>(p, num_sms, s);
    case 51: return launch_direct_variant<5, 1>(p, num_sms, s);
    case 52: return launch_direct_variant<5, 2>(p, num_sms, s);
    case 61: return launch_direct_variant<6, 1>(p, num_sms, s);
    case 62: return launch_direct_variant<6, 2>(p, num_sms, s);
    case 71: return launch_direct_variant<7, 1>(p, num_sms, s);
    case 72: return launch_direct_variant<7, 2>(p, num_sms, s);
    case 81: return launch_direct_variant<8, 1>(p, num_sms, s);
    case 82: return launch_direct_variant<8, 2>(p, num_sms, s);
    default: return cudaErrorInvalidValue;
  }
}

bool scan_direct_fits(const ScanParams &p) {
  return p.ks == 256 && !p.rot_t && p.probe_rec && p.dsub >= 1 && p.dsub <= 8 && p.k <= 64 &&
         direct_smem_bytes(p.M, p.dsub) <= 200 * 1024;
}

}  // namespace vg
