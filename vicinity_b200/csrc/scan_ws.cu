// Instantiations of the warp-specialised search kernel (256-entry codebooks).
// One case per (subvector dimensions, codebook entries per producer thread).
#include "scan_ws.cuh"

namespace vg {

cudaError_t launch_scan_ws(const ScanParams &p, int dsub, int ept, int num_sms, cudaStream_t s) {
  switch (dsub * 100 + ept) {
    case 103: return launch_ws_variant<1, 3, 1, 256>(p, num_sms, s);
    case 106: return launch_ws_variant<1, 6, 1, 256>(p, num_sms, s);
    case 111: return launch_ws_variant<1, 11, 1, 256>(p, num_sms, s);
    case 122: return launch_ws_variant<1, 22, 1, 256>(p, num_sms, s);
    case 203: return launch_ws_variant<2, 3, 1, 256>(p, num_sms, s);
    case 206: return launch_ws_variant<2, 6, 1, 256>(p, num_sms, s);
    case 211: return launch_ws_variant<2, 11, 1, 256>(p, num_sms, s);
    case 222: return launch_ws_variant<2, 22, 1, 256>(p, num_sms, s);
    case 303: return launch_ws_variant<3, 3, 1, 256>(p, num_sms, s);
    case 306: return launch_ws_variant<3, 6, 1, 256>(p, num_sms, s);
    case 311: return launch_ws_variant<3, 11, 1, 256>(p, num_sms, s);
    case 322: return launch_ws_variant<3, 22, 1, 256>(p, num_sms, s);
    case 403: return launch_ws_variant<4, 3, 1, 256>(p, num_sms, s);
    case 406: return launch_ws_variant<4, 6, 1, 256>(p, num_sms, s);
    case 411: return launch_ws_variant<4, 11, 1, 256>(p, num_sms, s);
    case 422: return launch_ws_variant<4, 22, 1, 256>(p, num_sms, s);
    case 503: return launch_ws_variant<5, 3, 1, 256>(p, num_sms, s);
    case 506: return launch_ws_variant<5, 6, 1, 256>(p, num_sms, s);
    case 511: return launch_ws_variant<5, 11, 1, 256>(p, num_sms, s);
    case 603: return launch_ws_variant<6, 3, 1, 256>(p, num_sms, s);
    case 606: return launch_ws_variant<6, 6, 1, 256>(p, num_sms, s);
    case 611: return launch_ws_variant<6, 11, 1, 256>(p, num_sms, s);
    case 703: return launch_ws_variant<7, 3, 1, 256>(p, num_sms, s);
    case 706: return launch_ws_variant<7, 6, 1, 256>(p, num_sms, s);
    case 711: return launch_ws_variant<7, 11, 1, 256>(p, num_sms, s);
    case 803: return launch_ws_variant<8, 3, 1, 256>(p, num_sms, s);
    case 806: return launch_ws_variant<8, 6, 1, 256>(p, num_sms, s);
    case 811: return launch_ws_variant<8, 11, 1, 256>(p, num_sms, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vg
