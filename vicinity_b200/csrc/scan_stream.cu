// Instantiations of the query-stream search kernel (256-entry codebooks).
// One case per (subvector dimensions, 4-entry groups per thread).
#include "scan_stream.cuh"

namespace vg {

cudaError_t launch_scan_stream(const ScanParams &p, int dsub, int gpt, int num_sms, cudaStream_t s) {
  switch (dsub * 100 + gpt) {
    case 101: return launch_stream_variant<1, 1, 1, 256>(p, num_sms, s);
    case 102: return launch_stream_variant<1, 2, 1, 256>(p, num_sms, s);
    case 104: return launch_stream_variant<1, 4, 1, 256>(p, num_sms, s);
    case 201: return launch_stream_variant<2, 1, 1, 256>(p, num_sms, s);
    case 202: return launch_stream_variant<2, 2, 1, 256>(p, num_sms, s);
    case 204: return launch_stream_variant<2, 4, 1, 256>(p, num_sms, s);
    case 301: return launch_stream_variant<3, 1, 1, 256>(p, num_sms, s);
    case 302: return launch_stream_variant<3, 2, 1, 256>(p, num_sms, s);
    case 304: return launch_stream_variant<3, 4, 1, 256>(p, num_sms, s);
    case 401: return launch_stream_variant<4, 1, 1, 256>(p, num_sms, s);
    case 402: return launch_stream_variant<4, 2, 1, 256>(p, num_sms, s);
    case 404: return launch_stream_variant<4, 4, 1, 256>(p, num_sms, s);
    case 501: return launch_stream_variant<5, 1, 1, 256>(p, num_sms, s);
    case 502: return launch_stream_variant<5, 2, 1, 256>(p, num_sms, s);
    case 601: return launch_stream_variant<6, 1, 1, 256>(p, num_sms, s);
    case 602: return launch_stream_variant<6, 2, 1, 256>(p, num_sms, s);
    case 701: return launch_stream_variant<7, 1, 1, 256>(p, num_sms, s);
    case 702: return launch_stream_variant<7, 2, 1, 256>(p, num_sms, s);
    case 801: return launch_stream_variant<8, 1, 1, 256>(p, num_sms, s);
    case 802: return launch_stream_variant<8, 2, 1, 256>(p, num_sms, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vg
