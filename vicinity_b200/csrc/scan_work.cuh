// Work items of the warp-per-query scan kernels (ScanParams::unit_probes,
// work, work_count).  A warp takes item numbers from a global counter; an item
// is a query, or a unit (query, group of probes) when unit_probes > 0, and a
// work list, when given, maps item numbers to items (heavy items first).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace vg {

struct ScanWork {
  uint32_t total = 0, front = 0, units = 1;

  __device__ __forceinline__ void init(const ScanParams &p) {
    units = p.unit_probes > 0 ? static_cast<uint32_t>((p.P + p.unit_probes - 1) / p.unit_probes) : 1u;
    if (p.work) {
      front = p.work_count[0];
      total = front + p.work_count[1];
    } else {
      total = static_cast<uint32_t>(p.nq) * units;
    }
  }

  // Item number w (< total) -> query q, unit g, probes [lo, hi) and the
  // output row of its keys.
  __device__ __forceinline__ void item(const ScanParams &p, uint32_t w, uint32_t &q, int &lo, int &hi,
                                       size_t &orow) const {
    uint32_t it = w;
    if (p.work) it = w < front ? p.work[w] : p.work[p.work_cap - 1 - (w - front)];
    q = it / units;
    const int g = static_cast<int>(it - q * units);
    lo = p.probe_from ? static_cast<int>(p.probe_from[q]) : 0;
    hi = p.P;
    orow = q;
    if (p.unit_probes > 0) {
      lo = max(lo, g * p.unit_probes);
      hi = min(hi, (g + 1) * p.unit_probes);
      orow = static_cast<size_t>(1 + g) * static_cast<size_t>(p.nq) + q;
    }
  }
};

}  // namespace vg
