// OPQ training helpers (host).
#pragma once

#include <cstddef>
#include <vector>

namespace vg {

// R = U V^T for the d x d cross-covariance m = U S V^T (row-major, double):
// the rotation compute_optimal_rotation returns (src/ivf_pq/opq.rs:207-290).
std::vector<float> procrustes_rotation(const std::vector<double> &m, size_t d);

}  // namespace vg
