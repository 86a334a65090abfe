// Host side of OPQ training (src/ivf_pq/opq.rs:207-290,
// compute_optimal_rotation): the orthogonal Procrustes solution R = U V^T of
// the cross-covariance M = U S V^T.  The reference takes the SVD from
// nalgebra; this is a one-sided Jacobi SVD in double precision (Hestenes'
// method), so trained rotations are not bit-identical to the reference's --
// only their use (encode and search with a given R) is.
#include <algorithm>
#include <cmath>
#include <vector>

#include "opq.h"

namespace vg {

std::vector<float> procrustes_rotation(const std::vector<double> &m, size_t d) {
  // A <- M; rotate column pairs of A (and of V) until they are orthogonal:
  // then A = U S and M = A V^T.
  std::vector<double> a(m), v(d * d, 0.0);
  for (size_t i = 0; i < d; ++i) v[i * d + i] = 1.0;
  for (int sweep = 0; sweep < 60; ++sweep) {
    double off = 0.0;
    for (size_t p = 0; p + 1 < d; ++p) {
      for (size_t q = p + 1; q < d; ++q) {
        double alpha = 0.0, beta = 0.0, gamma = 0.0;
        for (size_t i = 0; i < d; ++i) {
          const double ap = a[i * d + p], aq = a[i * d + q];
          alpha += ap * ap;
          beta += aq * aq;
          gamma += ap * aq;
        }
        if (gamma == 0.0 || std::fabs(gamma) <= 1e-15 * std::sqrt(alpha * beta)) continue;
        off = std::max(off, std::fabs(gamma) / std::sqrt(alpha * beta));
        const double zeta = (beta - alpha) / (2.0 * gamma);
        const double t = (zeta >= 0 ? 1.0 : -1.0) / (std::fabs(zeta) + std::sqrt(1.0 + zeta * zeta));
        const double c = 1.0 / std::sqrt(1.0 + t * t), s = c * t;
        for (size_t i = 0; i < d; ++i) {
          const double ap = a[i * d + p], aq = a[i * d + q];
          a[i * d + p] = c * ap - s * aq;
          a[i * d + q] = s * ap + c * aq;
          const double vp = v[i * d + p], vq = v[i * d + q];
          v[i * d + p] = c * vp - s * vq;
          v[i * d + q] = s * vp + c * vq;
        }
      }
    }
    if (off < 1e-14) break;
  }
  // U: columns of A normalised; columns of (near-)zero singular value are
  // completed to an orthonormal basis by Gram-Schmidt on unit vectors
  std::vector<double> u(d * d, 0.0), norm(d);
  double top = 0.0;
  for (size_t c = 0; c < d; ++c) {
    double s = 0.0;
    for (size_t i = 0; i < d; ++i) s += a[i * d + c] * a[i * d + c];
    norm[c] = std::sqrt(s);
    top = std::max(top, norm[c]);
  }
  std::vector<bool> have(d, false);
  for (size_t c = 0; c < d; ++c) {
    if (norm[c] > 1e-12 * top && norm[c] > 0.0) {
      for (size_t i = 0; i < d; ++i) u[i * d + c] = a[i * d + c] / norm[c];
      have[c] = true;
    }
  }
  size_t basis = 0;
  for (size_t c = 0; c < d; ++c) {
    if (have[c]) continue;
    for (; basis < d; ++basis) {
      std::vector<double> e(d, 0.0);
      e[basis] = 1.0;
      for (size_t o = 0; o < d; ++o) {
        if (!have[o]) continue;
        double dot = 0.0;
        for (size_t i = 0; i < d; ++i) dot += u[i * d + o] * e[i];
        for (size_t i = 0; i < d; ++i) e[i] -= dot * u[i * d + o];
      }
      double s = 0.0;
      for (double x : e) s += x * x;
      if (s > 1e-6) {
        s = std::sqrt(s);
        for (size_t i = 0; i < d; ++i) u[i * d + c] = e[i] / s;
        have[c] = true;
        ++basis;
        break;
      }
    }
  }
  // R = U V^T
  std::vector<float> r(d * d);
  for (size_t i = 0; i < d; ++i)
    for (size_t j = 0; j < d; ++j) {
      double s = 0.0;
      for (size_t k = 0; k < d; ++k) s += u[i * d + k] * v[j * d + k];
      r[i * d + j] = static_cast<float>(s);
    }
  return r;
}

}  // namespace vg
