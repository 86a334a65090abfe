// TEST INFRASTRUCTURE ONLY -- CPU restatement of the vicinity 0.12.0 IVF-PQ
// path; see ivfpq_oracle.h for the arithmetic contract and how it is pinned.
// Must be compiled with -ffp-contract=off (no FMA contraction) and without
// -ffast-math, so that every f32 sum is sequential and separately rounded as
// the Rust reference computes it.
#include "ivfpq_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

constexpr size_t kSimdBatchThreshold = 16;  // search.rs:32
constexpr size_t kFastscanMaxCodebooks = 65535 / 255;  // pq_simd.rs:517

// Sequential dot product: simd.rs:90-92 (fallback `dot`), summing products in
// index order.  The Rust fold starts at -0.0; starting at +0.0 differs only
// when every product is -0.0 (the sum is then +0.0 here, -0.0 there): 1 - dot
// cannot show it, and the flat search's -dot shows it only as the sign of a
// zero distance for such a row (a zero query against a row of negative
// coordinates, or the reverse).  The engine sums the same way.
inline float dot_seq(const float *a, const float *b, size_t d) {
  float s = 0.0f;
  for (size_t j = 0; j < d; ++j) s += a[j] * b[j];
  return s;
}

// simd.rs:121-124 (fallback `l2_distance_squared`): sum of (x - y)^2 in order.
inline float l2sq_seq(const float *a, const float *b, size_t d) {
  float s = 0.0f;
  for (size_t j = 0; j < d; ++j) {
    float diff = a[j] - b[j];
    s += diff * diff;
  }
  return s;
}

struct Cand {
  uint32_t key;  // total_cmp order key of the distance
  uint32_t id;
  float dist;
};

inline bool cand_less(const Cand &a, const Cand &b) {
  return a.key != b.key ? a.key < b.key : a.id < b.id;
}

inline Cand make_cand(uint32_t id, float dist) {
  return Cand{or_total_order_key(dist), id, dist};
}

// search.rs:64-75 (finish_top_k_by_distance): select k smallest, sort.
void finish_top_k(std::vector<Cand> &c, size_t k) {
  if (k == 0 || c.empty()) {
    c.clear();
    return;
  }
  if (c.size() > k) {
    std::nth_element(c.begin(), c.begin() + (k - 1), c.end(), cand_less);
    c.resize(k);
  }
  std::sort(c.begin(), c.end(), cand_less);
}

template <class F>
void parallel_for(size_t n, int threads, F &&fn) {
  if (threads <= 1 || n < 2) {
    for (size_t i = 0; i < n; ++i) fn(i);
    return;
  }
  size_t t = std::min<size_t>(static_cast<size_t>(threads), n);
  std::vector<std::thread> pool;
  pool.reserve(t);
  for (size_t w = 0; w < t; ++w) {
    pool.emplace_back([&, w]() {
      for (size_t i = w; i < n; i += t) fn(i);
    });
  }
  for (auto &th : pool) th.join();
}

}  // namespace

extern "C" {

uint32_t or_total_order_key(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// search.rs:55-62: norm = sqrt(sum x*x); divide when norm > 1e-10.
void or_normalize(const float *x, size_t n, size_t d, float *out) {
  for (size_t i = 0; i < n; ++i) {
    const float *row = x + i * d;
    float *o = out + i * d;
    float s = 0.0f;
    for (size_t j = 0; j < d; ++j) s += row[j] * row[j];
    float norm = std::sqrt(s);
    if (norm > 1e-10f) {
      for (size_t j = 0; j < d; ++j) o[j] = row[j] / norm;
    } else {
      for (size_t j = 0; j < d; ++j) o[j] = row[j];
    }
  }
}

// pq.rs:196-267.  The three branches (dsub == 1, dsub <= 8, general) compute
// the same sequential sum; they are kept separate to mirror the reference.
int or_adc_table(const float *q, size_t d, size_t M, size_t ks,
                 const float *cb, float *table) {
  if (M == 0 || d % M != 0) return -1;
  size_t dsub = d / M;
  if (dsub == 1) {  // pq.rs:210-229
    for (size_t m = 0; m < M; ++m)
      for (size_t c = 0; c < ks; ++c) {
        float diff = q[m] - cb[m * ks + c];
        table[m * ks + c] = diff * diff;
      }
    return 0;
  }
  if (dsub <= 8) {  // pq.rs:232-251
    for (size_t m = 0; m < M; ++m) {
      const float *qs = q + m * dsub;
      for (size_t c = 0; c < ks; ++c) {
        const float *cw = cb + (m * ks + c) * dsub;
        float dist = 0.0f;
        for (size_t j = 0; j < dsub; ++j) {
          float diff = qs[j] - cw[j];
          dist += diff * diff;
        }
        table[m * ks + c] = dist;
      }
    }
    return 0;
  }
  for (size_t m = 0; m < M; ++m)  // pq.rs:253-265
    for (size_t c = 0; c < ks; ++c)
      table[m * ks + c] = l2sq_seq(q + m * dsub, cb + (m * ks + c) * dsub, dsub);
  return 0;
}

// pq.rs:272-279.
float or_distance_with_table(const float *table, size_t M, size_t ks,
                             const uint8_t *codes) {
  float total = 0.0f;
  for (size_t m = 0; m < M; ++m) total += table[m * ks + codes[m]];
  return total;
}

// pq_simd.rs:314-369: the 256-entry kernel sums four candidates at a time and
// the generic kernel one at a time; both add each candidate's codebooks in
// order starting from 0.0, which is the per-row sum below.
void or_adc_batch(const uint8_t *codes, size_t n, size_t M, const float *lut,
                  size_t ks, float *out) {
  for (size_t i = 0; i < n; ++i)
    out[i] = or_distance_with_table(lut, M, ks, codes + i * M);
}

// pq.rs:136-160: per subspace, the first codeword with the strictly smallest
// squared L2 distance wins.
void or_pq_quantize(const float *x, size_t n, size_t d, size_t M, size_t ks,
                    const float *cb, uint8_t *codes) {
  size_t dsub = d / M;
  for (size_t i = 0; i < n; ++i) {
    const float *v = x + i * d;
    for (size_t m = 0; m < M; ++m) {
      uint8_t best = 0;
      float best_dist = std::numeric_limits<float>::infinity();
      for (size_t c = 0; c < ks; ++c) {
        float dist = l2sq_seq(v + m * dsub, cb + (m * ks + c) * dsub, dsub);
        if (dist < best_dist) {
          best_dist = dist;
          best = static_cast<uint8_t>(std::min<size_t>(c, 255));
        }
      }
      codes[i * M + m] = best;
    }
  }
}

// pq.rs:284-290.
void or_pq_reconstruct(const uint8_t *codes, size_t d, size_t M, size_t ks,
                       const float *cb, float *out) {
  size_t dsub = d / M;
  for (size_t m = 0; m < M; ++m)
    std::memcpy(out + m * dsub, cb + (m * ks + codes[m]) * dsub,
                dsub * sizeof(float));
}

// pq_simd.rs:426-486: 32-vector blocks; byte m*16+lane holds vector lane in
// the low nibble and vector lane+16 in the high nibble; padding codes are 0.
void or_pack_4bit(const uint8_t *codes, size_t n, size_t M, uint8_t *out) {
  size_t blocks = (n + 31) / 32;
  size_t bpb = M * 16;
  std::memset(out, 0, blocks * bpb);
  for (size_t b = 0; b < blocks; ++b) {
    size_t base = b * 32;
    for (size_t m = 0; m < M; ++m)
      for (size_t lane = 0; lane < 16; ++lane) {
        size_t lo = base + lane, hi = base + 16 + lane;
        uint8_t clo = lo < n ? (codes[lo * M + m] & 0x0F) : 0;
        uint8_t chi = hi < n ? (codes[hi * M + m] & 0x0F) : 0;
        out[b * bpb + m * 16 + lane] = static_cast<uint8_t>(clo | (chi << 4));
      }
  }
}

// pq_simd.rs:576-611.
void or_quantize_lut_flat(const float *lut, size_t M, uint8_t *q, float *scale,
                          float *offset) {
  size_t len = M * 16;
  if (len == 0) {
    *scale = 1.0f;
    *offset = 0.0f;
    return;
  }
  float gmin = std::numeric_limits<float>::infinity();
  float gmax = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < len; ++i) {
    if (lut[i] < gmin) gmin = lut[i];
    if (lut[i] > gmax) gmax = lut[i];
  }
  float range = gmax - gmin;
  const float eps = std::numeric_limits<float>::epsilon();
  float sc, off = gmin, inv;
  if (range < eps) {
    sc = 1.0f;
    inv = 0.0f;
  } else {
    sc = range / 255.0f;
    inv = 255.0f / range;
  }
  for (size_t i = 0; i < len; ++i) {
    // (v - offset) * inv_scale, .round() (half away from zero), clamp; a NaN
    // converts to 0 like Rust's saturating `as u8`.
    float v = std::round((lut[i] - off) * inv);
    if (std::isnan(v)) {
      q[i] = 0;
    } else {
      v = std::min(std::max(v, 0.0f), 255.0f);
      q[i] = static_cast<uint8_t>(v);
    }
  }
  *scale = sc;
  *offset = off;
}

// pq_simd.rs:629-654.
void or_fastscan_block(const uint8_t *block, const uint8_t *lut_q, size_t M,
                       uint16_t *out32) {
  for (int i = 0; i < 32; ++i) out32[i] = 0;
  for (size_t m = 0; m < M; ++m)
    for (size_t lane = 0; lane < 16; ++lane) {
      uint8_t byte = block[m * 16 + lane];
      out32[lane] = static_cast<uint16_t>(out32[lane] + lut_q[m * 16 + (byte & 0x0F)]);
      out32[lane + 16] =
          static_cast<uint16_t>(out32[lane + 16] + lut_q[m * 16 + (byte >> 4)]);
    }
}

// pq_simd.rs:716-769: distance = (sum as f32) * scale + offset * M, each
// operation rounded separately.
int or_fastscan_batch_flat(const uint8_t *packed, size_t n, size_t M,
                           const float *lut, float *out) {
  if (M > kFastscanMaxCodebooks) return -1;
  std::vector<uint8_t> q(M * 16);
  float scale, offset;
  or_quantize_lut_flat(lut, M, q.data(), &scale, &offset);
  float base_offset = offset * static_cast<float>(M);
  size_t blocks = (n + 31) / 32;
  uint16_t acc[32];
  for (size_t b = 0; b < blocks; ++b) {
    or_fastscan_block(packed + b * M * 16, q.data(), M, acc);
    size_t in_block = std::min<size_t>(32, n - b * 32);
    for (size_t i = 0; i < in_block; ++i) {
      float a = static_cast<float>(acc[i]) * scale;
      out[b * 32 + i] = a + base_offset;
    }
  }
  return 0;
}

size_t or_find_nearest_centroids(const float *q, size_t d, const float *cents,
                                 size_t L, size_t nprobe, uint32_t *ids,
                                 float *dists) {
  std::vector<Cand> c(L);
  for (size_t i = 0; i < L; ++i)
    c[i] = make_cand(static_cast<uint32_t>(i), 1.0f - dot_seq(q, cents + i * d, d));
  size_t p = std::min(nprobe, L);
  if (p == 0) return 0;
  if (p < L) {
    std::nth_element(c.begin(), c.begin() + p, c.end(), cand_less);
    c.resize(p);
  }
  std::sort(c.begin(), c.end(), cand_less);
  for (size_t i = 0; i < p; ++i) {
    ids[i] = c[i].id;
    dists[i] = c[i].dist;
  }
  return p;
}

size_t or_finish_top_k(const uint32_t *ids, const float *dists, size_t n,
                       size_t k, uint32_t *out_ids, float *out_dists) {
  std::vector<Cand> c(n);
  for (size_t i = 0; i < n; ++i) c[i] = make_cand(ids[i], dists[i]);
  finish_top_k(c, k);
  for (size_t i = 0; i < c.size(); ++i) {
    out_ids[i] = c[i].id;
    out_dists[i] = c[i].dist;
  }
  return c.size();
}

void or_assign(const float *xn, size_t n, size_t d, const float *cents,
               size_t L, uint32_t *out) {
  for (size_t i = 0; i < n; ++i) {
    const float *v = xn + i * d;
    uint32_t best = 0;
    uint32_t best_key = 0xFFFFFFFFu;
    for (size_t c = 0; c < L; ++c) {
      uint32_t key = or_total_order_key(1.0f - dot_seq(v, cents + c * d, d));
      if (key < best_key) {
        best_key = key;
        best = static_cast<uint32_t>(c);
      }
    }
    out[i] = best;
  }
}

void or_flat_search_ip(const float *db, size_t n, const float *queries,
                       size_t nq, size_t d, size_t k, int threads,
                       uint32_t *out_ids, float *out_dists,
                       uint32_t *out_count) {
  parallel_for(nq, threads, [&](size_t qi) {
    const float *q = queries + qi * d;
    std::vector<Cand> c(n);
    for (size_t i = 0; i < n; ++i)
      c[i] = make_cand(static_cast<uint32_t>(i), -dot_seq(q, db + i * d, d));
    finish_top_k(c, k);
    for (size_t j = 0; j < k; ++j) {
      out_ids[qi * k + j] = j < c.size() ? c[j].id : 0xFFFFFFFFu;
      out_dists[qi * k + j] =
          j < c.size() ? c[j].dist : std::numeric_limits<float>::infinity();
    }
    out_count[qi] = static_cast<uint32_t>(c.size());
  });
}

}  // extern "C"

// ---- index -----------------------------------------------------------------

struct or_index {
  size_t d, L, M, ks, dsub, nprobe;
  bool trained = false, built = false;
  std::vector<float> centroids;  // [L][d]
  std::vector<float> codebooks;  // [M][ks][dsub]
  std::vector<uint32_t> doc_ids;
  std::vector<float> vectors;  // normalised [n][d]
  std::vector<uint32_t> assign;
  std::vector<uint8_t> codes;  // [n][M], vector order
  std::vector<std::vector<uint32_t>> lists;
  std::vector<std::vector<uint8_t>> adc_codes;  // list order, |l| >= 16
  std::vector<std::vector<uint8_t>> packed;     // 4-bit blocks, |l| >= 16
  std::vector<float> rotation;  // OPQ rotation [d][d] row-major (empty: plain PQ)
  std::vector<uint8_t> category;   // filter category per vector (255: none)
  std::vector<uint64_t> bitmask;   // filter categories per list (at build)
};

namespace {

// opq.rs:181-192 (matrix_vector_multiply): out = R v, every row summed from
// 0.0 in column order.
void rotate(const float *r, const float *v, size_t d, float *out) {
  for (size_t i = 0; i < d; ++i) {
    float s = 0.0f;
    for (size_t j = 0; j < d; ++j) s += r[i * d + j] * v[j];
    out[i] = s;
  }
}

// opq.rs:194-205 (transpose_matrix_vector_multiply): out = R^T v.
void rotate_t(const float *r, const float *v, size_t d, float *out) {
  for (size_t i = 0; i < d; ++i) {
    float s = 0.0f;
    for (size_t j = 0; j < d; ++j) s += r[j * d + i] * v[j];
    out[i] = s;
  }
}

// search.rs:623-718 (lists in vector order) and 816-848 (build_scan_caches).
void build_lists(or_index *ix) {
  size_t n = ix->doc_ids.size();
  ix->lists.assign(ix->L, {});
  for (size_t i = 0; i < n; ++i) ix->lists[ix->assign[i]].push_back(static_cast<uint32_t>(i));
  ix->adc_codes.assign(ix->L, {});
  ix->packed.assign(ix->L, {});
  for (size_t l = 0; l < ix->L; ++l) {
    const auto &ids = ix->lists[l];
    if (ids.size() < kSimdBatchThreshold) continue;
    std::vector<uint8_t> batch(ids.size() * ix->M);
    for (size_t i = 0; i < ids.size(); ++i)
      std::memcpy(&batch[i * ix->M], &ix->codes[ids[i] * ix->M], ix->M);
    if (ix->ks == 16) {
      ix->packed[l].resize(((ids.size() + 31) / 32) * ix->M * 16);
      or_pack_4bit(batch.data(), ids.size(), ix->M, ix->packed[l].data());
    } else {
      ix->adc_codes[l] = std::move(batch);
    }
  }
  ix->built = true;
}

// search.rs:1175-1391 for one normalised query; returns (internal id, dist).
void search_one(const or_index *ix, const float *qn, size_t k, size_t nprobe,
                std::vector<Cand> &out) {
  out.clear();
  size_t p = std::min(nprobe, ix->L);
  std::vector<uint32_t> pid(p);
  std::vector<float> pdist(p);
  p = or_find_nearest_centroids(qn, ix->d, ix->centroids.data(), ix->L, p,
                                pid.data(), pdist.data());
  std::vector<float> qres(ix->d), qrot(ix->d), table(ix->M * ix->ks), dist;
  for (size_t pi = 0; pi < p; ++pi) {
    uint32_t l = pid[pi];
    const auto &ids = ix->lists[l];
    const float *c = &ix->centroids[static_cast<size_t>(l) * ix->d];
    for (size_t j = 0; j < ix->d; ++j) qres[j] = qn[j] - c[j];  // 1239-1245
    const float *tq = qres.data();
    if (!ix->rotation.empty()) {  // opq.rs:115-121: table of the rotated residual
      rotate(ix->rotation.data(), qres.data(), ix->d, qrot.data());
      tq = qrot.data();
    }
    or_adc_table(tq, ix->d, ix->M, ix->ks, ix->codebooks.data(), table.data());
    if (ids.size() >= kSimdBatchThreshold) {
      dist.resize(ids.size());
      if (ix->ks == 16) {  // 1277-1316 (FastScan over prepacked blocks)
        or_fastscan_batch_flat(ix->packed[l].data(), ids.size(), ix->M,
                               table.data(), dist.data());
      } else {  // 1318-1347
        or_adc_batch(ix->adc_codes[l].data(), ids.size(), ix->M, table.data(),
                     ix->ks, dist.data());
      }
      for (size_t i = 0; i < ids.size(); ++i) out.push_back(make_cand(ids[i], dist[i]));
    } else {  // 1355-1375 (scalar path)
      for (uint32_t id : ids)
        out.push_back(make_cand(
            id, or_distance_with_table(table.data(), ix->M, ix->ks, &ix->codes[id * ix->M])));
    }
  }
  finish_top_k(out, k);
}

// search.rs:1407-1549 (search_with_filter) for one normalised query.
void search_filtered_one(const or_index *ix, const float *qn, size_t k, int want,
                         std::vector<Cand> &out) {
  out.clear();
  const uint64_t bit = uint64_t(1) << want;
  size_t p = std::min(ix->nprobe, ix->L);
  std::vector<uint32_t> order(p);
  std::vector<float> pdist(p);
  p = or_find_nearest_centroids(qn, ix->d, ix->centroids.data(), ix->L, p, order.data(), pdist.data());
  order.resize(p);
  std::vector<bool> scanned(ix->L, false);
  std::vector<float> qres(ix->d), qrot(ix->d), table(ix->M * ix->ks);
  for (;;) {
    for (uint32_t l : order) {
      if (scanned[l]) continue;
      scanned[l] = true;
      if ((ix->bitmask[l] & bit) == 0) continue;  // 1502-1505
      const float *c = &ix->centroids[static_cast<size_t>(l) * ix->d];
      for (size_t j = 0; j < ix->d; ++j) qres[j] = qn[j] - c[j];
      const float *tq = qres.data();
      if (!ix->rotation.empty()) {
        rotate(ix->rotation.data(), qres.data(), ix->d, qrot.data());
        tq = qrot.data();
      }
      or_adc_table(tq, ix->d, ix->M, ix->ks, ix->codebooks.data(), table.data());
      for (uint32_t id : ix->lists[l])  // 1512-1530: matching documents, float table
        if (ix->category[id] == static_cast<uint8_t>(want))
          out.push_back(make_cand(
              id, or_distance_with_table(table.data(), ix->M, ix->ks, &ix->codes[id * ix->M])));
    }
    if (out.size() >= k || order.size() == ix->L) break;  // 1539-1546: widen once
    order.resize(ix->L);
    for (size_t l = 0; l < ix->L; ++l) order[l] = static_cast<uint32_t>(l);
  }
  finish_top_k(out, k);
}

void write_row(const or_index *ix, const std::vector<Cand> &res, size_t k,
               size_t row, uint32_t *out_ids, float *out_dists,
               uint32_t *out_count) {
  for (size_t j = 0; j < k; ++j) {
    if (j < res.size()) {
      out_ids[row * k + j] = ix->doc_ids[res[j].id];
      out_dists[row * k + j] = res[j].dist;
    } else {  // python.rs:778-779 padding
      out_ids[row * k + j] = 0xFFFFFFFFu;
      out_dists[row * k + j] = std::numeric_limits<float>::infinity();
    }
  }
  out_count[row] = static_cast<uint32_t>(res.size());
}

}  // namespace

extern "C" {

or_index *or_index_new(size_t d, size_t L, size_t M, size_t ks, size_t nprobe) {
  if (d == 0 || L == 0 || M == 0 || ks == 0 || ks > 256 || d % M != 0) return nullptr;
  auto *ix = new or_index();
  ix->d = d;
  ix->L = L;
  ix->M = M;
  ix->ks = ks;
  ix->dsub = d / M;
  ix->nprobe = nprobe;
  return ix;
}

void or_index_free(or_index *ix) { delete ix; }

int or_index_set_trained(or_index *ix, const float *centroids, const float *codebooks) {
  ix->centroids.assign(centroids, centroids + ix->L * ix->d);
  ix->codebooks.assign(codebooks, codebooks + ix->M * ix->ks * ix->dsub);
  ix->trained = true;
  return 0;
}

int or_index_add(or_index *ix, const uint32_t *doc_ids, const float *x, size_t n) {
  if (ix->built) return -5;  // AlreadyBuilt
  size_t old = ix->vectors.size();
  ix->vectors.resize(old + n * ix->d);
  or_normalize(x, n, ix->d, ix->vectors.data() + old);
  ix->doc_ids.insert(ix->doc_ids.end(), doc_ids, doc_ids + n);
  return 0;
}

int or_index_finalize(or_index *ix) {
  if (!ix->trained) return -4;
  size_t n = ix->doc_ids.size();
  if (n == 0) return -1;  // EmptyIndex
  ix->assign.resize(n);
  or_assign(ix->vectors.data(), n, ix->d, ix->centroids.data(), ix->L, ix->assign.data());
  std::vector<float> residual(ix->d), rotated(ix->d);
  ix->codes.resize(n * ix->M);
  for (size_t i = 0; i < n; ++i) {  // 720-729 then 776-781
    const float *v = &ix->vectors[i * ix->d];
    const float *c = &ix->centroids[static_cast<size_t>(ix->assign[i]) * ix->d];
    for (size_t j = 0; j < ix->d; ++j) residual[j] = v[j] - c[j];
    const float *enc = residual.data();
    if (!ix->rotation.empty()) {  // opq.rs:107-113: encode the rotated residual
      rotate(ix->rotation.data(), residual.data(), ix->d, rotated.data());
      enc = rotated.data();
    }
    or_pq_quantize(enc, 1, ix->d, ix->M, ix->ks, ix->codebooks.data(), &ix->codes[i * ix->M]);
  }
  build_lists(ix);
  return 0;
}

int or_index_adopt_codes(or_index *ix, const uint32_t *assignments, const uint8_t *codes) {
  size_t n = ix->doc_ids.size();
  ix->assign.assign(assignments, assignments + n);
  ix->codes.assign(codes, codes + n * ix->M);
  for (size_t i = 0; i < n; ++i)
    if (ix->assign[i] >= ix->L) return -9;
  build_lists(ix);
  return 0;
}

// The built state without raw vectors (what IVFPQIndex keeps after compact,
// search.rs:901-904): doc ids, list assignments and codes of n vectors.
// Searches run; reranking needs the raw vectors and is not available.
int or_index_adopt_state(or_index *ix, const uint32_t *doc_ids, size_t n, const uint32_t *assignments,
                         const uint8_t *codes) {
  if (ix->built) return -5;
  if (!ix->trained) return -4;
  ix->doc_ids.assign(doc_ids, doc_ids + n);
  ix->vectors.clear();
  ix->assign.assign(assignments, assignments + n);
  ix->codes.assign(codes, codes + n * ix->M);
  for (size_t i = 0; i < n; ++i)
    if (ix->assign[i] >= ix->L) return -9;
  build_lists(ix);
  return 0;
}

void or_index_set_nprobe(or_index *ix, size_t nprobe) { ix->nprobe = nprobe; }

void or_rotate(const float *r, const float *v, size_t d, float *out) { rotate(r, v, d, out); }
void or_rotate_t(const float *r, const float *v, size_t d, float *out) { rotate_t(r, v, d, out); }

int or_index_set_filter(or_index *ix, const uint8_t *category, const uint64_t *bitmask) {
  const size_t n = ix->doc_ids.size();
  ix->category.assign(category, category + n);
  if (bitmask) {
    ix->bitmask.assign(bitmask, bitmask + ix->L);
  } else {  // search.rs:626-651: categories of each list's vectors
    if (!ix->built) return -4;
    ix->bitmask.assign(ix->L, 0);
    for (size_t i = 0; i < n; ++i)
      if (ix->category[i] < 64) ix->bitmask[ix->assign[i]] |= uint64_t(1) << ix->category[i];
  }
  return 0;
}

int or_index_search_filtered_batch(const or_index *ix, const float *queries, size_t nq, size_t k,
                                   int want, int threads, uint32_t *out_ids, float *out_dists,
                                   uint32_t *out_count) {
  if (!ix->built) return -4;
  if (want < 0 || want >= 64 || ix->category.size() != ix->doc_ids.size()) return -2;
  parallel_for(nq, threads, [&](size_t qi) {
    std::vector<float> qn(ix->d);
    or_normalize(queries + qi * ix->d, 1, ix->d, qn.data());
    std::vector<Cand> res;
    search_filtered_one(ix, qn.data(), k, want, res);
    write_row(ix, res, k, qi, out_ids, out_dists, out_count);
  });
  return 0;
}

void or_index_set_rotation(or_index *ix, const float *rotation) {
  if (rotation) ix->rotation.assign(rotation, rotation + ix->d * ix->d);
  else ix->rotation.clear();
}
size_t or_index_num_vectors(const or_index *ix) { return ix->doc_ids.size(); }

void or_index_get_assignments(const or_index *ix, uint32_t *out) {
  std::copy(ix->assign.begin(), ix->assign.end(), out);
}
void or_index_get_codes(const or_index *ix, uint8_t *out) {
  std::copy(ix->codes.begin(), ix->codes.end(), out);
}
void or_index_get_list_offsets(const or_index *ix, uint64_t *out) {
  out[0] = 0;
  for (size_t l = 0; l < ix->L; ++l) out[l + 1] = out[l] + ix->lists[l].size();
}
void or_index_get_list_ids(const or_index *ix, uint32_t *out) {
  size_t o = 0;
  for (const auto &ids : ix->lists)
    for (uint32_t id : ids) out[o++] = id;
}
void or_index_get_vectors(const or_index *ix, float *out) {
  std::copy(ix->vectors.begin(), ix->vectors.end(), out);
}

int or_index_reconstruct(const or_index *ix, size_t idx, float *out) {
  if (!ix->built || idx >= ix->doc_ids.size()) return -2;
  or_pq_reconstruct(&ix->codes[idx * ix->M], ix->d, ix->M, ix->ks, ix->codebooks.data(), out);
  if (!ix->rotation.empty()) {  // opq.rs:126-136: back to the original space
    std::vector<float> rec(out, out + ix->d);
    rotate_t(ix->rotation.data(), rec.data(), ix->d, out);
  }
  const float *c = &ix->centroids[static_cast<size_t>(ix->assign[idx]) * ix->d];
  for (size_t j = 0; j < ix->d; ++j) out[j] += c[j];
  return 0;
}

int or_index_search_batch(const or_index *ix, const float *queries, size_t nq,
                          size_t k, size_t nprobe, int threads,
                          uint32_t *out_ids, float *out_dists,
                          uint32_t *out_count) {
  if (!ix->built) return -4;
  size_t np = nprobe ? nprobe : ix->nprobe;
  parallel_for(nq, threads, [&](size_t qi) {
    std::vector<float> qn(ix->d);
    or_normalize(queries + qi * ix->d, 1, ix->d, qn.data());
    std::vector<Cand> res;
    search_one(ix, qn.data(), k, np, res);
    write_row(ix, res, k, qi, out_ids, out_dists, out_count);
  });
  return 0;
}

int or_index_search_reranked_batch(const or_index *ix, const float *queries,
                                   size_t nq, size_t k, size_t pool,
                                   size_t nprobe, int threads,
                                   uint32_t *out_ids, float *out_dists,
                                   uint32_t *out_count) {
  if (!ix->built) return -4;
  if (ix->vectors.empty()) return -6;  // Unsupported after compact
  size_t np = nprobe ? nprobe : ix->nprobe;
  size_t pl = std::max(pool, k);
  parallel_for(nq, threads, [&](size_t qi) {
    std::vector<float> qn(ix->d);
    or_normalize(queries + qi * ix->d, 1, ix->d, qn.data());
    std::vector<Cand> approx;
    search_one(ix, qn.data(), pl, np, approx);
    std::vector<Cand> exact;
    exact.reserve(approx.size());
    for (const Cand &c : approx)  // cosine_distance_normalized, distance.rs:104-109
      exact.push_back(make_cand(c.id, 1.0f - dot_seq(qn.data(), &ix->vectors[c.id * ix->d], ix->d)));
    finish_top_k(exact, k);
    write_row(ix, exact, k, qi, out_ids, out_dists, out_count);
  });
  return 0;
}

}  // extern "C"
