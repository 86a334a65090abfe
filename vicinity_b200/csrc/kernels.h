// Host-side launchers for the engine's CUDA kernels.  Every launcher enqueues
// on the given stream and returns the launch status; none synchronises.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace vg {

// ---- search_kernels.cu ----------------------------------------------------

// out[i] = x[i] / ||x[i]|| when the norm exceeds 1e-10, else x[i]
// (search.rs:55-62, 503-508).  Sequential sum, IEEE sqrt and divide.
cudaError_t launch_normalize_rows(const float *x, size_t n, int d, float *out,
                                  cudaStream_t s);

// dist[b][c] = 1 - dot(q[b], cent[c]) with the dot summed in index order
// (search.rs:1602-1617, distance.rs:104-109).  Writes rows [0, B) of a
// row-major matrix with leading dimension ld.
cudaError_t launch_coarse_dist(const float *q, size_t B, const float *cent,
                               size_t L, int d, float *dist, size_t ld,
                               cudaStream_t s);

// best[b] = min over c of pack_key(1 - dot(q[b], cent[c]), c): the argmin
// centroid with ties to the lowest index.  best must be pre-set to ~0.
cudaError_t launch_coarse_argmin(const float *q, size_t B, const float *cent,
                                 size_t L, int d, unsigned long long *best,
                                 cudaStream_t s);

// best[b] = min over c of pack_key(-dot(q[b], db[c]), c + col_base) for the
// flat inner-product path; dist written when non-null like coarse_dist but
// with -dot.
cudaError_t launch_neg_dot(const float *q, size_t B, const float *db, size_t n,
                           int d, float *dist, size_t ld, cudaStream_t s);

// OPQ rotation of rows (opq.rs:181-192, 207-222): out[i] = R x[i] with R
// [d][d] row-major, every output summed from 0.0 in column order with
// separately rounded products.
cudaError_t launch_rotate_rows(const float *x, size_t n, int d, const float *rotation,
                               float *out, cudaStream_t s);

// Per row: the k smallest (value, column) of a row-major [rows][cols]
// matrix, ascending, ties to the lower column.  Rows with fewer than k
// columns are padded with id 0xffffffff and +inf.  k <= 256.
cudaError_t launch_select_rows(const float *dist, size_t rows, size_t cols,
                               size_t ld, int k, uint32_t *out_ids,
                               float *out_dist, size_t out_ld,
                               uint32_t col_base, cudaStream_t s);

// One probe of one query as the streaming 8-bit kernel reads it: 32 bytes,
// copied into shared memory a query at a time.
struct ProbeRec {
  uint32_t list;  // 0xffffffff: no list to scan (empty probe or list not owned)
  uint32_t len;   // vectors in the list
  uint64_t lbeg;  // list_off[list]
  uint64_t coff;  // code_off[list]
  float lb;       // distance lower bound (list pruning)
  uint32_t pad;
};

// List-pruning bounds and probe records of selected probes, written beside
// them (same row stride); lb == nullptr: none.  Same values as
// launch_probe_lb.
struct ProbeBoundArgs {
  const float *radius;
  int M, dsub;
  const uint64_t *list_off, *code_off;
  const uint8_t *owner;  // nullable: every list owned
  float *lb;
  ProbeRec *rec;         // nullable
  // 4-bit tables: a lower bound on every quantised distance of the probe,
  // known before its table is built (sub_radius[M]: the largest codeword
  // norm of any subspace); lbq == nullptr: none
  const float *sub_radius;
  float *lbq;
};

// ---- tc_select.cu: tensor-core products with a fused candidate window ----

// K padding of a binary16 operand image for row length d: 64 or 128 (0: d
// beyond 128, no tensor-core path).
int umma_kp(int d);

// Bytes of the operand image of `rows` rows: rows rounded up to 128, kp
// binary16 elements each.
size_t umma_image_bytes(size_t rows, int kp);

// Operand image of x [rows][d] (f32, rounded to nearest binary16, zero
// padded to kp columns and to whole 128-row tiles): 128-row tiles of kp/64
// blocks of 128 rows x 128 bytes in the 128-byte-swizzled K-major layout the
// tensor core reads.  With eps set, also eps[r] = rel |x_r| cmax + abs_coef
// (1 + |x_r| + cmax) + 2^-20 (rounded up; +inf for rows too long for binary16),
// the bound on |s - x_r . c| of the approximate products.
cudaError_t launch_umma_image(const float *x, size_t rows, int d, int kp, void *img, const float *cmax,
                              double rel, double abs_coef, float *eps, cudaStream_t s);

// Error coefficients of the approximate products for row length d: operand
// rounding of both sides, tensor-core accumulation (16 ulp per add), the
// exact sequential dot's own rounding and the subtractions from 1 (rel);
// subnormal binary16 operands (abs_coef).
void tc_error_coefs(int d, double *rel, double *abs_coef);

// The P best columns of every query row by exact distance (mode 0: 1 - q.x,
// the probe order of find_nearest_centroids; mode 1: -q.x, exact inner-
// product search), ascending, ties to the lower column, padded with
// 0xffffffff / +inf: out_ids / out_dist [rows][out_ld].  Products come from
// the tensor cores on the two images; columns within twice the error bound
// of the P-th approximate product are re-scored with the reference's
// sequential f32 dot from q [rows][d] and x [cols][d].  With bnd.lb set
// (mode 0), the probes' pruning bounds and records are written beside them.
struct TcSelect {
  const void *a_img;      // query image (umma_image_bytes(rows, kp))
  const float *q;         // [rows][d] f32 query rows
  size_t rows;
  const void *b_img;      // column image
  const float *x;         // [cols][d] f32 column rows
  size_t cols;
  int d, kp, P, mode;     // P in 1..256
  const float *eps;       // [rows] from launch_umma_image
  void *workspace;        // tc_select_workspace_bytes(rows, cols, P, num_sms)
  uint32_t *out_ids;
  float *out_dist;
  size_t out_ld;
  uint32_t *out_count;    // [rows] real result counts (nullable)
  ProbeBoundArgs bnd;     // bnd.lb == nullptr: no bounds
  int *error;             // set nonzero when a bounded wait of the kernel gives up
  cudaEvent_t marks[3];   // recorded (when non-null) before the window kernel, between it and the finisher, after
};
size_t tc_select_workspace_bytes(size_t rows, size_t cols, int P, int num_sms);

// The same result as launch_tc_select (mode 1 or 0, no probe bounds) for many
// columns: the product GEMM first writes the chunk maxima of a sample of the
// columns' tiles (sample_img: whole 128-column tiles of b_img, sample_cols
// columns), whose P-th largest per row bounds the row's P-th product; one
// more pass over every column gathers the columns that can reach the top P
// (a few P per row), and the finisher re-scores them exactly.
struct TcSampledSelect {
  const void *a_img;
  const float *q;
  size_t rows;
  const void *b_img;
  const float *x;
  size_t cols;
  const void *sample_img;
  size_t sample_cols;     // a multiple of 128
  int d, kp, P, mode;     // P in 1..256
  const float *eps;
  void *workspace;        // tc_sampled_workspace_bytes(rows, cols, sample_cols, P)
  uint32_t *out_ids;
  float *out_dist;
  size_t out_ld;
  uint32_t *out_count;    // nullable
  int *error;
  cudaEvent_t marks[3];   // before the sampled pass, before the finisher, after it (nullable)
};
size_t tc_sampled_workspace_bytes(size_t rows, size_t cols, size_t sample_cols, int P);
cudaError_t launch_tc_sampled_select(const TcSampledSelect &t, int num_sms, cudaStream_t s);

// out[r][c] (binary16, row stride ld) = q_r . x_c from the tensor cores
// (binary16 operand images, f32 accumulation, rounded to nearest): the
// approximate coarse products the probe shortlist ranks.  With cmax set,
// also cmax[r][j] (binary16, row stride cstride >= 4 ceil(cols / 128)) = the
// largest product of columns [32 j, 32 j + 32) of row r (-inf past cols).
// Waits on an mbarrier phase nothing completes, for at most limit_cycles SM
// cycles (at most the pipelined kernels' own limit), then sets *error = 4:
// the bounded-wait path of the tensor-core kernels, run on its own.
cudaError_t launch_bounded_wait_check(long long limit_cycles, int *error, cudaStream_t s);

cudaError_t launch_tc_gemm_f16(const void *a_img, size_t rows, const void *b_img, size_t cols, int d, int kp,
                               void *out, size_t ld, void *cmax, size_t cstride, int *error, int num_sms,
                               cudaStream_t s);

// Exact top-k probes per row from approximate products s[row][l] ~ q . c_l
// (binary16 with s_half, else f32): candidates within eps = rel |q| cmax +
// abs_coef (1 + cmax) + 2^-20 of the k-th are re-scored with the reference's
// sequential 1 - dot; rows with too many candidates or non-finite inputs are
// scored exactly over all L.  Same output as launch_select_rows on exact
// 1 - dot distances; with bounds.lb set, the probes' pruning bounds and
// records are written beside them (shortlist.cu).
// With chunk_max set (binary16 products only, row stride chunk_stride: the
// GEMM's chunk maxima), the bound comes from the chunk maxima and only chunks
// whose maximum reaches the window are read.
cudaError_t launch_probe_shortlist(const void *s, bool s_half, size_t rows, size_t L, size_t ld, const float *qn,
                                   int d, const float *cent, const float *cmax, double rel, double abs_coef, int k,
                                   uint32_t *out_ids, float *out_dist, size_t out_ld, const ProbeBoundArgs &bounds,
                                   cudaStream_t st, const void *chunk_max = nullptr, size_t chunk_stride = 0);
cudaError_t launch_tc_select(const TcSelect &t, int num_sms, cudaStream_t s);

// Same selection, but writing packed keys (for later merging).
cudaError_t launch_select_rows_keys(const float *dist, size_t rows,
                                    size_t cols, size_t ld, int k,
                                    unsigned long long *out_keys,
                                    size_t out_ld, uint32_t col_base,
                                    cudaStream_t s);

// Build the list-major pair order: probes is [B][P] list ids (0xffffffff =
// none); owner (nullable) marks lists this device scans.  Produces
// work[0..total) = pair ids (b*P + slot) grouped by list, and total in
// *d_total.  counts/cursor are [L] scratch.  When stats is non-null,
// stats[0..3) accumulates (pairs, scanned vectors, scanned code bytes) using
// list_off and the code layout (M bytes per vector, or M/2 packed for
// 4-bit lists of at least 16 vectors).
cudaError_t launch_build_pairs(const uint32_t *probes, size_t B, int P,
                               const uint8_t *owner, size_t L,
                               uint32_t *counts, uint32_t *cursor,
                               uint32_t *work, uint32_t *d_total,
                               const uint64_t *list_off, int M, bool four_bit,
                               unsigned long long *stats, cudaStream_t s);

// Profiling counters: for every valid owned probe of [B][P], adds
// (1 pair, list length, code bytes scanned) to stats[0..3).
cudaError_t launch_probe_stats(const uint32_t *probes, size_t B, int P,
                               const uint8_t *owner, size_t L,
                               const uint64_t *list_off, int M, bool four_bit,
                               unsigned long long *stats, cudaStream_t s);

// Per row r: the k smallest of keys[r][0..width) (sentinel ~0 = none);
// emits doc ids (ids_map[key id]) and distances, padded with 0xffffffff/+inf,
// the real count, and optionally the raw keys [rows][k].
cudaError_t launch_merge_keys(const unsigned long long *keys, size_t rows,
                              size_t width, size_t row_stride, int k,
                              const uint32_t *ids_map, uint32_t *out_ids,
                              float *out_dist, uint32_t *out_count,
                              unsigned long long *out_keys, cudaStream_t s);

// Merge G shard results laid out [G][rows][k] into [rows][k].
cudaError_t launch_merge_shards(const unsigned long long *keys, int G,
                                size_t rows, int k, const uint32_t *ids_map,
                                uint32_t *out_ids, float *out_dist,
                                uint32_t *out_count, unsigned long long *out_keys,
                                cudaStream_t s);

// Exact rerank of [rows][width] candidate keys (internal ids) by
// 1 - dot(qn[row], vectors[id]); emits the k best as doc ids (ids_map).
cudaError_t launch_rerank(const float *qn, const float *vectors, int d,
                          const unsigned long long *cand, size_t rows, int width,
                          int k, const uint32_t *ids_map, uint32_t *out_ids,
                          float *out_dist, uint32_t *out_count, cudaStream_t s);

// Filtered search (search.rs:1407-1549): counts[l * 64 + c] = number of
// vectors of list l (assign) with category c (< 64).  counts must be zeroed.
cudaError_t launch_category_counts(const uint8_t *category, const uint32_t *assign, size_t n,
                                   uint32_t *counts, cudaStream_t s);

// widen[q] = 1 when the lists query q probes (probes [nq][P]) that carry
// category want hold fewer than k vectors of that category: the reference
// then scans every remaining list (search.rs:1489-1547).
cudaError_t launch_filter_widen(const uint32_t *probes, size_t nq, int P, const uint64_t *bitmask,
                                const uint32_t *counts, int want, size_t k, uint8_t *widen,
                                cudaStream_t s);

// List pruning.  radius[l] = max over the list's vectors of the norm of the
// reconstructed residual (concatenated codewords), in double, rounded up to
// float (list_codes [L] lists at code_off, codebooks [M][ks][dsub]).
cudaError_t launch_list_radius(const uint8_t *list_codes, const uint64_t *code_off, const uint64_t *list_off,
                               size_t L, int M, int ks, int dsub, const float *codebooks, float *radius,
                               cudaStream_t s);

// rad[m] = the largest codeword norm of subspace m (double, rounded up);
// rad[M] = the largest of them.  rad holds M + 1 floats.
cudaError_t launch_subspace_radius(const float *codebooks, int M, int ks, int dsub, float *rad, cudaStream_t s);

// *out = the largest centroid norm (double, rounded up to float), NaN when a
// centroid holds a NaN.
cudaError_t launch_centroid_norm_max(const float *cent, size_t L, int d, float *out, cudaStream_t s);

// lb[q][p] = a lower bound on every computed ADC distance of probe p of query
// q: (||r|| - radius)^2 with r the float residual qn[q] - centroid (computed
// as the scan kernels compute it), times 1 - (M + dsub + 2) 2^-24 for the
// rounding of the table sums, rounded down; 0 when ||r|| <= radius.
// b.lb[q][p] (and, when non-null, b.lbq and b.rec) for every probe, with
// the same values the probe shortlist writes beside the probes it selects;
// b.rec[q][p].list is 0xffffffff when the probe is empty or its list not owned.
cudaError_t launch_probe_lb(const float *qn, size_t nq, int d, const uint32_t *probes, int P,
                            const float *centroids, const struct ProbeBoundArgs &b, cudaStream_t s);

// rec[i] for probes[i] (i < n): the list's record with the local layout
// (list_off, code_off) and bound lb[i] when owner marks the list, else an
// empty record (list 0xffffffff).
cudaError_t launch_probe_records(const uint32_t *probes, const float *lb, size_t n, const uint8_t *owner,
                                 const uint64_t *list_off, const uint64_t *code_off, ProbeRec *rec, cudaStream_t s);

// Work lists of a list-sharded search's two scan passes (ScanParams::work).
// Seed pass: the queries whose probe 0 is an owned list (seed_next[q] = 1 for
// the others, which the pass skips); with seed_next null, every query, heavy
// ones (long probe-0 list) first -- the order of a single-GPU scan.  Main pass: the units (query, G probes
// from first[q] on) with an owned list whose bound (lbq for 4-bit codes, lb
// for 8-bit) lies at or below the query's ceiling key.  An item whose lists
// hold at least `heavy` vectors goes to the front (count[0]), the others to
// the back (count[1], from work[cap - 1] down); count is zeroed first.
cudaError_t launch_order_seed(const uint32_t *probes, int P, const uint8_t *owner, const uint64_t *list_off,
                              size_t nq, uint32_t heavy, uint32_t *work, uint32_t *count, uint32_t cap,
                              uint32_t *seed_next, cudaStream_t s);
cudaError_t launch_order_units(const uint32_t *probes, int P, int G, const uint8_t *owner, const uint64_t *list_off,
                               const float *bound, const unsigned long long *ceiling, const uint32_t *first,
                               size_t nq, uint32_t heavy, uint32_t *work, uint32_t *count, uint32_t cap,
                               cudaStream_t s);

// dst + dst_off[i] <- bytes[i] bytes of src + src_off[i], i < count (a block
// per segment; offsets and sizes in device memory).
cudaError_t launch_copy_segments(const void *src, void *dst, const uint64_t *src_off, const uint64_t *dst_off,
                                 const uint64_t *bytes, size_t count, cudaStream_t s);

// Number of positions where a[i] != b[i] added to *changed.
cudaError_t launch_count_diff_u8(const uint8_t *a, const uint8_t *b, size_t n,
                                 unsigned int *changed, cudaStream_t s);
cudaError_t launch_count_diff_u32(const uint32_t *a, const uint32_t *b, size_t n,
                                  unsigned int *changed, cudaStream_t s);

// ---- scan_kernels.cu ------------------------------------------------------

struct ScanParams {
  const float *qn;          // [nq][d] normalised queries
  const float *centroids;   // [L][d]
  const float *codebooks;   // [M][ks][dsub]
  const uint32_t *probes;   // [nq][P] list ids, nearest first (0xffffffff = none)
  const uint8_t *owner;     // [L] nonzero for lists this device scans (nullable = all)
  uint32_t *counter;        // device scalar, zeroed before launch (query counter)
  const uint64_t *list_off; // [L+1] vector offsets into list_ids
  const uint64_t *code_off; // [L] byte offsets into list_codes (16-aligned)
  const uint8_t *list_codes;
  const uint64_t *pack_off; // [L] byte offsets into packed (4-bit only)
  const uint8_t *packed;
  const uint32_t *list_ids; // internal vector ids, list order
  const uint32_t *doc_ids;  // internal id -> caller id (for out_ids)
  int d, M, ks, dsub, P, k, nq;
  unsigned long long *out_keys;  // [nq][k] keys (nullable)
  uint32_t *out_ids;             // [nq][k] doc ids, padded 0xffffffff (nullable)
  float *out_dist;               // [nq][k] distances, padded +inf
  uint32_t *out_count;           // [nq] real result counts (nullable)
  int *error;                    // set nonzero when a bounded pipeline wait gives up
  float neg_zero;                // -0.0f; kernels take it as a run-time value (see f32x2.cuh)
  const float *rot_t;            // OPQ rotation transposed, [d][d] (nullable: plain PQ)
  // filtered search (query-major kernel only; zero-initialised = off):
  const uint32_t *qmap;          // work item -> query row (nullable: identity)
  int probes_shared;             // nonzero: every query reads probe row 0 (P entries)
  const uint8_t *category;       // [n] filter category per vector id, 255 = none (nullable: no filter)
  const uint64_t *bitmask;       // [L] categories present per list (at build)
  int want_cat;                  // category to keep, 0..63
  const float *probe_lb;         // [nq][P] distance lower bound per probe (nullable: no list pruning)
  const ProbeRec *probe_rec;     // [nq][P] probe records (streaming 8-bit kernel; nullable)
  const float *probe_lbq;        // [nq][P] bound on quantised 4-bit distances before the table (nullable)
  unsigned long long *scored;    // [4]: lists and vectors scored after pruning, tables built and 16-code
                                 // groups summed (4-bit) (nullable; warp-per-query kernels)
  // [nq] keys already selected by an earlier pass: only keys above a query's
  // floor compete (nullable; query-major and 4-bit block kernels, which serve
  // k up to 256: top-k beyond 256 in passes)
  const unsigned long long *key_floor;
  // list-sharded search (warp-per-query kernels only; zero-initialised = off):
  // seed pass (seed_next set): a query whose probe 0 is this rank's list
  // visits this rank's lists of probes 0, 1, ... and stops before the first
  // list it reaches with k keys already kept; seed_next[q] = that probe (P
  // when every probe was visited, 1 when probe 0 is another rank's: nothing
  // visited).  Main pass: probe_from[q] = the query's first probe (nullable: 0)
  uint32_t *seed_next;
  const uint32_t *probe_from;
  // work items: with unit_probes = G > 0 an item is a unit (query q, probes
  // [g G, (g + 1) G) from probe_from[q] on) whose top-k, bounded by the key
  // ceiling, goes to out_keys[((1 + g) nq + q) k ...]; otherwise an item is a
  // query.  work (nullable: every item, in order) lists the items to run:
  // work_count[0] of them from work[0] up, then work_count[1] from
  // work[work_cap - 1] down (a list built heavy items first)
  int unit_probes;
  const uint32_t *work;
  const uint32_t *work_count;
  uint32_t work_cap;
  const unsigned long long *init_keys;   // [nq][k] keys the query's top-k starts from (nullable)
  unsigned long long *out_kth;           // [nq] the query's k-th kept key (kEmptyKey: fewer than k) (nullable)
  const unsigned long long *key_ceiling; // keys above the query's ceiling are never kept (nullable) ...
  int ceiling_stride;                    // ... read at key_ceiling[q * ceiling_stride] (0: stride 1)
  int force_warp;                        // use the warp-per-query kernels at any batch size
};

// Fused per-query kernel: for each probed list the query residual, the ADC
// table in shared memory and the code scan (8-bit table sum or 4-bit
// FastScan), with the query's top-k kept on chip.
cudaError_t launch_ivfpq_scan(const ScanParams &p, int num_sms,
                              cudaStream_t s);

// The query-major kernel for any shape: the path of filtered search, whose
// probe lists, query map and filter only that kernel reads.
cudaError_t launch_ivfpq_scan_generic(const ScanParams &p, int num_sms, cudaStream_t s);

// Whether launch_ivfpq_scan with force_warp runs a warp-per-query kernel for
// p (the kernels that honour seed_next, probe_from, init_keys, out_kth and key_ceiling).
bool ivfpq_scan_warp_applies(const ScanParams &p);

// Name of the kernel variant launch_ivfpq_scan would run for p.
int ivfpq_scan_variant_name(const ScanParams &p, int num_sms, char *buf, size_t len);

// Kernel family selection (VICINITY_SCAN_KERNEL): 4 (default) = the
// warp-per-query kernels for batches of at least 16 queries per SM, else the
// query-stream (8-bit) and 4-bit block kernels; 5 = the warp-per-query
// kernels wherever they apply; 3 = never the warp-per-query kernels; 1 = the
// query-major kernel.
void set_scan_family(int family);

// ---- build_kernels.cu -----------------------------------------------------

// codes[i][m] = first argmin_c ||(x[i] - cent[assign[i]])_m - cw[m][c]||^2
// (search.rs:720-729 residuals, pq.rs:136-160 quantize).
cudaError_t launch_encode(const float *xn, size_t n, int d,
                          const uint32_t *assign, const float *cent,
                          const float *codebooks, int M, int ks,
                          uint8_t *codes, cudaStream_t s);

// Same argmin on rows that are already residuals (training).
cudaError_t launch_encode_residuals(const float *r, size_t n, int d,
                                    const float *codebooks, int M, int ks,
                                    uint8_t *codes, cudaStream_t s);

// residual[i] = x[i] - cent[assign[i]]
cudaError_t launch_residuals(const float *xn, size_t n, int d,
                             const uint32_t *assign, const float *cent,
                             float *out, cudaStream_t s);

// Unpack argmin keys into u32 assignments and count reassignments against
// prev (nullable); changed is a device counter.
cudaError_t launch_keys_to_assign(const unsigned long long *best, size_t n,
                                  uint32_t *assign, const uint32_t *prev,
                                  unsigned int *changed, cudaStream_t s);

// Gather list-ordered codes: for sorted position p (list l), copy
// codes[sorted_ids[p]] to list_codes[code_off[l] + (p - list_off[l]) * M].
cudaError_t launch_gather_list_codes(const uint8_t *codes, const uint32_t *sorted_ids,
                                     const uint32_t *sorted_lists, size_t n,
                                     int M, const uint64_t *list_off,
                                     const uint64_t *code_off, uint8_t *list_codes,
                                     cudaStream_t s);

// 4-bit scan layout of every list with at least 16 vectors (the lists the
// reference scans with quantised tables, search.rs:816-848): vector-major,
// code 2j | code 2j+1 << 4 per byte, ceil(M/2) bytes per vector, at
// pack_off[l].
cudaError_t launch_pack_lists_4bit(const uint8_t *list_codes, const uint64_t *list_off,
                                   const uint64_t *code_off, const uint64_t *pack_off,
                                   size_t L, int M, uint8_t *packed, cudaStream_t s);

// k-means update: for each cluster c with members sorted_ids[seg[c]..seg[c+1])
// (ascending), new_cent[c] = mean of rows (sequential, deterministic), then
// normalised when spherical != 0.  Empty clusters keep old_cent.
cudaError_t launch_kmeans_update(const float *x, int d, const uint32_t *sorted_ids,
                                 const uint32_t *seg, size_t k, const float *old_cent,
                                 float *new_cent, int spherical, cudaStream_t s);

// Per-subspace update for PQ codebooks: members of codeword (m, c) are the
// rows with codes[i][m] == c; x holds residual rows [n][d].
cudaError_t launch_pq_update(const float *x, size_t n, int d, int M, int ks,
                             const uint32_t *sorted_rows, const uint32_t *seg,
                             const float *old_cb, float *new_cb, cudaStream_t s);

cudaError_t launch_gather_rows(const float *x, int d, const uint32_t *rows, size_t n,
                               float *out, cudaStream_t s);

cudaError_t launch_iota(uint32_t *out, size_t n, cudaStream_t s);

// keys[row*M + m] = m*ks + codes[row][m], vals = row (PQ training segments).
cudaError_t launch_pq_keys(const uint8_t *codes, size_t n, int M, int ks,
                           uint32_t *keys, uint32_t *vals, cudaStream_t s);

// seg[c] = lower bound of c in sorted_keys, for c in [0, nseg].
cudaError_t launch_segments(const uint32_t *sorted_keys, size_t n, size_t nseg,
                            uint32_t *seg, cudaStream_t s);

// Stable LSD radix sort of (key, value) pairs on bits [0, end_bit); call
// with temp == nullptr to size temp_bytes.
cudaError_t sort_pairs_u32(void *temp, size_t &temp_bytes, const uint32_t *kin,
                           uint32_t *kout, const uint32_t *vin, uint32_t *vout,
                           size_t n, int end_bit, cudaStream_t s);

}  // namespace vg
