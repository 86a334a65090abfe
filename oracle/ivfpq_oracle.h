/*
 * TEST INFRASTRUCTURE ONLY -- CPU restatement of the vicinity 0.12.0 IVF-PQ
 * search path (Rust crate, `src/ivf_pq/`, `src/pq_simd.rs`, `src/simd.rs`).
 *
 * This library is the parity checker for the CUDA engine and the timed CPU
 * baseline.  Only tests, the smoke check and the benchmark's CPU-baseline leg
 * may load it; the engine never calls into it.
 *
 * Arithmetic contract: every sum is a sequential f32 sum in the reference's
 * iteration order, with no fused multiply-add (built with -ffp-contract=off),
 * which is what the reference's scalar `simd::fallback` backend computes
 * (`src/simd.rs:83-127`).  Ties that the reference breaks arbitrarily
 * (unstable selects) are broken here by (distance, internal index), ordered
 * with Rust's `f32::total_cmp`.
 *
 * Pinning: the reference cannot be compiled in this environment (no Rust
 * toolchain, crates not vendored), so the restatement is pinned against the
 * reference's own known-answer tests and properties, committed as fixtures
 * under tests/golden/ and checked by tests/test_oracle.py.
 */
#ifndef VICINITY_IVFPQ_ORACLE_H
#define VICINITY_IVFPQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitives ------------------------------------------------------- */

/* search.rs:55-62 (normalize_query) and search.rs:503-508 (add_slice). */
void or_normalize(const float *x, size_t n, size_t d, float *out);

/* pq.rs:196-267 (compute_adc_table_into). Returns 0, or -1 on a bad shape. */
int or_adc_table(const float *query_residual, size_t d, size_t num_codebooks,
                 size_t codebook_size, const float *codebooks, float *table);

/* pq.rs:272-279 (distance_with_table). */
float or_distance_with_table(const float *table, size_t num_codebooks,
                             size_t codebook_size, const uint8_t *codes);

/* pq_simd.rs:314-369 (adc_batch_dispatch_into). */
void or_adc_batch(const uint8_t *codes, size_t n, size_t num_codebooks,
                  const float *lut, size_t codebook_size, float *out);

/* pq.rs:136-160 (quantize), row by row. */
void or_pq_quantize(const float *x, size_t n, size_t d, size_t num_codebooks,
                    size_t codebook_size, const float *codebooks,
                    uint8_t *codes);

/* pq.rs:284-290 (reconstruct). */
void or_pq_reconstruct(const uint8_t *codes, size_t d, size_t num_codebooks,
                       size_t codebook_size, const float *codebooks,
                       float *out);

/* pq_simd.rs:426-486 (PackedCodes4bit::pack). out has
 * ceil(n/32) * num_codebooks * 16 bytes. */
void or_pack_4bit(const uint8_t *codes, size_t n, size_t num_codebooks,
                  uint8_t *out);

/* pq_simd.rs:576-611 (quantize_lut_flat). */
void or_quantize_lut_flat(const float *lut, size_t num_codebooks, uint8_t *q,
                          float *scale, float *offset);

/* pq_simd.rs:629-654 (fastscan_block_portable): 32 u16 sums. */
void or_fastscan_block(const uint8_t *block, const uint8_t *lut_q,
                       size_t num_codebooks, uint16_t *out32);

/* pq_simd.rs:716-769 (fastscan_batch_flat). Returns -1 when num_codebooks
 * exceeds FASTSCAN_MAX_CODEBOOKS (the reference panics there). */
int or_fastscan_batch_flat(const uint8_t *packed, size_t n,
                           size_t num_codebooks, const float *lut, float *out);

/* search.rs:1602-1617 (find_nearest_centroids): ids and distances of the
 * nprobe nearest centroids by 1 - dot, ascending. Returns the count. */
size_t or_find_nearest_centroids(const float *query, size_t d,
                                 const float *centroids, size_t num_centroids,
                                 size_t nprobe, uint32_t *ids, float *dists);

/* search.rs:64-75 (finish_top_k_by_distance) over (id, distance) pairs; the
 * tie rule is (distance, id). Returns the count written. */
size_t or_finish_top_k(const uint32_t *ids, const float *dists, size_t n,
                       size_t k, uint32_t *out_ids, float *out_dists);

/* f32::total_cmp order key (unsigned compare reproduces total_cmp). */
uint32_t or_total_order_key(float x);

/* kmeans.rs:97-107 (assign_clusters): argmin over centroids of 1 - dot,
 * first index wins ties. */
void or_assign(const float *xn, size_t n, size_t d, const float *centroids,
               size_t num_centroids, uint32_t *out);

/* Exact inner-product search, distance.rs:125-130 (-dot), ascending with
 * ties by row index; benchmark/evaluation.rs:250-268 is the reference's
 * exhaustive ground truth. Runs on `threads` host threads. */
void or_flat_search_ip(const float *db, size_t n, const float *queries,
                       size_t nq, size_t d, size_t k, int threads,
                       uint32_t *out_ids, float *out_dists,
                       uint32_t *out_count);

/* ---- index ------------------------------------------------------------ */

typedef struct or_index or_index;

/* search.rs:382-413 (IVFPQIndex::new). NULL on an invalid shape. */
or_index *or_index_new(size_t d, size_t num_clusters, size_t num_codebooks,
                       size_t codebook_size, size_t nprobe);
void or_index_free(or_index *ix);

/* Adopt trained coarse centroids [num_clusters][d] and PQ codebooks
 * [M][ks][d/M] (the outputs of build's two k-means stages). */
int or_index_set_trained(or_index *ix, const float *centroids,
                         const float *codebooks);

/* search.rs:488-512 (add_slice) for n rows. */
int or_index_add(or_index *ix, const uint32_t *doc_ids, const float *x,
                 size_t n);

/* search.rs:620-787 after training: assign, lists in vector order,
 * residuals, encode, build_scan_caches (816-848). */
int or_index_finalize(or_index *ix);

/* Adopt assignments [n] and codes [n][M] computed elsewhere, then build the
 * lists and scan caches exactly as or_index_finalize does. */
int or_index_adopt_codes(or_index *ix, const uint32_t *assignments,
                         const uint8_t *codes);

/* The built state of a compacted index without raw vectors (search.rs:901-904):
 * doc ids, list assignments and codes of n vectors; searches run, reranking
 * does not. */
int or_index_adopt_state(or_index *ix, const uint32_t *doc_ids, size_t n,
                         const uint32_t *assignments, const uint8_t *codes);

void or_index_set_nprobe(or_index *ix, size_t nprobe);
/* Filter state of search.rs:1407-1549: category [n] per vector (255: none)
 * and bitmask [L] per list (NULL: computed from the categories as
 * search.rs:626-651 does at build).  Call after finalize. */
int or_index_set_filter(or_index *ix, const uint8_t *category, const uint64_t *bitmask);

/* search.rs:1407-1549 (search_with_filter) for category `want` (0..63). */
int or_index_search_filtered_batch(const or_index *ix, const float *queries, size_t nq,
                                   size_t k, int want, int threads, uint32_t *out_ids,
                                   float *out_dists, uint32_t *out_count);

/* opq.rs:181-192 (matrix_vector_multiply) and 194-205 (transpose): out = R v
 * and out = R^T v with R [d][d] row-major, each output summed from 0.0. */
void or_rotate(const float *r, const float *v, size_t d, float *out);
void or_rotate_t(const float *r, const float *v, size_t d, float *out);

/* OPQ rotation [d][d] row-major (opq.rs:31-41), applied to residuals before
 * encoding (opq.rs:107-113) and to query residuals before each table
 * (opq.rs:115-121); NULL clears it.  Set it before or_index_finalize. */
void or_index_set_rotation(or_index *ix, const float *rotation);
size_t or_index_num_vectors(const or_index *ix);

/* Export views (sizes: n, n*M, num_clusters+1, n). list_offsets counts
 * vectors, not bytes. */
void or_index_get_assignments(const or_index *ix, uint32_t *out);
void or_index_get_codes(const or_index *ix, uint8_t *out);
void or_index_get_list_offsets(const or_index *ix, uint64_t *out);
void or_index_get_list_ids(const or_index *ix, uint32_t *out);
void or_index_get_vectors(const or_index *ix, float *out);

/* search.rs:857-884 (reconstruct). */
int or_index_reconstruct(const or_index *ix, size_t idx, float *out);

/* search.rs:1087-1093 (search) mapped over rows, padded like
 * python.rs:745-795 (ids UINT32_MAX, distances +inf); out_count[i] holds the
 * number of real results. nprobe == 0 uses the index default. */
int or_index_search_batch(const or_index *ix, const float *queries, size_t nq,
                          size_t k, size_t nprobe, int threads,
                          uint32_t *out_ids, float *out_dists,
                          uint32_t *out_count);

/* search.rs:1117-1158 (search_reranked) mapped over rows. */
int or_index_search_reranked_batch(const or_index *ix, const float *queries,
                                   size_t nq, size_t k, size_t pool,
                                   size_t nprobe, int threads,
                                   uint32_t *out_ids, float *out_dists,
                                   uint32_t *out_count);

#ifdef __cplusplus
}
#endif

#endif
