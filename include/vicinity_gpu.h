/*
 * vicinity_gpu.h -- C ABI of the B200 IVF-PQ engine.
 *
 * This is the boundary a host binding links against in place of the
 * reference's in-process Rust implementation of `vicinity::ivf_pq`
 * (vicinity 0.12.0).  Each entry point cites the reference interface it
 * replaces (paths are relative to the vicinity crate root).
 *
 * Conventions
 *   - Every function returns an int status: VG_OK (0) or a negative
 *     vg_status mirroring the reference's RetrieveError variants
 *     (src/error.rs:17-147).  vg_last_error() returns the message of the
 *     last failure on the calling thread.  Nothing throws across the ABI.
 *   - Array arguments may be host or device memory; device pointers
 *     (checked with cudaPointerGetAttributes) are used in place, host
 *     buffers are copied.  Output buffers are caller-owned.
 *   - A vg_index is externally synchronised, as the reference's callers
 *     serialise searches (src/python.rs:1081-1084).  Search calls block
 *     until their outputs are written.
 *   - Distances follow the reference: squared L2 between the L2-normalised
 *     query and the reconstruction, no square root (src/ivf_pq/mod.rs:100-110).
 */
#ifndef VICINITY_GPU_H
#define VICINITY_GPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum vg_status {
  VG_OK = 0,
  VG_ERR_EMPTY_INDEX = -1,        /* RetrieveError::EmptyIndex */
  VG_ERR_INVALID_PARAMETER = -2,  /* RetrieveError::InvalidParameter */
  VG_ERR_INVALID_CONFIG = -3,     /* RetrieveError::InvalidConfig */
  VG_ERR_NOT_BUILT = -4,          /* RetrieveError::NotBuilt */
  VG_ERR_ALREADY_BUILT = -5,      /* RetrieveError::AlreadyBuilt */
  VG_ERR_UNSUPPORTED = -6,        /* RetrieveError::Unsupported */
  VG_ERR_DIMENSION_MISMATCH = -7, /* RetrieveError::DimensionMismatch */
  VG_ERR_IO = -8,                 /* RetrieveError::Io */
  VG_ERR_FORMAT = -9,             /* RetrieveError::FormatError */
  VG_ERR_CUDA = -10,              /* device failure (no reference variant) */
  VG_ERR_NCCL = -11,              /* collective failure (no reference variant) */
  VG_ERR_OUT_OF_MEMORY = -12,     /* device allocation failed */
  VG_ERR_OTHER = -13,             /* RetrieveError::Other */
  VG_ERR_NOT_FOUND = -14          /* RetrieveError::Io of kind NotFound */
} vg_status;

/* src/ivf_pq/search.rs:286-329 (IVFPQParams). */
typedef struct vg_ivfpq_params {
  uint64_t num_clusters;  /* default 1024 */
  uint64_t nprobe;        /* default 100 */
  uint64_t num_codebooks; /* default 8 */
  uint64_t codebook_size; /* default 256, at most 256 */
  int32_t use_opq;        /* OPQ: build trains a rotation (opq.rs:65-105) */
  int32_t reserved;
  uint64_t seed;          /* default 42 */
} vg_ivfpq_params;

typedef struct vg_ivfpq_info {
  uint64_t dimension, num_vectors, num_clusters, num_centroids, nprobe;
  uint64_t num_codebooks, codebook_size, subvector_dim;
  int32_t built, trained, compacted, use_opq;
  int32_t device, shard_rank, shard_world, reserved;
  uint64_t device_bytes; /* bytes of index state resident on the device */
} vg_ivfpq_info;

/* Per-phase device timings (CUDA events on the index stream) and counters,
 * accumulated over search calls while profiling is on.  Mirrors
 * IVFPQSearchProfile (src/ivf_pq/search.rs:86-139). */
typedef struct vg_search_profile {
  double h2d_ms, normalize_ms, coarse_ms, select_ms, pairs_ms, scan_ms,
      merge_ms, collective_ms, d2h_ms, total_ms;
  uint64_t calls, queries, probed_pairs, scanned_vectors, scanned_code_bytes;
  uint64_t kernel_launches, scan_launches;
  /* lists and vectors actually scored after list pruning (filled by the
   * warp-per-query kernels; 0 where another kernel ran); probed_pairs and
   * scanned_vectors count every probed list */
  uint64_t scored_lists, scored_vectors;
  /* 4-bit warp-per-query kernel: tables built (lists past the pre-table
   * bound) and 16-code groups summed (candidates x groups before early exit);
   * seed_*: the same counters of a list-sharded search's seed pass, which the
   * fields above do not include */
  uint64_t tables_built, code_groups;
  uint64_t seed_scored_lists, seed_scored_vectors, seed_tables_built, seed_code_groups;
} vg_search_profile;

typedef struct vg_index vg_index;

/* Message of the last failed call on this thread (always NUL-terminated). */
int vg_last_error(char *buf, size_t len);

/* Engine version, e.g. "vicinity-b200 0.1.0 (sm_100a)". */
const char *vg_version(void);

/* Number of CUDA devices visible (0 when none). */
int vg_device_count(int *out);

/* No counterpart in the reference: runs, on `device`, the bounded-wait path
 * of the pipelined tensor-core kernels on its own -- a wait of at most
 * limit_us (1..1e6) microseconds on a barrier phase nothing completes, which
 * must expire and report through the device error flag.  *out_expired = 1
 * when it did; the device stays usable afterwards. */
int vg_selftest_bounded_wait(int device, uint32_t limit_us, int *out_expired);

/* src/ivf_pq/search.rs:382-413 (IVFPQIndex::new): InvalidConfig for a zero
 * dimension, codebook_size > 256, or num_codebooks not dividing dim. */
int vg_ivfpq_create(size_t dim, const vg_ivfpq_params *params, int device,
                    vg_index **out);

/* Drop (frees every device buffer the index owns). */
int vg_ivfpq_destroy(vg_index *ix);

/* src/ivf_pq/search.rs:478-512 (add / add_slice) over n rows: every row is
 * L2-normalised on insertion; AlreadyBuilt after build. */
int vg_ivfpq_add(vg_index *ix, const uint32_t *doc_ids, const float *x,
                 size_t n);

/* Adopt trained coarse centroids [num_centroids][dim] and PQ codebooks
 * [num_codebooks][codebook_size][dim/num_codebooks], so that build skips
 * training (the state src/ivf_pq/search.rs:606-775 produces before
 * encoding; also the parity hook for identical codebooks). */
int vg_ivfpq_set_trained(vg_index *ix, const float *centroids,
                         size_t num_centroids, const float *codebooks);

/* Adopt an OPQ rotation [dim][dim] row-major (OptimizedProductQuantizer's
 * `rotation`, src/ivf_pq/opq.rs:31-41) before build: residuals are rotated
 * before encoding and query residuals before every table; NULL removes it.
 * With set_trained this is the state a trained OPQ quantizer holds. */
int vg_ivfpq_set_rotation(vg_index *ix, const float *rotation);

/* src/ivf_pq/search.rs:515-787 (build, build_with_training_sample,
 * build_with_training_options): training_sample_size 0 trains on every
 * vector; kmeans_max_iter bounds both k-means stages.  Then assigns,
 * encodes residuals and lays out the inverted lists on the device. */
int vg_ivfpq_build(vg_index *ix, size_t training_sample_size,
                   size_t kmeans_max_iter);

/* src/ivf_pq/search.rs:347 (set_nprobe). */
int vg_ivfpq_set_nprobe(vg_index *ix, size_t nprobe);

/* Run the index's device work on `stream` (a cudaStream_t of the index's
 * device; NULL restores the index's own stream).  No reference counterpart:
 * the reference has no device streams. */
int vg_ivfpq_set_stream(vg_index *ix, void *stream);

/* Query rows per tile of the coarse stage of a search (the query x centroid
 * products and the probe selection run tile by tile), at most the automatic
 * size (1 GiB of f32 products); 0 restores the automatic size.  A tuning knob
 * with no reference counterpart: results do not depend on it. */
int vg_ivfpq_set_coarse_tile_rows(vg_index *ix, size_t rows);

/* src/ivf_pq/search.rs:352-379 getters, plus engine state. */
int vg_ivfpq_get_info(const vg_index *ix, vg_ivfpq_info *out);

/* src/ivf_pq/search.rs:1087-1093 (search) over nq query rows, batched as
 * src/python.rs:745-795 (batch_search): out_ids/out_dist are [nq][k] in
 * ascending distance; rows with fewer than k results are padded with id
 * 0xFFFFFFFF and +inf, and out_count[nq] (nullable) holds the real count.
 * nprobe 0 uses the index default. k at most 256. */
int vg_ivfpq_search_batch(vg_index *ix, const float *queries, size_t nq,
                          size_t k, size_t nprobe, uint32_t *out_ids,
                          float *out_dist, uint32_t *out_count);

/* src/ivf_pq/search.rs:1602-1617 (find_nearest_centroids) over nq query
 * rows, normalised first as search does (search.rs:55-66, 1202-1208): out_lists /
 * out_dist are [nq][p], p = min(nprobe (0: the index default), num
 * centroids), each row the p nearest lists by 1 - q.c ascending (ties by
 * list id), with those distances.  nprobe at most 256. */
int vg_ivfpq_nearest_lists(vg_index *ix, const float *queries, size_t nq,
                           size_t nprobe, uint32_t *out_lists, float *out_dist);

/* src/ivf_pq/search.rs:1117-1158 (search_reranked) over nq rows: the
 * candidate_pool best approximate candidates re-scored by exact cosine
 * distance 1 - dot.  k at most 256; candidate_pool at most 2^20 (above 256
 * it is selected in passes of 256 and needs an unsharded index).
 * Unsupported after compact. */
int vg_ivfpq_search_batch_reranked(vg_index *ix, const float *queries,
                                   size_t nq, size_t k, size_t candidate_pool,
                                   size_t nprobe, uint32_t *out_ids,
                                   float *out_dist, uint32_t *out_count);

/* src/ivf_pq/search.rs:414-434 (with_filtering): enable metadata filtering
 * on `field` (before build).  Builds then record, per inverted list, the
 * bitmask of the field's categories among its vectors. */
int vg_ivfpq_set_filter_field(vg_index *ix, const char *field);

/* src/ivf_pq/search.rs:436-475 (add_metadata): metadata of a document as a
 * JSON object in the reference's serde form, e.g.
 * {"category": {"Int": 3}, "label": {"Str": "x"}}; the filter field's value
 * must be an Int in 0..63.  Replaces earlier metadata of doc_id.  Unsupported
 * unless filtering is enabled. */
int vg_ivfpq_add_metadata(vg_index *ix, uint32_t doc_id, const char *metadata_json);

/* src/ivf_pq/search.rs:1407-1549 (search_with_filter) over nq rows with the
 * equality filter field == value (value_json in serde form, {"Int": 3}):
 * the nprobe nearest lists whose bitmask holds the category, then every list
 * when they hold fewer than k matching documents.  Outputs as
 * vg_ivfpq_search_batch.  Unsupported on a sharded index. */
int vg_ivfpq_search_filtered_batch(vg_index *ix, const float *queries,
                                   size_t nq, size_t k, const char *field,
                                   const char *value_json, uint32_t *out_ids,
                                   float *out_dist, uint32_t *out_count);

/* src/ivf_pq/search.rs:857-884 (reconstruct) of insertion index idx. */
int vg_ivfpq_reconstruct(const vg_index *ix, size_t idx, float *out);

/* src/ivf_pq/search.rs:901-904 (compact): drop the raw vectors. */
int vg_ivfpq_compact(vg_index *ix);

/* src/ivf_pq/search.rs:912-1015 (save_to_dir): write the index as a
 * directory snapshot in the reference's format (manifest.json, centroids.bin,
 * doc_ids.bin, codes.bin, list_offsets.bin, list_codes.bin, clusters.bin and,
 * unless compacted, raw_vectors.bin).  VG_ERR_NOT_BUILT before build. */
int vg_ivfpq_save(const vg_index *ix, const char *dir);

/* src/ivf_pq/search.rs:1034-1084 (load_from_dir): create a built index on
 * `device` from a directory snapshot.  Missing files give VG_ERR_NOT_FOUND,
 * malformed ones VG_ERR_FORMAT. */
int vg_ivfpq_load(const char *dir, int device, vg_index **out);

/* src/ivf_pq/search.rs:916-935 (save_to_generation) with
 * persistence/generation.rs:30-140 (GenerationWriter): the snapshot is
 * staged in root/generations/.staging-<id> with its component list in the
 * manifest, read back, inventoried in GENERATION.json (length and CRC-32 of
 * every file) and published under root/.PUBLISH.lock: renamed to
 * root/generations/<id>, then root/CURRENT replaced atomically.  Earlier
 * generations stay.  A concurrent publisher, or CURRENT changing meanwhile,
 * gives VG_ERR_IO. */
int vg_ivfpq_save_generation(const vg_index *ix, const char *root);

/* src/ivf_pq/search.rs:939-943 (load_from_generation): vg_ivfpq_load of the
 * directory root/CURRENT names (persistence/generation.rs:191-205). */
int vg_ivfpq_load_generation(const char *root, int device, vg_index **out);

/* persistence/generation.rs:191-205 (open_current): the path of the
 * generation root/CURRENT names, NUL-terminated into out[len]. */
int vg_generation_current(const char *root, char *out, size_t len);

/* persistence/generation.rs:285-365 (verify_generation): every file of a
 * generation directory against its GENERATION.json inventory; a missing or
 * malformed inventory, an unlisted or missing file, or a length or CRC-32
 * mismatch gives VG_ERR_FORMAT.  Host only. */
int vg_verify_generation(const char *dir);

/* Copies of index state for parity checks and persistence (host or device
 * destination, `bytes` must match):
 *   VG_EXPORT_CENTROIDS    f32 [num_centroids][dim]
 *   VG_EXPORT_CODEBOOKS    f32 [M][ks][dsub]
 *   VG_EXPORT_ASSIGNMENTS  u32 [n]       list of each insertion index
 *   VG_EXPORT_CODES        u8  [n][M]    vector order (codes.bin)
 *   VG_EXPORT_LIST_OFFSETS u64 [num_centroids+1] vector offsets
 *   VG_EXPORT_LIST_IDS     u32 [n]       insertion indices, list order
 *   VG_EXPORT_DOC_IDS      u32 [n]
 *   VG_EXPORT_VECTORS      f32 [n][dim]  normalised rows (until compact)
 *   VG_EXPORT_ROTATION     f32 [dim][dim] OPQ rotation, row-major (when set) */
enum {
  VG_EXPORT_CENTROIDS = 0,
  VG_EXPORT_CODEBOOKS = 1,
  VG_EXPORT_ASSIGNMENTS = 2,
  VG_EXPORT_CODES = 3,
  VG_EXPORT_LIST_OFFSETS = 4,
  VG_EXPORT_LIST_IDS = 5,
  VG_EXPORT_DOC_IDS = 6,
  VG_EXPORT_VECTORS = 7,
  VG_EXPORT_ROTATION = 8
};
int vg_ivfpq_export(const vg_index *ix, int what, void *dst, size_t bytes);

/* Turn per-phase profiling on (1) or off (0); reset clears the totals. */
int vg_ivfpq_set_profiling(vg_index *ix, int on);
int vg_ivfpq_get_profile(const vg_index *ix, vg_search_profile *out);
int vg_ivfpq_reset_profile(vg_index *ix);

/* ---- multi-GPU: inverted lists sharded by list across ranks ----------- */

/* A 128-byte NCCL unique id for a new communicator (call on one rank and
 * distribute the bytes to the others). */
int vg_nccl_unique_id(uint8_t out[128]);

/* Make a built index one shard of a world_size-rank group: lists are
 * assigned to ranks by greedy size-balanced packing (largest list first),
 * the rank scans only its lists, and each search merges the per-rank
 * top-k with one all-gather.  Every rank must hold the same built index
 * and call every search with the same queries. */
int vg_ivfpq_shard(vg_index *ix, int rank, int world_size,
                   const uint8_t nccl_id[128], int timeout_ms);

/* The list owner map used by vg_ivfpq_shard (host-only; no device work):
 * owner[l] in [0, world_size) for list sizes sizes[0..num_lists). */
int vg_shard_assign_lists(const uint64_t *sizes, size_t num_lists,
                          int world_size, int32_t *owner);

/* ---- exact flat search ------------------------------------------------ */

/* Exhaustive inner-product search (src/distance.rs:125-130, distance -dot,
 * ascending, ties to the lower row; the exhaustive ground truth of
 * src/benchmark/evaluation.rs:250-268): out_ids/out_dist [nq][k] padded
 * like vg_ivfpq_search_batch. Runs on `device`. k at most 256. */
int vg_flat_search_ip(const float *db, size_t n, const float *queries,
                      size_t nq, size_t dim, size_t k, int device,
                      uint32_t *out_ids, float *out_dist, uint32_t *out_count);

/* An exhaustive inner-product index over n rows of `dim` floats: the same
 * search as vg_flat_search_ip, with the rows' device state (the caller's
 * device rows in place -- they must outlive the index -- or a device copy of
 * host rows, plus a binary16 image for the tensor-core products and, from
 * 8,192 rows, a copy of every 4th 128-row tile of that image: about 2.5 n kp
 * bytes with kp = 64 or 128 the padded row length) built once.  Searches of
 * large databases take the queries in row tiles to keep their per-call
 * workspace near 1 GiB.
 * The reference computes this ground truth with a loop over the rows
 * (src/benchmark/evaluation.rs:250-268, src/distance.rs:125-130).
 */
typedef struct vg_flat vg_flat;
int vg_flat_create(const float *db, size_t n, size_t dim, int device, vg_flat **out);
int vg_flat_destroy(vg_flat *f);

/* vg_flat_search_ip over the rows of f: queries and outputs host or device
 * memory; the work runs on `stream` (a cudaStream_t of f's device, NULL = f's
 * own stream) and the call returns when the outputs are written.  k at most
 * 256. */
int vg_flat_search(vg_flat *f, const float *queries, size_t nq, size_t k, void *stream, uint32_t *out_ids,
                   float *out_dist, uint32_t *out_count);

/* Profiling of vg_flat_search calls (on: 1; clears the totals): device time
 * of the query image (normalize_ms), the tensor-core window kernel (scan_ms)
 * and the exact re-score (merge_ms), from CUDA events on the search stream. */
int vg_flat_set_profiling(vg_flat *f, int on);
int vg_flat_get_profile(const vg_flat *f, vg_search_profile *out);

/* No counterpart in the reference.  vg_flat_search_ip for callers that
 * cannot allocate device memory at search time (memory handed out up front
 * to another allocator or budget, loops that cannot take cudaMalloc's
 * synchronisation, embedders that forbid allocation after start-up).  Same
 * results; allocates nothing.  All pointers must be device memory of
 * `device`; work runs on `stream` (a cudaStream_t, NULL = legacy default
 * stream) and the call returns once it is done.  Scratch is one fixed
 * 32 MiB device array per GPU, shared by every call: requests whose scratch
 * would exceed it (nq > 32768, or nq * k * tiles too large) return
 * VG_ERR_INVALID_PARAMETER -- split the batch.  The first call on a device
 * resolves the array's address (cudaGetSymbolAddress) and caches it.  Every
 * call, failed ones included, returns only after its GPU work on the
 * scratch is done.  Calls whose GPU work overlaps race on the scratch and
 * must be serialised by the caller. */
int vg_flat_search_ip_noalloc(const float *db, size_t n, const float *queries,
                              size_t nq, size_t dim, size_t k, int device,
                              void *stream, uint32_t *out_ids, float *out_dist,
                              uint32_t *out_count);

#ifdef __cplusplus
}
#endif

#endif /* VICINITY_GPU_H */
