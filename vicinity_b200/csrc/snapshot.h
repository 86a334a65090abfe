// Host-side image of a built index in the terms of the reference's directory
// snapshot (src/ivf_pq/search.rs:945-1084, persistence.rs, manifest.rs):
// what save_to_dir writes and load_from_dir reads.  index.cu converts between
// it and the device layout; snapshot.cu converts between it and the files.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

#include "vicinity_gpu.h"

struct vg_index;

namespace vg {

struct SnapshotState {
  size_t dim = 0, num_vectors = 0, num_centroids = 0;
  vg_ivfpq_params params{};
  std::vector<float> centroids;         // [num_centroids][dim]
  std::vector<float> codebooks;         // [M][ks][dsub] (pq.rs:19-21)
  bool optimized = false;               // quantizer is Quantizer::Optimized
  std::vector<float> rotation;          // [dim][dim] row-major; empty = none
  std::vector<uint32_t> doc_ids;        // [num_vectors]
  std::vector<uint8_t> codes;           // [num_vectors][M], insertion order
  std::vector<uint64_t> list_offsets;   // [num_clusters + 1] cluster CSR
  std::vector<uint32_t> list_ids;       // cluster members, cluster by cluster
  std::vector<uint64_t> bitmasks;       // [num_clusters] filter category bits
  std::vector<float> vectors;           // [num_vectors][dim] or empty
  bool has_filter_field = false;
  std::string filter_field;
  // (doc_id, metadata object as JSON text in the reference's serde form),
  // ascending doc_id
  std::vector<std::pair<uint32_t, std::string>> metadata;
};

// Device -> host.  Fails with VG_ERR_NOT_BUILT on an unbuilt index.
int snapshot_export(const vg_index *ix, SnapshotState &st);

// Host -> device into a fresh index created with st.dim and st.params.
// Validates the state; on success the index is built.
int snapshot_adopt(vg_index *ix, SnapshotState &st);

void set_last_error(const char *msg);

// Validate one document's metadata, a JSON object in the reference's serde
// form ({"field": {"Int": 3}, "label": {"Str": "x"}}, DocumentMetadata of
// src/filtering/mod.rs), and read the category of `field`: 0..63, or -1 when
// the document has no value for it (search.rs:439-470).  On success
// `canonical` holds the object re-serialised compactly.  Returns a vg_status
// (VG_ERR_INVALID_PARAMETER with the reference's message on a bad value).
int parse_metadata(const char *json, const std::string &field, int *category, std::string *canonical);

// Validate a filter value in the same serde form ({"Int": 3}) as the
// category search_with_filter accepts (search.rs:1428-1446): 0..63.
int parse_filter_category(const char *value_json, int *category);

}  // namespace vg
