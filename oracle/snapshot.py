"""TEST INFRASTRUCTURE ONLY: a Python restatement of the reference's IVF-PQ
directory snapshot (vicinity 0.12.0), used by the tests to write snapshots
the engine must load and to read back what the engine saves.

Follows src/ivf_pq/search.rs:945-1084 (save_to_dir / load_from_dir),
src/ivf_pq/persistence.rs:9-260 (component files, cluster file, manifest
validation), src/ivf_pq/manifest.rs:4-104 (manifest fields) and
src/ivf_pq/file_storage.rs:39-72 (list_offsets / list_codes).  The manifest
is written the way serde_json serialises IVFPQManifest: externally tagged
enums ({"Product": {...}}), f32 arrays as JSON numbers.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

FORMAT_VERSION = 1  # persistence.rs:9
CLUSTER_MAGIC = b"VICIVF1\0"  # persistence.rs:10


def _pq(dim, m, ks, codebooks):
    return {
        "dimension": int(dim),
        "num_codebooks": int(m),
        "codebook_size": int(ks),
        "subvector_dim": int(dim // m),
        "codebooks": [float(v) for v in np.asarray(codebooks, np.float32).ravel()],
    }


def write_snapshot(path, *, dim, params, centroids, codebooks, doc_ids, codes, lists, bitmasks=None,
                   vectors=None, rotation=None, optimized=False, filter_field=None, filter_metadata=()):
    """Write the component files of save_to_dir.

    params: dict with num_clusters, nprobe, num_codebooks, codebook_size,
    use_opq, seed.  lists: one id array per cluster (num_clusters of them).
    filter_metadata: (doc_id, {field: {"Int": n}, ...}) pairs.
    """
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    m, ks = params["num_codebooks"], params["codebook_size"]
    codes = np.asarray(codes, np.uint8).reshape(-1, m)
    n = codes.shape[0]
    pq = _pq(dim, m, ks, codebooks)
    if optimized:
        quantizer = {"Optimized": {
            "dimension": int(dim), "num_codebooks": int(m), "codebook_size": int(ks),
            "rotation": None if rotation is None else [float(v) for v in np.asarray(rotation, np.float32).ravel()],
            "pq": pq,
        }}
    else:
        quantizer = {"Product": pq}
    manifest = {
        "version": FORMAT_VERSION,
        "dimension": int(dim),
        "num_vectors": int(n),
        "num_centroids": int(np.asarray(centroids).shape[0]),
        "raw_vectors_present": vectors is not None,
        "params": {k: (bool(v) if k == "use_opq" else int(v)) for k, v in params.items()},
        "quantizer": quantizer,
        "filter_field": filter_field,
        "filter_metadata": [{"doc_id": int(d), "metadata": md} for d, md in sorted(filter_metadata)],
    }
    (path / "manifest.json").write_text(json.dumps(manifest, indent=2))
    np.asarray(centroids, "<f4").tofile(path / "centroids.bin")
    np.asarray(doc_ids, "<u4").tofile(path / "doc_ids.bin")
    codes.tofile(path / "codes.bin")
    offsets = [0]
    list_codes = []
    for ids in lists:
        for i in ids:
            list_codes.append(codes[int(i)])
        offsets.append(len(list_codes) * m)
    np.asarray(offsets, "<u8").tofile(path / "list_offsets.bin")
    (np.stack(list_codes) if list_codes else np.zeros((0, m), np.uint8)).tofile(path / "list_codes.bin")
    bitmasks = [0] * len(lists) if bitmasks is None else bitmasks
    with open(path / "clusters.bin", "wb") as f:
        f.write(CLUSTER_MAGIC)
        f.write(np.uint64(len(lists)).tobytes())
        for ids, mask in zip(lists, bitmasks):
            ids = np.asarray(ids, "<u4")
            f.write(np.uint64(mask).tobytes())
            f.write(np.uint64(ids.size).tobytes())
            f.write(ids.tobytes())
    if vectors is not None:
        np.asarray(vectors, "<f4").tofile(path / "raw_vectors.bin")


def read_snapshot(path) -> dict:
    """Read what load_from_dir reads, with its size and format checks."""
    path = Path(path)
    man = json.loads((path / "manifest.json").read_text())
    assert man["version"] == FORMAT_VERSION
    dim, n, nc = man["dimension"], man["num_vectors"], man["num_centroids"]
    p = man["params"]
    m = p["num_codebooks"]

    def exact(name, dtype, count):
        raw = np.fromfile(path / name, dtype=dtype)
        assert raw.size == count, f"{name} size mismatch"
        return raw

    (variant, q), = man["quantizer"].items()
    pq = q["pq"] if variant == "Optimized" else q
    out = {
        "manifest": man,
        "doc_ids": exact("doc_ids.bin", "<u4", n),
        "centroids": exact("centroids.bin", "<f4", nc * dim).reshape(nc, dim),
        "codes": exact("codes.bin", np.uint8, n * m).reshape(n, m),
        "codebooks": np.asarray(pq["codebooks"], np.float32),
        "rotation": (np.asarray(q["rotation"], np.float32).reshape(dim, dim)
                     if variant == "Optimized" and q.get("rotation") is not None else None),
        "vectors": (exact("raw_vectors.bin", "<f4", n * dim).reshape(n, dim)
                    if man["raw_vectors_present"] else None),
    }
    raw = (path / "clusters.bin").read_bytes()
    assert raw[:8] == CLUSTER_MAGIC
    count = int(np.frombuffer(raw[8:16], "<u8")[0])
    assert count == p["num_clusters"]
    pos, lists, masks = 16, [], []
    for _ in range(count):
        mask, ln = np.frombuffer(raw[pos:pos + 16], "<u8")
        pos += 16
        lists.append(np.frombuffer(raw[pos:pos + 4 * int(ln)], "<u4").copy())
        masks.append(int(mask))
        pos += 4 * int(ln)
    assert pos == len(raw), "trailing bytes in cluster file"
    out["lists"], out["bitmasks"] = lists, masks
    offs = np.fromfile(path / "list_offsets.bin", "<u8")
    out["list_offsets"] = offs
    out["list_codes"] = np.fromfile(path / "list_codes.bin", np.uint8)
    return out
