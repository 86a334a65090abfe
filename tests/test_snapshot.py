"""Directory snapshots in the reference's format (save_to_dir / load_from_dir,
src/ivf_pq/search.rs:945-1084; python.rs:654-681 for the Python errors).

CPU tests cover every failure the loader reports before it needs a device;
GPU tests cover save -> read back (with the independent Python restatement in
oracle/snapshot.py), save -> load -> identical search, and snapshots written
by that restatement from an oracle index -> search identical to the oracle.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

import oracle as orc
from oracle import snapshot as osnap
from vicinity_b200 import IVFPQIndex
from vicinity_b200.synthetic import mixture

D, L, M, KS = 32, 16, 8, 256


def _tiny_parts(n=40, seed=0):
    g = np.random.default_rng(seed)
    cent = g.standard_normal((L, D)).astype(np.float32)
    cb = g.standard_normal((M, KS, D // M)).astype(np.float32)
    assign = g.integers(0, L, n)
    lists = [np.nonzero(assign == l)[0].astype(np.uint32) for l in range(L)]
    return dict(
        dim=D,
        params=dict(num_clusters=L, nprobe=4, num_codebooks=M, codebook_size=KS, use_opq=False, seed=42),
        centroids=cent, codebooks=cb, doc_ids=np.arange(n, dtype=np.uint32) + 100,
        codes=g.integers(0, KS, (n, M)).astype(np.uint8), lists=lists,
        vectors=g.standard_normal((n, D)).astype(np.float32),
    )


def _write(tmp_path, **over):
    parts = _tiny_parts()
    parts.update(over)
    path = tmp_path / "snap"
    osnap.write_snapshot(path, **parts)
    return path


# ---- CPU: errors the loader reports before touching a device ---------------

def test_missing_snapshot_raises_file_not_found(tmp_path):
    with pytest.raises(FileNotFoundError):
        IVFPQIndex.load(tmp_path / "missing")


def test_corrupt_manifest_raises_runtime_error(tmp_path):
    path = tmp_path / "ivfpq"
    path.mkdir()
    (path / "manifest.json").write_text("not valid JSON", encoding="utf-8")
    with pytest.raises(RuntimeError):
        IVFPQIndex.load(path)


@pytest.mark.parametrize("field,value,match", [
    ("version", 2, "unsupported IVF-PQ format version 2"),
    ("dimension", 0, "zero dimension"),
    ("num_vectors", 0, "zero vectors"),
    ("num_centroids", 0, "zero centroids"),
])
def test_manifest_validation(tmp_path, field, value, match):
    path = _write(tmp_path)
    man = json.loads((path / "manifest.json").read_text())
    man[field] = value
    (path / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(RuntimeError, match=match):
        IVFPQIndex.load(path)


def test_missing_component_raises_file_not_found(tmp_path):
    path = _write(tmp_path)
    (path / "doc_ids.bin").unlink()
    with pytest.raises(FileNotFoundError):
        IVFPQIndex.load(path)


def test_component_size_mismatch(tmp_path):
    path = _write(tmp_path)
    (path / "codes.bin").write_bytes((path / "codes.bin").read_bytes()[:-1])
    with pytest.raises(RuntimeError, match="size mismatch"):
        IVFPQIndex.load(path)


@pytest.mark.parametrize("corrupt,match", [
    (lambda b: b"XXXXXXXX" + b[8:], "magic"),
    (lambda b: b + b"\0", "trailing bytes"),
    (lambda b: b[:-2], "truncated"),
])
def test_cluster_file_checks(tmp_path, corrupt, match):
    path = _write(tmp_path)
    (path / "clusters.bin").write_bytes(corrupt((path / "clusters.bin").read_bytes()))
    with pytest.raises(RuntimeError, match=match):
        IVFPQIndex.load(path)


def test_cluster_id_beyond_vector_count(tmp_path):
    parts = _tiny_parts()
    path = _write(tmp_path)
    lists = list(parts["lists"])
    lists[3] = np.append(lists[3], np.uint32(9999))
    with open(path / "clusters.bin", "wb") as f:  # persistence.rs:51-69 layout
        f.write(osnap.CLUSTER_MAGIC + np.uint64(L).tobytes())
        for ids in lists:
            f.write(np.uint64(0).tobytes() + np.uint64(ids.size).tobytes() + ids.astype("<u4").tobytes())
    with pytest.raises(RuntimeError, match="exceeds vector count"):
        IVFPQIndex.load(path)


def test_filter_metadata_without_field(tmp_path):
    path = _write(tmp_path, filter_metadata=[(100, {"category": {"Int": 3}})])
    with pytest.raises(RuntimeError, match="without filter_field"):
        IVFPQIndex.load(path)


# ---- GPU --------------------------------------------------------------------

def _engine(x, ks=KS, m=M, l=L, d=D, nprobe=6):
    ix = IVFPQIndex(d, num_clusters=l, num_codebooks=m, codebook_size=ks, nprobe=nprobe, seed=5)
    ix.add_items(x)
    ix.build(training_sample_size=None, kmeans_max_iter=5)
    return ix


@pytest.mark.gpu
@pytest.mark.parametrize("ks", [256, 16])
def test_save_then_read_back_with_the_reference_format(tmp_path, ks):
    x, q = mixture(3000, D, 20, 0.2, seed=1, nq=50)
    ix = _engine(x, ks=ks)
    ix.save(tmp_path / "snap")
    got = osnap.read_snapshot(tmp_path / "snap")
    man = got["manifest"]
    assert man["num_vectors"] == 3000 and man["dimension"] == D and man["raw_vectors_present"]
    assert man["params"]["codebook_size"] == ks and man["params"]["num_clusters"] == L
    assert set(man["quantizer"]) == {"Product"}
    assert np.array_equal(got["centroids"], ix.centroids())
    assert np.array_equal(got["codebooks"].reshape(ix.codebooks().shape), ix.codebooks())
    assert np.array_equal(got["codes"], ix.codes())
    assert np.array_equal(got["vectors"], ix.vectors())
    offs = ix.list_offsets()
    lids = ix.list_ids()
    for l in range(L):
        assert np.array_equal(got["lists"][l], lids[offs[l]:offs[l + 1]])
    # list_codes.bin: codes of the lists, list by list; offsets in bytes
    assert np.array_equal(got["list_offsets"], np.append(offs, [offs[-1]] * (L + 1 - offs.size)) * M)
    assert np.array_equal(got["list_codes"].reshape(-1, M), ix.codes()[lids])


@pytest.mark.gpu
@pytest.mark.parametrize("ks", [256, 16])
def test_save_load_round_trip_searches_identically(tmp_path, ks):
    x, q = mixture(3000, D, 20, 0.2, seed=2, nq=60)
    ix = _engine(x, ks=ks)
    ix.save(tmp_path / "snap")
    loaded = IVFPQIndex.load(tmp_path / "snap")
    assert len(loaded) == len(ix) and loaded.dimension == ix.dimension and loaded.nprobe == ix.nprobe
    for rerank in (0, 40):
        a_ids, a_d = ix.batch_search(q, 10, rerank_pool=rerank or None)
        b_ids, b_d = loaded.batch_search(q, 10, rerank_pool=rerank or None)
        assert np.array_equal(a_ids, b_ids)
        assert np.array_equal(a_d.view(np.uint32), b_d.view(np.uint32))


@pytest.mark.gpu
def test_loaded_index_rerank_finds_the_stored_vector(tmp_path):
    # tests/test_python.py:592-604: rerank every vector of a small index
    x, _ = mixture(200, D, 10, 0.2, seed=6, nq=1)
    ix = _engine(x, ks=16, l=4)
    ix.save(tmp_path / "snap")
    loaded = IVFPQIndex.load(tmp_path / "snap")
    ids, dists = loaded.search(x[0], k=5, nprobe=8, rerank_pool=len(x))
    assert ids[0] == 0 and abs(float(dists[0])) < 1e-4


@pytest.mark.gpu
def test_oracle_written_snapshot_searches_like_the_oracle(tmp_path):
    x, q = mixture(4000, D, 25, 0.2, seed=3, nq=80)
    src = _engine(x)  # trained centroids and codebooks to share
    cent, cb = src.centroids(), src.codebooks()
    ref = orc.OracleIndex(D, cent.shape[0], M, KS, 6)
    ref.set_trained(cent, cb)
    doc = np.arange(4000, dtype=np.uint32) * 3 + 7
    ref.add(doc, x)
    ref.finalize()
    offs, lids = ref.list_offsets(), ref.list_ids()
    lists = [lids[offs[l]:offs[l + 1]] for l in range(cent.shape[0])] + [np.zeros(0, np.uint32)] * (L - cent.shape[0])
    osnap.write_snapshot(
        tmp_path / "snap", dim=D,
        params=dict(num_clusters=L, nprobe=6, num_codebooks=M, codebook_size=KS, use_opq=False, seed=5),
        centroids=cent, codebooks=cb, doc_ids=doc, codes=ref.codes(), lists=lists, vectors=ref.vectors())
    ix = IVFPQIndex.load(tmp_path / "snap")
    gi, gd = ix.batch_search(q, 10)
    ri, rd, rc = ref.search_batch(q, 10, nprobe=6)
    ri = ri.astype(np.int64)
    ri[np.arange(10)[None, :] >= rc.astype(np.int64)[:, None]] = -1
    assert np.array_equal(gi, ri)
    assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


@pytest.mark.gpu
def test_compacted_snapshot_has_no_raw_vectors(tmp_path):
    x, q = mixture(2000, D, 20, 0.2, seed=4, nq=10)
    ix = _engine(x)
    ix.compact()
    ix.save(tmp_path / "snap")
    assert not (tmp_path / "snap" / "raw_vectors.bin").exists()
    loaded = IVFPQIndex.load(tmp_path / "snap")
    a, _ = ix.batch_search(q, 5)
    b, _ = loaded.batch_search(q, 5)
    assert np.array_equal(a, b)
    with pytest.raises(ValueError):
        loaded.batch_search(q, 5, rerank_pool=20)


@pytest.mark.gpu
def test_save_before_build_is_a_value_error(tmp_path):
    ix = IVFPQIndex(8, num_clusters=8, num_codebooks=4, codebook_size=8)
    with pytest.raises(ValueError, match="is not built"):
        ix.save(tmp_path / "ivfpq")


@pytest.mark.gpu
def test_clusters_that_do_not_partition_the_vectors(tmp_path):
    parts = _tiny_parts()
    lists = parts["lists"]
    # one vector listed twice, another in no list: the count still matches
    donor = next(l for l in range(2, L) if lists[l].size)
    lists[0] = np.append(lists[0], lists[1][:1])
    lists[donor] = lists[donor][1:]
    path = tmp_path / "snap"
    osnap.write_snapshot(path, **parts)
    with pytest.raises(RuntimeError, match="more than one cluster"):
        IVFPQIndex.load(path)
