"""Metadata-filtered search (search_with_filter, src/ivf_pq/search.rs:1407-1549;
with_filtering / add_metadata, search.rs:414-475).

The oracle restates the reference loop (probe order, lists skipped by their
build-time category bitmask, matching documents scored with the float table,
one widening pass over every list when fewer than k matches are found); the
GPU must return exactly its results.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

import oracle as orc
from oracle import snapshot as osnap
from vicinity_b200 import IVFPQIndex
from vicinity_b200.synthetic import mixture


def _oracle(d, cent, cb, M, ks, nprobe, x, doc, cats, rotation=None, bitmask=None):
    ref = orc.OracleIndex(d, cent.shape[0], M, ks, nprobe)
    ref.set_trained(cent, cb)
    if rotation is not None:
        ref.set_rotation(rotation)
    ref.add(np.asarray(doc, np.uint32), x)
    ref.finalize()
    ref.set_filter(np.asarray(cats, np.uint8), bitmask)
    return ref


# ---- oracle (CPU) -------------------------------------------------------------

def test_oracle_widens_past_nprobe():
    # search.rs:2648-2685: nprobe = 1, three documents carry tag 0
    g = np.random.default_rng(77)
    x = g.random((240, 16), dtype=np.float32)
    cent = orc.normalize(x[g.choice(240, 8, replace=False)])
    cb = g.random((4, 16, 4), dtype=np.float32) - 0.5
    doc = 50_000 + np.arange(240)
    cats = np.where(np.arange(240) < 3, 0, 1)
    ref = _oracle(16, cent, cb, 4, 16, 1, x, doc, cats)
    q = g.random((1, 16), dtype=np.float32)
    ids, dists, counts = ref.search_filtered_batch(q, 5, 0)
    assert counts[0] == 3
    assert all(i < 50_003 for i in ids[0, :3])


def test_oracle_unnormalised_query_matches_normalised():
    # correctness_regression/tests_feature_gated.rs:181-225
    g = np.random.default_rng(3)
    x = g.standard_normal((100, 16)).astype(np.float32)
    cent = orc.normalize(x[:4])
    cb = g.standard_normal((4, 16, 4)).astype(np.float32)
    ref = _oracle(16, cent, cb, 4, 16, 4, x, np.arange(100), np.zeros(100))
    raw = np.arange(1, 17, dtype=np.float32)[None, :]
    a = ref.search_filtered_batch(raw, 5, 0)
    b = ref.search_filtered_batch(orc.normalize(raw), 5, 0)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


# ---- GPU -------------------------------------------------------------------------

def _engine(x, d, L, M, ks, nprobe, doc, cats, field="category", use_opq=False, extra=None):
    ix = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=nprobe, seed=4,
                    use_opq=use_opq, filter_field=field)
    ix.add_items(x, np.asarray(doc, np.int64))
    for i, (dd, c) in enumerate(zip(doc, cats)):
        md = {} if c == 255 else {field: int(c)}
        if extra is not None:
            md["label"] = f"doc-{i}"
        if md:
            ix.add_metadata(int(dd), md)
    ix.build(training_sample_size=None, kmeans_max_iter=5)
    return ix


def _same(gpu, ref):
    gi, gd = gpu
    ri, rd, rc = ref
    ri = ri.astype(np.int64)
    ri[np.arange(ri.shape[1])[None, :] >= rc.astype(np.int64)[:, None]] = -1
    assert np.array_equal(gi, ri)
    assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("d,L,M,ks,opq", [(32, 64, 8, 256, False), (48, 48, 24, 16, False), (32, 32, 8, 256, True)])
def test_filtered_search_matches_oracle(d, L, M, ks, opq):
    n = 6000
    x, q = mixture(n, d, 50, 0.25, seed=d + L, nq=120)
    g = np.random.default_rng(1)
    # category 0 common, 1..6 rare (widening), 7 absent; some documents have none
    cats = np.where(g.random(n) < 0.7, 0, g.integers(1, 7, n)).astype(np.uint8)
    cats[g.random(n) < 0.05] = 255
    doc = np.arange(n) * 2 + 11
    ix = _engine(x, d, L, M, ks, 4, doc, cats, use_opq=opq)
    ref = _oracle(d, ix.centroids(), ix.codebooks(), M, ks, 4, x, doc, cats, rotation=ix.rotation())
    for want in (0, 1, 5, 7):
        for k in (1, 10, 40):
            _same(ix.batch_search_with_filter(q, k, "category", want), ref.search_filtered_batch(q, k, want))
    ids, dists = ix.search_with_filter(q[0], 10, "category", 3)
    assert ids.size <= 10 and np.all(np.diff(dists) >= 0)


@pytest.mark.gpu
def test_filtered_search_widens_past_nprobe():
    # search.rs:2648-2685 on the GPU
    g = np.random.default_rng(77)
    x = g.random((240, 16), dtype=np.float32)
    doc = 50_000 + np.arange(240)
    cats = np.where(np.arange(240) < 3, 0, 1)
    ix = _engine(x, 16, 8, 4, 16, 1, doc, cats, field="tag")
    ids, _ = ix.search_with_filter(g.random(16, dtype=np.float32), 5, "tag", 0)
    assert ids.size == 3 and np.all(ids < 50_003)


@pytest.mark.gpu
def test_metadata_changed_after_build_keeps_build_time_bitmasks():
    n, d = 3000, 32
    x, q = mixture(n, d, 30, 0.25, seed=9, nq=40)
    cats = np.zeros(n, np.uint8)
    doc = np.arange(n)
    ix = _engine(x, d, 16, 8, 256, 4, doc, cats)
    # after build: some documents move to category 2, which no bitmask records
    moved = np.arange(0, n, 7)
    for i in moved:
        ix.add_metadata(int(doc[i]), {"category": 2})
    cats2 = cats.copy()
    cats2[moved] = 2
    build_masks = np.zeros(16, np.uint64)
    build_masks[:] = 1  # every list held only category 0 at build
    ref = _oracle(d, ix.centroids(), ix.codebooks(), 8, 256, 4, x, doc, cats2, bitmask=build_masks[:ix.centroids().shape[0]])
    for want in (0, 2):
        _same(ix.batch_search_with_filter(q, 10, "category", want), ref.search_filtered_batch(q, 10, want))


@pytest.mark.gpu
def test_save_load_preserves_filter_metadata(tmp_path):
    # search.rs:2541-2586
    n, d = 240, 16
    g = np.random.default_rng(115)
    x = g.random((n, d), dtype=np.float32)
    doc = 30_000 + np.arange(n)
    ix = _engine(x, d, 4, 4, 16, 4, doc, np.arange(n) % 4, field="group", extra=True)
    query = g.random(d, dtype=np.float32)
    before = ix.search_with_filter(query, 10, "group", 2)
    assert before[0].size
    ix.save(tmp_path / "snap")
    man = json.loads((tmp_path / "snap" / "manifest.json").read_text())
    assert man["filter_field"] == "group"
    assert man["filter_metadata"][0] == {"doc_id": 30_000, "metadata": {"group": {"Int": 0}, "label": {"Str": "doc-0"}}}
    assert len(man["filter_metadata"]) == n
    snap = osnap.read_snapshot(tmp_path / "snap")
    assert any(snap["bitmasks"])
    loaded = IVFPQIndex.load(tmp_path / "snap")
    after = loaded.search_with_filter(query, 10, "group", 2)
    assert np.array_equal(before[0], after[0]) and np.array_equal(before[1].view(np.uint32), after[1].view(np.uint32))


@pytest.mark.gpu
def test_filter_errors():
    x, _ = mixture(500, 16, 10, 0.2, seed=2, nq=1)
    plain = IVFPQIndex(16, num_clusters=4, num_codebooks=4, codebook_size=16, nprobe=2)
    plain.add_items(x)
    with pytest.raises(ValueError, match="with_filtering"):
        plain.add_metadata(0, {"category": 1})
    plain.build(kmeans_max_iter=3)
    with pytest.raises(ValueError, match="doesn't match index filter field"):
        plain.search_with_filter(x[0], 5, "category", 1)
    ix = IVFPQIndex(16, num_clusters=4, num_codebooks=4, codebook_size=16, nprobe=2, filter_field="category")
    ix.add_items(x)
    with pytest.raises(ValueError, match="exceeds bitmask limit of 63"):
        ix.add_metadata(0, {"category": 64})
    with pytest.raises(ValueError, match="must be an integer in 0..63"):
        ix.add_metadata(0, {"category": "blue"})
    ix.add_metadata(0, {"category": 1, "weight": 0.5, "ok": True})
    ix.build(kmeans_max_iter=3)
    with pytest.raises(ValueError, match="doesn't match index filter field"):
        ix.search_with_filter(x[0], 5, "other", 1)
    with pytest.raises(ValueError, match="exceeds bitmask limit of 63"):
        ix.search_with_filter(x[0], 5, "category", 64)
    with pytest.raises(ValueError, match="must be an integer in 0..63"):
        ix.search_with_filter(x[0], 5, "category", 1.5)
    ids, _ = ix.search_with_filter(x[0], 5, "category", 1)
    assert list(ids) == [0]
