"""The tensor-core candidate window (tc_select.cu) against the oracle.

Exact inner-product search (src/distance.rs:125-130, the ground truth of
src/benchmark/evaluation.rs:250-268) and list assignment
(src/partitioning/kmeans.rs:97-107) rank columns by binary16 tensor-core
products and re-score, with the reference's sequential f32 dot, every column
the error bound cannot rule out.  Results must equal the oracle's exact scan
bit for bit: ids, distances and counts.  The cases cover both K paddings (64
and 128), rows past 128 floats (the exact path), partial row and column
tiles, k from 1 to 256, exact duplicates and near-duplicate clusters (windows
that overflow into the exact re-score of a whole row), unnormalised queries
and column ranges split across work units.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from vicinity_b200 import FlatIndex, IVFPQIndex, MISSING_LABEL, flat_search_ip

pytestmark = pytest.mark.gpu


def _oracle(db, q, k):
    ri, rd, rc = orc.flat_search_ip(db, q, k, threads=8)
    ri = ri.astype(np.int64)
    ri[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = MISSING_LABEL
    return ri, rd


def _same(gi, gd, ri, rd):
    bad = np.nonzero((gi != ri).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ, first {bad[:4]}: {gi[bad[0]][:6]} vs {ri[bad[0]][:6]}"
    assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


@pytest.mark.parametrize("n,d,nq", [(3000, 64, 130), (20_000, 100, 257), (9_999, 128, 64), (5_000, 33, 40),
                                    (4_000, 130, 20)])
def test_flat_matches_oracle(n, d, nq):
    g = np.random.default_rng(n + d)
    db = orc.normalize(g.standard_normal((n, d)).astype(np.float32))
    q = orc.normalize(g.standard_normal((nq, d)).astype(np.float32))
    f = FlatIndex(db)
    for k in (1, 7, 32, 100, 256):
        _same(*f.search(q, k), *_oracle(db, q, k))


def test_flat_adversarial_rows():
    g = np.random.default_rng(3)
    n, d = 12_000, 96
    db = orc.normalize(g.standard_normal((n, d)).astype(np.float32))
    db[100:900] = db[5]                                   # 800 exact duplicates: the window overflows
    db[2000:2300] = orc.normalize(db[2000] + g.standard_normal((300, d)).astype(np.float32) * 1e-4)
    db[5000] = 0.0                                        # a zero row
    q = g.standard_normal((96, d)).astype(np.float32) * 3.0   # unnormalised queries
    q[0] = db[5]
    q[1] = db[2000]
    q[2] = 0.0                                            # every distance -0 / +0: ties by row
    q[3, 0] = 1e-39                                       # subnormal coordinate
    q[4] *= 1e4                                           # long query
    f = FlatIndex(db)
    for k in (1, 10, 100):
        _same(*f.search(q, k), *_oracle(db, q, k))


def test_flat_many_column_ranges():
    # more columns than one range holds (u16 histogram counts): several
    # ranges per row block, merged by the finisher
    g = np.random.default_rng(11)
    n, d = 150_000, 64
    db = orc.normalize(g.standard_normal((n, d)).astype(np.float32))
    q = orc.normalize(g.standard_normal((200, d)).astype(np.float32))
    _same(*flat_search_ip(db, q, 50), *_oracle(db, q, 50))


def test_flat_sampled_threshold_edges():
    # 300,000 rows: the chunk maxima of every 8th operand tile bound each
    # query's k-th product before the gather pass over every column.  k up to
    # 256; one row duplicated across sampled and unsampled tiles (ties at the
    # top), a tight cluster, a query opposite to a row (a negative k-th product)
    g = np.random.default_rng(21)
    n, d = 300_000, 96
    db = orc.normalize(g.standard_normal((n, d)).astype(np.float32))
    db[::997] = db[3]
    db[150_000:150_400] = orc.normalize(db[150_000] + g.standard_normal((400, d)).astype(np.float32) * 1e-4)
    q = orc.normalize(g.standard_normal((64, d)).astype(np.float32))
    q[0] = db[3]
    q[1] = db[150_000]
    q[2] = -db[3]
    f = FlatIndex(db)
    for k in (1, 64, 256):
        _same(*f.search(q, k), *_oracle(db, q, k))
    f.close()


def test_flat_fewer_rows_than_k_and_empty():
    g = np.random.default_rng(4)
    db = orc.normalize(g.standard_normal((70, 48)).astype(np.float32))
    q = orc.normalize(g.standard_normal((9, 48)).astype(np.float32))
    gi, gd = FlatIndex(db).search(q, 100)
    ri, rd = _oracle(db, q, 100)
    _same(gi, gd, ri, rd)
    assert (gi[:, 70:] == MISSING_LABEL).all() and np.isinf(gd[:, 70:]).all()
    gi, gd = FlatIndex(np.zeros((0, 48), np.float32)).search(q, 5)
    assert (gi == MISSING_LABEL).all() and np.isinf(gd).all()


def test_flat_search_on_a_caller_stream():
    import torch

    g = np.random.default_rng(5)
    db = orc.normalize(g.standard_normal((8_000, 100)).astype(np.float32))
    q = orc.normalize(g.standard_normal((300, 100)).astype(np.float32))
    xd = torch.from_numpy(db).cuda()
    qd = torch.from_numpy(q).cuda()
    f = FlatIndex.from_device(xd.data_ptr(), db.shape[0], db.shape[1])
    ids = torch.empty((300, 20), dtype=torch.int32, device="cuda")
    dist = torch.empty((300, 20), dtype=torch.float32, device="cuda")
    cnt = torch.empty((300,), dtype=torch.int32, device="cuda")
    s = torch.cuda.Stream()
    f.search_raw(qd.data_ptr(), 300, 20, s.cuda_stream, ids.data_ptr(), dist.data_ptr(), cnt.data_ptr())
    ri, rd = _oracle(db, q, 20)
    _same(ids.cpu().numpy().astype(np.int64), dist.cpu().numpy(), ri, rd)
    assert (cnt.cpu().numpy() == 20).all()
    f.close()


@pytest.mark.parametrize("L,d", [(600, 64), (2048, 96)])
def test_assignments_and_codes_match_oracle(L, d):
    # list assignment with the tensor-core window (P = 1) and the encode on top
    g = np.random.default_rng(L)
    n, M, ks = 40_000, 8, 256
    cent = orc.normalize(g.standard_normal((L, d)).astype(np.float32))
    cent[50:60] = cent[7]                                 # tied centroids: lowest list wins
    x = g.standard_normal((n, d)).astype(np.float32)
    x[:20] = cent[7]                                      # rows on the tied centroid
    cb = (g.standard_normal((M, ks, d // M)) * 0.05).astype(np.float32)
    ix = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=8)
    ix.add_items(x)
    ix.set_trained(cent, cb)
    ix.build()
    ref = orc.OracleIndex(d, L, M, ks, 8)
    ref.set_trained(cent, cb)
    ref.add(np.arange(n, dtype=np.uint32), x)
    ref.finalize()
    assert np.array_equal(ix.assignments(), ref.assignments())
    assert np.array_equal(ix.codes(), ref.codes())
    assert (ix.assignments()[:20] == 7).all()
