"""OPQ on the GPU (src/ivf_pq/opq.rs): residuals are rotated before encoding
and query residuals before every table.  With the same rotation, centroids
and codebooks, assignments, codes, search results, reranked results and
reconstructions must equal the oracle's bit for bit.  Training the rotation
is a build tool (the reference's SVD comes from nalgebra): its output is
checked for the properties the reference's own test asserts.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from oracle import snapshot as osnap
from vicinity_b200 import IVFPQIndex
from vicinity_b200.synthetic import mixture

pytestmark = pytest.mark.gpu


def _rotation(d, seed):
    q, r = np.linalg.qr(np.random.default_rng(seed).standard_normal((d, d)))
    return (q * np.sign(np.diag(r))).astype(np.float32)


def _pair(x, d, L, M, ks, rot, nprobe=6):
    src = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=nprobe, seed=9)
    src.add_items(x)
    src.set_rotation(rot)
    src.build(training_sample_size=None, kmeans_max_iter=5)  # codebooks of the rotated residuals
    cent, cb = src.centroids(), src.codebooks()
    ix = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=nprobe, seed=9)
    ix.add_items(x)
    ix.set_trained(cent, cb, rotation=rot)
    ix.build()
    ref = orc.OracleIndex(d, cent.shape[0], M, ks, nprobe)
    ref.set_trained(cent, cb)
    ref.set_rotation(rot)
    ref.add(np.arange(x.shape[0], dtype=np.uint32), x)
    ref.finalize()
    return ix, ref


def _same_search(ix, ref, q, k, nprobe, rerank=0):
    gi, gd = ix.batch_search(q, k, nprobe=nprobe, rerank_pool=rerank or None)
    ri, rd, rc = ref.search_batch(q, k, nprobe=nprobe, rerank_pool=rerank)
    ri = ri.astype(np.int64)
    ri[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = -1
    assert np.array_equal(gi, ri)
    assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


@pytest.mark.parametrize("d,L,M,ks", [(32, 32, 8, 256), (48, 24, 24, 16), (36, 16, 3, 64)])
def test_opq_parity_with_a_given_rotation(d, L, M, ks):
    x, q = mixture(6000, d, 40, 0.25, seed=d, nq=150)
    rot = _rotation(d, seed=L)
    ix, ref = _pair(x, d, L, M, ks, rot)
    assert np.array_equal(ix.assignments(), ref.assignments())
    assert np.array_equal(ix.codes(), ref.codes())
    assert np.array_equal(ix.rotation(), rot)
    for nprobe in (1, 6):
        _same_search(ix, ref, q, 10, nprobe)
    _same_search(ix, ref, q, 10, 6, rerank=50)
    for i in (0, 17, 5999):
        assert np.array_equal(ix.reconstruct(i), ref.reconstruct(i))


def test_opq_training_gives_an_orthonormal_rotation(kats):
    kat = kats["opq_training_rows_orthonormal"]
    d, M, ks, n = kat["dimension"], kat["num_codebooks"], kat["codebook_size"], kat["num_vectors"]
    i, j = np.meshgrid(np.arange(n), np.arange(d), indexing="ij")
    x = (((i * 7 + j * 3) % 100) / 100.0).astype(np.float32)
    ix = IVFPQIndex(d, num_clusters=2, num_codebooks=M, codebook_size=ks, nprobe=2, use_opq=True, seed=1)
    ix.add_items(x)
    ix.build(kmeans_max_iter=10)
    r = ix.rotation()
    assert r is not None and ix.use_opq
    np.testing.assert_array_less(np.abs((r.astype(np.float64) ** 2).sum(axis=1) - 1.0), kat["row_norm_sq_tolerance"])
    # the trained state searches exactly as the oracle does with it
    ref = orc.OracleIndex(d, ix.centroids().shape[0], M, ks, 2)
    ref.set_trained(ix.centroids(), ix.codebooks())
    ref.set_rotation(r)
    ref.add(np.arange(n, dtype=np.uint32), x)
    ref.finalize()
    assert np.array_equal(ix.codes(), ref.codes())
    _same_search(ix, ref, x[:20] + 0.01, 5, 2)


def test_opq_trained_index_recall_is_sane():
    x, q = mixture(20000, 32, 60, 0.3, seed=5, nq=200)
    ix = IVFPQIndex(32, num_clusters=64, num_codebooks=8, codebook_size=256, nprobe=16, use_opq=True, seed=3)
    ix.add_items(x)
    ix.build(training_sample_size=8000, kmeans_max_iter=6)
    r = ix.rotation()
    np.testing.assert_allclose(r @ r.T, np.eye(32), atol=1e-3)
    ids, _ = ix.batch_search(q, 10)
    xn = x / np.linalg.norm(x, axis=1, keepdims=True)
    qn = q / np.linalg.norm(q, axis=1, keepdims=True)
    truth = np.argsort(-(qn @ xn.T), axis=1)[:, :10]
    recall = np.mean([len(set(a) & set(b)) / 10 for a, b in zip(ids.tolist(), truth.tolist())])
    assert recall > 0.3


def test_opq_snapshot_round_trip(tmp_path):
    d, L, M, ks = 32, 16, 8, 256
    x, q = mixture(4000, d, 30, 0.25, seed=8, nq=60)
    rot = _rotation(d, seed=3)
    ix, ref = _pair(x, d, L, M, ks, rot)
    ix.save(tmp_path / "snap")
    got = osnap.read_snapshot(tmp_path / "snap")
    assert set(got["manifest"]["quantizer"]) == {"Optimized"}
    assert np.array_equal(got["rotation"], rot)
    loaded = IVFPQIndex.load(tmp_path / "snap")
    a_ids, a_d = ix.batch_search(q, 10)
    b_ids, b_d = loaded.batch_search(q, 10)
    assert np.array_equal(a_ids, b_ids) and np.array_equal(a_d.view(np.uint32), b_d.view(np.uint32))
    _same_search(loaded, ref, q, 10, 6)
