"""Probe selection (find_nearest_centroids, src/ivf_pq/search.rs:1602-1617):
the nprobe nearest lists of each normalised query by 1 - q.c, ties by list
id.  From 1024 lists up the engine ranks lists with an approximate binary16
tensor-core product and re-scores, with the reference's sequential f32
arithmetic, every list the approximation's error bound cannot rule out; the
lists and distances it returns must still equal the oracle's exactly.  The
cases here crowd the bound: exact duplicates (ties broken by id), clusters
of near-duplicates (many lists inside the error window), centroids of mixed
norms, zero and unnormalised queries, and centroids too long for a useful
bound (the exact path).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from vicinity_b200 import IVFPQIndex

pytestmark = pytest.mark.gpu


def _index(cent, M=4, ks=16, nprobe=8, n=3000, seed=0):
    L, d = cent.shape
    g = np.random.default_rng(seed)
    ix = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=nprobe)
    x = g.standard_normal((n, d)).astype(np.float32)
    ix.add_items(x)
    cb = (g.standard_normal((M, ks, d // M)) * 0.1).astype(np.float32)
    ix.set_trained(cent, cb)
    ix.build()
    return ix, x, cb


def _oracle_lists(q, cent, p):
    qn = orc.normalize(q)
    ids = np.empty((q.shape[0], p), np.int64)
    dists = np.empty((q.shape[0], p), np.float32)
    for i in range(q.shape[0]):
        a, b = orc.find_nearest_centroids(qn[i], cent, p)
        ids[i], dists[i] = a, b
    return ids, dists


def _check(ix, q, cent, p):
    gl, gd = ix.nearest_lists(q, nprobe=p)
    rl, rd = _oracle_lists(q, cent, p)
    bad = np.nonzero((gl != rl).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ, first {bad[:4]}: {gl[bad[0]][:8]} vs {rl[bad[0]][:8]}"
    assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


def _unit(x):
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32)


def _adversarial_centroids(L, d, seed):
    g = np.random.default_rng(seed)
    cent = _unit(g.standard_normal((L, d)))
    cent[10:610] = cent[3]                       # 600 exact duplicates of list 3: the window overflows
    base = cent[700]
    near = base[None, :] + g.standard_normal((150, d)).astype(np.float32) * 1e-4
    cent[700:850] = _unit(near)                  # 150 lists within the error window of each other
    return cent


def _queries(cent, d, seed, nq=400):
    g = np.random.default_rng(seed + 1)
    q = g.standard_normal((nq, d)).astype(np.float32)
    q[0] = 0.0                                   # zero query: every distance is 1, all ties
    q[1] = cent[3] * 7.5                         # on the duplicated centroid, unnormalised
    q[2] = cent[700]                             # inside the near-duplicate cluster
    q[3:40] = cent[700:737] + g.standard_normal((37, d)).astype(np.float32) * 1e-3
    q[40:60] = cent[g.integers(0, cent.shape[0], 20)]
    q[60] = 1e-30                                # tiny query: left unnormalised
    q[61, 0] = 1e-39                             # a subnormal coordinate
    return q


@pytest.mark.parametrize("L,d", [(1024, 32), (2048, 96), (4096, 128)])
def test_probe_lists_match_oracle(L, d):
    cent = _adversarial_centroids(L, d, seed=L + d)
    ix, _, _ = _index(cent, M=4, ks=16)
    q = _queries(cent, d, seed=d)
    for p in (1, 10, 32, 64, 128, 200):          # 200: the exact path
        _check(ix, q, cent, p)


def test_probe_lists_mixed_norm_centroids():
    L, d = 1536, 64
    g = np.random.default_rng(5)
    cent = _unit(g.standard_normal((L, d))) * g.uniform(0.2, 3.0, (L, 1)).astype(np.float32)
    ix, _, _ = _index(cent.astype(np.float32), M=8, ks=16)
    _check(ix, _queries(cent, d, seed=5), cent, 48)


def test_probe_lists_large_centroids_score_every_list_exactly():
    L, d = 1024, 32
    g = np.random.default_rng(6)
    cent = (_unit(g.standard_normal((L, d))) * 1000.0).astype(np.float32)
    ix, _, _ = _index(cent, M=4, ks=16)
    _check(ix, g.standard_normal((64, d)).astype(np.float32), cent, 16)


def test_search_through_shortlist_matches_oracle():
    # full search parity with 2048 lists, where the shortlist selects the probes
    L, d, M, ks = 2048, 48, 8, 256
    cent = _adversarial_centroids(L, d, seed=11)
    ix, x, cb = _index(cent, M=M, ks=ks, n=40_000, seed=3)
    ref = orc.OracleIndex(d, L, M, ks, 8)
    ref.set_trained(cent, cb)
    ref.add(np.arange(x.shape[0], dtype=np.uint32), x)
    ref.finalize()
    q = _queries(cent, d, seed=4, nq=300)
    for nprobe, k in ((8, 10), (64, 100)):
        gi, gd = ix.batch_search(q, k, nprobe=nprobe)
        ri, rd, rc = ref.search_batch(q, k, nprobe=nprobe)
        ri = ri.astype(np.int64)
        ri[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = -1
        assert np.array_equal(gi, ri)
        assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


def test_nearest_lists_errors():
    cent = _unit(np.random.default_rng(0).standard_normal((16, 8)))
    ix = IVFPQIndex(8, num_clusters=16, num_codebooks=2, codebook_size=16, nprobe=4)
    with pytest.raises(Exception):
        ix.nearest_lists(np.zeros((1, 8), np.float32))      # not built
    ix.add_items(np.random.default_rng(1).standard_normal((200, 8)).astype(np.float32))
    ix.set_trained(cent, np.zeros((2, 16, 4), np.float32))
    ix.build()
    lists, dists = ix.nearest_lists(cent[:3])
    assert lists.shape == (3, 4) and list(lists[:, 0]) == [0, 1, 2]
    with pytest.raises(ValueError):
        ix.nearest_lists(np.zeros((1, 7), np.float32))
