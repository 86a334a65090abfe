"""GPU parity: the sm_100a engine against the CPU oracle on identical inputs
and identical trained codebooks.

Bar (integer/index work bit-exact, floating point as the reference computes
it): list assignments, PQ codes and list layout must be identical; returned
ids and distances must be identical too, because every kernel on the path
reproduces the reference's sequential, separately rounded f32 arithmetic
(distance tolerance 0 -- stricter than the 1e-5 relative the spec allows).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from vicinity_b200 import IVFPQIndex, MISSING_LABEL, flat_search_ip
from vicinity_b200.synthetic import mixture

pytestmark = pytest.mark.gpu


def build_pair(x, d, L, M, ks, nprobe=8, seed=42, sample=None, iters=8, doc_base=0):
    """Engine index trained on device, and the oracle index built from the
    engine's trained centroids and codebooks."""
    ix = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=nprobe, seed=seed)
    doc = np.arange(doc_base, doc_base + x.shape[0], dtype=np.int64)
    ix.add_items(x, doc)
    ix.build(training_sample_size=sample, kmeans_max_iter=iters)
    cent, cb = ix.centroids(), ix.codebooks()
    ref = orc.OracleIndex(d, cent.shape[0], M, ks, nprobe)
    ref.set_trained(cent, cb)
    ref.add(doc.astype(np.uint32), x)
    ref.finalize()
    return ix, ref


def assert_same_layout(ix, ref):
    assert np.array_equal(ix.vectors(), ref.vectors()), "normalised rows differ"
    assert np.array_equal(ix.assignments(), ref.assignments()), "list assignments differ"
    assert np.array_equal(ix.codes(), ref.codes()), "PQ codes differ"
    assert np.array_equal(ix.list_offsets(), ref.list_offsets()), "list offsets differ"
    assert np.array_equal(ix.list_ids(), ref.list_ids()), "list order differs"


def assert_same_results(ix, ref, q, k, nprobe, rerank=0):
    if rerank:
        gi, gd = ix.batch_search(q, k, nprobe=nprobe, rerank_pool=rerank)
    else:
        gi, gd = ix.batch_search(q, k, nprobe=nprobe)
    ri, rd, rc = ref.search_batch(q, k, nprobe=nprobe, rerank_pool=rerank)
    ri = ri.astype(np.int64)
    ri[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = MISSING_LABEL
    bad = np.nonzero((gi != ri).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ, first {bad[:5]}: {gi[bad[0]][:8]} vs {ri[bad[0]][:8]}"
    assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32)), "distances differ"


# shapes: (d, L, M, ks) covering register-codebook variants of dsub 1..8,
# the general variant (dsub 12), 4-bit FastScan and odd codebook sizes
SHAPES = [
    (32, 64, 8, 256),    # dsub 4
    (96, 48, 16, 256),   # dsub 6 (config-0 subspace shape)
    (24, 32, 24, 256),   # dsub 1
    (96, 32, 8, 256),    # dsub 12 -> general variant (reference default M=8 at d=96)
    (48, 64, 24, 16),    # 4-bit FastScan, dsub 2 (config-3 subspace shape)
    (32, 40, 8, 16),     # 4-bit, dsub 4
    (16, 16, 4, 8),      # 3-bit-sized codebook through the general 8-bit path
    (40, 24, 5, 200),    # odd M and ks, dsub 8
]


@pytest.mark.parametrize("d,L,M,ks", SHAPES)
def test_build_and_search_match_oracle(d, L, M, ks):
    x, q = mixture(6000, d, 40, 0.3, seed=d * 7 + ks, nq=64)
    ix, ref = build_pair(x, d, L, M, ks)
    assert_same_layout(ix, ref)
    for nprobe, k in [(1, 10), (8, 10), (L, 32), (5, 1), (3, 64), (L, 200)]:
        assert_same_results(ix, ref, q, k, nprobe)


def test_config0_shape_matches_oracle():
    # BASELINE config 0 shape at a reduced n: d=96, nlist=256, M=16 x 8-bit, nprobe=16, k=10
    x, q = mixture(30_000, 96, 100, 0.15, seed=11, nq=200)
    ix, ref = build_pair(x, 96, 256, 16, 256, nprobe=16, sample=20_000, iters=6)
    assert_same_layout(ix, ref)
    assert_same_results(ix, ref, q, 10, 16)


def test_config1_shape_matches_oracle():
    # BASELINE config 1 shape at a reduced n: integer data 0..255, d=128, M=32 x 8-bit, nprobe=32
    x, q = mixture(40_000, 128, 100, 12.0, seed=3, centre="uniform120", integer=True, nq=200)
    ix, ref = build_pair(x, 128, 512, 32, 256, nprobe=32, sample=30_000, iters=5)
    assert_same_layout(ix, ref)
    assert_same_results(ix, ref, q, 10, 32)


def test_rerank_matches_oracle():
    x, q = mixture(8000, 32, 30, 0.3, seed=9, nq=50)
    ix, ref = build_pair(x, 32, 32, 8, 256)
    for pool in (10, 50, 200):
        assert_same_results(ix, ref, q, 10, 8, rerank=pool)


@pytest.mark.parametrize("ks", [256, 16])
def test_rerank_pool_above_256_matches_oracle(ks):
    # pools above 256 are selected in passes of 256 keys; the last pass is
    # partial, and pools larger than the probed candidates exhaust them
    x, q = mixture(8000, 32, 30, 0.3, seed=19, nq=40)
    ix, ref = build_pair(x, 32, 32, 8, ks)
    for k, nprobe, pool in [(10, 8, 257), (10, 8, 300), (10, 8, 700), (200, 8, 1000), (20, 32, 5000)]:
        assert_same_results(ix, ref, q, k, nprobe, rerank=pool)


def test_adc_odd_sizes_exact(kats):
    # pq_simd.rs:1108-1132 on the device: list sizes 0..257 must give the
    # reference's sequential sums exactly, including the tail of each list.
    kat = kats["adc_odd_sizes"]
    rng = np.random.default_rng(1)
    sizes = kat["n_candidates"]
    d, M = 20, 5
    for ks in kat["codebook_sizes"]:
        L = len(sizes)
        basis = orc.normalize(rng.standard_normal((L, d)).astype(np.float32))
        rows = []
        for li, s in enumerate(sizes):
            rows.append(basis[li] + 0.01 * rng.standard_normal((s, d)).astype(np.float32))
        x = np.concatenate(rows).astype(np.float32)
        cb = (0.05 * rng.standard_normal((M, ks, d // M))).astype(np.float32)
        ix = IVFPQIndex(d, num_clusters=L, num_codebooks=M, codebook_size=ks, nprobe=L)
        ix.add_items(x)
        ix.set_trained(basis, cb)
        ix.build()
        ref = orc.OracleIndex(d, L, M, ks, L)
        ref.set_trained(basis, cb)
        ref.add(np.arange(x.shape[0], dtype=np.uint32), x)
        ref.finalize()
        assert_same_layout(ix, ref)
        sizes_got = np.diff(ix.list_offsets())
        assert sorted(sizes_got.tolist()) == sorted(sizes)
        q = x[rng.choice(x.shape[0], 16, replace=False)]
        assert_same_results(ix, ref, q, 256, L)


def test_edge_cases():
    x, q = mixture(3000, 16, 10, 0.3, seed=2, nq=5)
    ix, ref = build_pair(x, 16, 16, 4, 16, nprobe=4)
    # k = 0 and empty batches
    gi, gd = ix.batch_search(q, 0)
    assert gi.shape == (5, 0)
    gi, gd = ix.batch_search(q[:0], 10)
    assert gi.shape == (0, 10)
    # nprobe beyond the number of lists is clamped (search.rs:1611)
    assert_same_results(ix, ref, q, 10, 1000)
    # k beyond the candidates is padded (python.rs:778-779)
    gi, gd = ix.batch_search(q, 256, nprobe=1)
    ri, rd, rc = ref.search_batch(q, 256, nprobe=1)
    for r in range(q.shape[0]):
        c = int(rc[r])
        assert (gi[r, c:] == MISSING_LABEL).all() and np.isinf(gd[r, c:]).all()
        assert np.array_equal(gi[r, :c], ri[r, :c].astype(np.int64))
    # zero query: kept as is (norm <= 1e-10), still searchable
    assert_same_results(ix, ref, np.zeros((1, 16), np.float32), 10, 4)
    # scale invariance of the query
    a, _ = ix.batch_search(q, 10)
    b, _ = ix.batch_search(q * np.float32(7.5), 10)
    assert np.array_equal(a, b)
    # single search API
    ids, dists = ix.search(q[0], 5)
    assert ids.dtype == np.int64 and dists.dtype == np.float32 and ids.shape == (5,)


def test_errors_mirror_reference():
    ix = IVFPQIndex(8, num_clusters=4, num_codebooks=2, codebook_size=8)
    with pytest.raises(ValueError, match="not built"):
        ix.batch_search(np.zeros((1, 8), np.float32), 5)
    with pytest.raises(ValueError, match="empty"):
        ix.build()
    ix.add_items(np.random.default_rng(0).standard_normal((4, 8)).astype(np.float32))
    with pytest.raises(ValueError, match="at least codebook_size"):
        ix.build()
    with pytest.raises(ValueError, match="duplicate doc_id"):
        ix.add_items(np.ones((2, 8), np.float32), ids=[100, 100])
    ix.add_items(np.random.default_rng(1).standard_normal((60, 8)).astype(np.float32))
    with pytest.raises(ValueError, match="kmeans_max_iter"):
        ix.build(kmeans_max_iter=0)
    ix.build(kmeans_max_iter=3)
    with pytest.raises(ValueError, match="already built"):
        ix.add_items(np.ones((1, 8), np.float32))
    with pytest.raises(ValueError, match="dimension mismatch"):
        ix.batch_search(np.zeros((1, 9), np.float32), 5)
    ix.compact()
    with pytest.raises(ValueError, match="compact"):
        ix.batch_search(np.zeros((1, 8), np.float32), 5, rerank_pool=10)
    ix.batch_search(np.zeros((1, 8), np.float32), 5)  # approximate search still works


def test_python_padding_kat(kats):
    # tests/test_python.py:555-564 (rerank pool 16 over 16 vectors, k = 20)
    kat = kats["python_batch_padding"]
    rng = np.random.default_rng(0)
    x = rng.standard_normal((kat["n"], kat["dim"])).astype(np.float32)
    ix = IVFPQIndex(kat["dim"], num_clusters=kat["num_clusters"], num_codebooks=kat["num_codebooks"],
                    codebook_size=kat["codebook_size"], nprobe=8, seed=0)
    ix.add_items(x)
    ix.build(training_sample_size=16, kmeans_max_iter=5)
    ids, dists = ix.batch_search(x[:2], k=kat["k"], nprobe=8, rerank_pool=16)
    assert ids.shape == (2, kat["k"]) and dists.shape == (2, kat["k"])
    assert np.all(ids[:, 16:] == kat["missing_label"])
    assert np.all(np.isinf(dists[:, 16:]))
    ids, dists = ix.search(x[0], k=5, nprobe=8, rerank_pool=len(x))
    assert ids[0] == 0 and abs(float(dists[0])) < 1e-4


def test_recall_floor_on_seeded_set():
    # search.rs:3336-3434 and tests/recall_ground_truth.rs:306-348 style floor:
    # recall@10 is monotone in nprobe and well above the reference floors.
    x, q = mixture(20_000, 64, 200, 0.2, seed=4, nq=100)
    ix = IVFPQIndex(64, num_clusters=128, num_codebooks=16, codebook_size=256, nprobe=8)
    ix.add_items(x)
    ix.build(training_sample_size=10_000, kmeans_max_iter=10)
    xn, qn = orc.normalize(x), orc.normalize(q)
    truth, _, _ = orc.flat_search_ip(xn, qn, 10, threads=4)
    recalls = []
    for nprobe in (1, 4, 8, 16, 32):
        ids, _ = ix.batch_search(q, 10, nprobe=nprobe)
        hits = sum(len(set(a.tolist()) & set(b.tolist())) for a, b in zip(ids, truth.astype(np.int64)))
        recalls.append(hits / truth.size)
    assert recalls[2] >= 0.2
    assert all(b >= a - 1e-9 for a, b in zip(recalls, recalls[1:]))


def test_flat_ip_matches_oracle():
    rng = np.random.default_rng(8)
    db = orc.normalize(rng.standard_normal((20_000, 100)).astype(np.float32))
    q = orc.normalize(rng.standard_normal((64, 100)).astype(np.float32))
    for k in (1, 10, 100):
        gi, gd = flat_search_ip(db, q, k)
        ri, rd, _ = orc.flat_search_ip(db, q, k, threads=4)
        assert np.array_equal(gi, ri.astype(np.int64))
        assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))
    gi, gd = flat_search_ip(db[:50], q, 100)
    assert (gi[:, 50:] == MISSING_LABEL).all()


@pytest.mark.parametrize("L,M,ks", [(64, 8, 256), (1100, 8, 256), (1100, 16, 16)])
def test_large_host_batch_matches_small_batches(L, M, ks):
    # queries are searched independently: one large host batch, the same
    # queries in smaller batches, and the oracle agree bit for bit
    x, q = mixture(30_000, 32, 60, 0.3, seed=L + ks, nq=6000)
    ix, ref = build_pair(x, 32, L, M, ks, nprobe=12, sample=20_000, iters=4)
    big_ids, big_d = ix.batch_search(q, 10)
    parts = [ix.batch_search(q[i:i + 2000], 10) for i in range(0, 6000, 2000)]
    assert np.array_equal(big_ids, np.concatenate([p[0] for p in parts]))
    assert np.array_equal(big_d.view(np.uint32), np.concatenate([p[1] for p in parts]).view(np.uint32))
    ri, rd, rc = ref.search_batch(q[:300], 10, nprobe=12)
    ri = ri.astype(np.int64)
    ri[np.arange(10)[None, :] >= rc.astype(np.int64)[:, None]] = MISSING_LABEL
    assert np.array_equal(big_ids[:300], ri)
    assert np.array_equal(big_d[:300].view(np.uint32), rd.view(np.uint32))


def test_direct_kernel_matches_oracle_on_every_shape():
    # Large batches (16 queries per SM and up) are scored by the direct-ADC
    # kernel, the small batches above by the query-stream kernel.  Re-run the
    # shape tests in a child process that sends every batch to the direct
    # kernel, so that both kernels are checked against the oracle on all
    # subvector sizes.
    import os
    import subprocess
    import sys
    from pathlib import Path

    env = dict(os.environ, VICINITY_SCAN_KERNEL="direct")
    root = Path(__file__).resolve().parents[1]
    res = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", str(root / "tests" / "test_gpu_parity.py"),
         "-k", "test_build_and_search_match_oracle or test_config0 or test_config1 or test_rerank or test_edge_cases",
         "-m", "gpu"],
        cwd=root, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]


def test_add_device_builds_the_same_index_as_add_items():
    # rows already in device memory (a CUDA tensor) added in two calls give
    # the index add_items builds from the same rows on the host
    import torch

    x, q = mixture(6000, 32, 30, 0.3, seed=5, nq=64)
    a = IVFPQIndex(32, num_clusters=32, num_codebooks=8, nprobe=8, seed=7)
    a.add_items(x)
    a.build(kmeans_max_iter=6)
    b = IVFPQIndex(32, num_clusters=32, num_codebooks=8, nprobe=8, seed=7)
    xd = torch.from_numpy(x).cuda()
    torch.cuda.synchronize()
    b.add_device(xd[:2500].data_ptr(), 2500)
    b.add_device(xd[2500:].data_ptr(), 3500)
    assert len(b) == 6000
    with pytest.raises(ValueError, match="duplicate"):
        b.add_items(x[:1], [17])
    b.build(kmeans_max_iter=6)
    assert np.array_equal(a.doc_ids(), b.doc_ids())
    assert np.array_equal(a.codes(), b.codes())
    ia, da = a.batch_search(q, 10)
    ib, db = b.batch_search(q, 10)
    assert np.array_equal(ia, ib) and np.array_equal(da.view(np.uint32), db.view(np.uint32))
