"""Parity at the benchmark's full sizes -- the kernels and batch shapes that
bench.py times: configurations 1 and 3 (1e6 and 1e7 vectors, batches of
10,000 queries), configuration 2 (exact flat search, 1e6 x 100, k = 100) and
configuration 4 (1e8 vectors drawn on the GPU, sampled queries).

The oracle computes the list assignments and codes of sampled rows from the
engine's trained centroids and codebooks (they must be bit-identical), adopts
the engine's index and searches a sample of the batch; the engine's rows for
those queries must be bit-identical.  Over the whole batch the
size-independent properties are checked: every row sorted by (distance, id),
ids unique within a row, and the batch result equal to the same queries
searched in smaller batches (which run other kernels).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from vicinity_b200 import FlatIndex, IVFPQIndex, MISSING_LABEL
from vicinity_b200.synthetic import CONFIGS, config_data

pytestmark = pytest.mark.gpu

SAMPLE = 300  # queries re-searched by the oracle


def _check(cfg_id: int):
    cfg = CONFIGS[cfg_id]
    x, q = config_data(cfg_id, seed=0)
    ix = IVFPQIndex(cfg["d"], num_clusters=cfg["nlist"], num_codebooks=cfg["M"], codebook_size=cfg["ks"],
                    nprobe=cfg["nprobe"], seed=42)
    ix.add_items(x)
    ix.build(training_sample_size=131_072, kmeans_max_iter=10)
    k = cfg["k"]
    ids, dists = ix.batch_search(q, k)

    # list assignments and codes of sampled rows, computed by the oracle from
    # the engine's trained centroids and codebooks (kmeans.rs:97-107,
    # pq.rs:136-160): bit-identical
    Lc = int(ix.info().num_centroids)
    srows = np.linspace(0, x.shape[0] - 1, 4000).astype(np.int64)
    sub = orc.OracleIndex(cfg["d"], Lc, cfg["M"], cfg["ks"], cfg["nprobe"])
    sub.set_trained(ix.centroids(), ix.codebooks())
    sub.add(np.arange(srows.size, dtype=np.uint32), x[srows])
    sub.finalize()
    assert np.array_equal(sub.assignments(), ix.assignments()[srows]), "sampled list assignments differ"
    assert np.array_equal(sub.codes(), ix.codes()[srows]), "sampled codes differ"

    # oracle on the same index, a sample of the batch
    ref = orc.OracleIndex(cfg["d"], int(ix.info().num_centroids), cfg["M"], cfg["ks"], cfg["nprobe"])
    ref.set_trained(ix.centroids(), ix.codebooks())
    ref.add(ix.doc_ids(), x)
    ref.adopt_codes(ix.assignments(), ix.codes())
    del x
    rows = np.linspace(0, q.shape[0] - 1, SAMPLE).astype(np.int64)
    ri, rd, rc = ref.search_batch(q[rows], k, threads=8)
    ri = ri.astype(np.int64)
    ri[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = MISSING_LABEL
    bad = np.nonzero((ids[rows] != ri).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} sampled rows differ from the oracle, first query {rows[bad[0]]}"
    assert np.array_equal(dists[rows].view(np.uint32), rd.view(np.uint32)), "sampled distances differ"

    # properties over the whole batch
    real = ids != MISSING_LABEL
    assert real.all(), "a full-size query returned fewer than k results"
    d64 = dists.astype(np.float64)
    order_ok = (d64[:, 1:] > d64[:, :-1]) | ((d64[:, 1:] == d64[:, :-1]) & (ids[:, 1:] > ids[:, :-1]))
    assert order_ok.all(), "rows not sorted by (distance, id)"
    srt = np.sort(ids, axis=1)
    assert (srt[:, 1:] != srt[:, :-1]).all(), "an id repeats within a row"
    # the same queries in batches below 16 per SM run the block kernels
    for s0 in (0, 5000):
        si, sd = ix.batch_search(q[s0:s0 + 1000], k)
        assert np.array_equal(si, ids[s0:s0 + 1000]), "batch size changed the ids"
        assert np.array_equal(sd.view(np.uint32), dists[s0:s0 + 1000].view(np.uint32))
    ix.close()


def test_config1_full_size_matches_oracle():
    _check(1)


def test_config3_full_size_matches_oracle():
    _check(3)


def _row_properties(ids, dists, k):
    assert (ids != MISSING_LABEL).all(), "a full-size query returned fewer than k results"
    d64 = dists.astype(np.float64)
    order_ok = (d64[:, 1:] > d64[:, :-1]) | ((d64[:, 1:] == d64[:, :-1]) & (ids[:, 1:] > ids[:, :-1]))
    assert order_ok.all(), "rows not sorted by (distance, id)"
    srt = np.sort(ids, axis=1)
    assert (srt[:, 1:] != srt[:, :-1]).all(), "an id repeats within a row"


def test_config2_full_size_matches_oracle():
    # exact inner-product top-100 (distance.rs:125-130, evaluation.rs:250-268)
    cfg = CONFIGS[2]
    x, q = config_data(2, seed=0)
    f = FlatIndex(x)
    ids, dists = f.search(q, cfg["k"])
    f.close()
    rows = np.linspace(0, q.shape[0] - 1, 200).astype(np.int64)
    ri, rd, rc = orc.flat_search_ip(x, q[rows], cfg["k"], threads=8)
    assert (rc == cfg["k"]).all()
    bad = np.nonzero((ids[rows] != ri.astype(np.int64)).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} sampled rows differ from the oracle, first query {rows[bad[0]]}"
    assert np.array_equal(dists[rows].view(np.uint32), rd.view(np.uint32)), "sampled distances differ"
    _row_properties(ids, dists, cfg["k"])


def test_config4_sampled_rows_match_oracle():
    # 1e8 vectors drawn on the GPU (never on the host); the oracle adopts the
    # engine's compacted state (doc ids, assignments, codes: no raw vectors)
    import torch

    from vicinity_b200.synthetic import device_mixture

    cfg = CONFIGS[4]
    nq, k = 2000, cfg["k"]
    ix = IVFPQIndex(cfg["d"], num_clusters=cfg["nlist"], num_codebooks=cfg["M"], codebook_size=cfg["ks"],
                    nprobe=cfg["nprobe"], seed=42)
    _, chunks, q = device_mixture(4, seed=0, device=0, nq=nq)
    first = None
    for xc in chunks:
        torch.cuda.synchronize()
        ix.add_device(xc.data_ptr(), xc.shape[0])
        if first is None:
            first = xc[:: xc.shape[0] // 2000][:2000].cpu().numpy()  # sampled rows of the first chunk
        del xc
    torch.cuda.empty_cache()
    ix.build(training_sample_size=cfg["train_sample"], kmeans_max_iter=8)
    Lc = int(ix.info().num_centroids)
    step = (1 << 22) // 2000
    srows = np.arange(2000, dtype=np.int64) * step
    sub = orc.OracleIndex(cfg["d"], Lc, cfg["M"], cfg["ks"], cfg["nprobe"])
    sub.set_trained(ix.centroids(), ix.codebooks())
    sub.add(np.arange(2000, dtype=np.uint32), first)
    sub.finalize()
    assign, codes = ix.assignments(), ix.codes()
    assert np.array_equal(sub.assignments(), assign[srows]), "sampled list assignments differ"
    assert np.array_equal(sub.codes(), codes[srows]), "sampled codes differ"
    ix.compact()
    ids, dists = ix.batch_search(q, k)
    ref = orc.OracleIndex(cfg["d"], Lc, cfg["M"], cfg["ks"], cfg["nprobe"])
    ref.set_trained(ix.centroids(), ix.codebooks())
    ref.adopt_state(ix.doc_ids(), assign, codes)
    del assign, codes
    rows = np.linspace(0, nq - 1, 100).astype(np.int64)
    ri, rd, rc = ref.search_batch(q[rows], k, threads=8)
    ri = ri.astype(np.int64)
    ri[np.arange(k)[None, :] >= rc.astype(np.int64)[:, None]] = MISSING_LABEL
    bad = np.nonzero((ids[rows] != ri).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} sampled rows differ from the oracle, first query {rows[bad[0]]}"
    assert np.array_equal(dists[rows].view(np.uint32), rd.view(np.uint32)), "sampled distances differ"
    _row_properties(ids, dists, k)
    ix.close()
