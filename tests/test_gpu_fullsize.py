"""Parity at the benchmark's full sizes (configurations 1 and 3: 1e6 and 1e7
vectors, batches of 10,000 queries) -- the kernels and batch shapes that
bench.py times.

The oracle adopts the engine's trained index (centroids, codebooks, list
assignments and codes) and searches a sample of the batch; the engine's rows
for those queries must be bit-identical.  Over the whole batch the
size-independent properties are checked: every row sorted by (distance, id),
ids unique within a row, and the batch result equal to the same queries
searched in smaller batches (which run other kernels).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as orc
from vicinity_b200 import IVFPQIndex, MISSING_LABEL
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
