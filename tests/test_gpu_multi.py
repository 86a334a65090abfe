"""Multi-GPU list sharding (one process per GPU, NCCL all-gather merge) and
its failure path.

The sharded search must return exactly what one GPU returns for the same
index: lists are partitioned, every rank scans only its own, and the
per-rank top-k keys (distance, id) are merged after one all-gather.
"""
from __future__ import annotations

import os
import time
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N, D, L, M, KS, NPROBE, K, NQ = 30_000, 64, 128, 16, 256, 12, 10, 200


def _data():
    from vicinity_b200.synthetic import mixture

    return mixture(N, D, 80, 0.25, seed=21, nq=NQ)


def _build(device: int):
    from vicinity_b200 import IVFPQIndex

    x, q = _data()
    ix = IVFPQIndex(D, num_clusters=L, num_codebooks=M, codebook_size=KS, nprobe=NPROBE, seed=3, device=device)
    ix.add_items(x)
    ix.build(training_sample_size=12_000, kmeans_max_iter=6)
    return ix, q


def _rank_main(rank: int, world: int, workdir: str):
    os.environ.pop("VICINITY_SCAN_KERNEL", None)
    from vicinity_b200 import nccl_unique_id

    wd = Path(workdir)
    ix, q = _build(rank)
    idfile = wd / "nccl.id"
    if rank == 0:
        uid = nccl_unique_id()
        tmp = wd / "nccl.id.tmp"
        tmp.write_bytes(uid)
        tmp.rename(idfile)
    else:
        deadline = time.time() + 120
        while not idfile.exists():
            if time.time() > deadline:
                raise TimeoutError("rank 0 never published the NCCL id")
            time.sleep(0.05)
        uid = idfile.read_bytes()
    ix.shard(rank, world, uid, timeout_ms=60_000)
    ids, dists = ix.batch_search(q, K)
    rids, rdists = ix.batch_search(q, K, rerank_pool=40)
    np.save(wd / f"rank{rank}.npy", np.stack([ids.astype(np.float64), dists.astype(np.float64),
                                              rids.astype(np.float64), rdists.astype(np.float64)]))
    ix.close()


def test_two_gpu_sharded_search_matches_one_gpu(tmp_path):
    from vicinity_b200 import device_count

    if device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank_main, args=(2, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    ix, q = _build(0)
    ids, dists = ix.batch_search(q, K)
    rids, rdists = ix.batch_search(q, K, rerank_pool=40)
    for rank in range(2):
        got = np.load(tmp_path / f"rank{rank}.npy")
        assert np.array_equal(got[0].astype(np.int64), ids), f"rank {rank} ids differ"
        assert np.array_equal(got[1].astype(np.float32).view(np.uint32), dists.view(np.uint32))
        assert np.array_equal(got[2].astype(np.int64), rids), f"rank {rank} reranked ids differ"
        assert np.array_equal(got[3].astype(np.float32).view(np.uint32), rdists.view(np.uint32))


def test_shard_with_a_peer_that_never_joins_times_out():
    # host-made failure: rank 1 of a 2-rank group never starts, so the
    # bounded communicator set-up must return an error instead of waiting
    from vicinity_b200 import VicinityError, nccl_unique_id

    ix, _ = _build(0)
    t0 = time.time()
    with pytest.raises(VicinityError, match="NCCL"):
        ix.shard(0, 2, nccl_unique_id(), timeout_ms=3000)
    assert time.time() - t0 < 60
    ids, _ = ix.batch_search(np.zeros((1, D), np.float32), K)  # still usable unsharded
    assert ids.shape == (1, K)
