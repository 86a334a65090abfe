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

N, D, NPROBE, K = 30_000, 64, 12, 10
# (lists, subspaces, codebook size, queries): a small batch on few lists (block
# kernels, exact coarse scores), then batches above 16 queries per SM on 1024
# lists (warp-per-query kernels, binary16 probe shortlist) for 8-bit and 4-bit codes
CASES = [(128, 16, 256, 200), (1024, 16, 256, 3000), (1024, 32, 16, 3000)]
L, M, KS, NQ = CASES[0]


def _data(nq=NQ):
    from vicinity_b200.synthetic import mixture

    return mixture(N, D, 80, 0.25, seed=21, nq=nq)


def _build(device: int, case=CASES[0]):
    from vicinity_b200 import IVFPQIndex

    lists, m, ks, nq = case
    x, q = _data(nq)
    ix = IVFPQIndex(D, num_clusters=lists, num_codebooks=m, codebook_size=ks, nprobe=NPROBE, seed=3, device=device)
    ix.add_items(x)
    ix.build(training_sample_size=12_000, kmeans_max_iter=6)
    return ix, q


def _rank_main(rank: int, world: int, workdir: str):
    os.environ.pop("VICINITY_SCAN_KERNEL", None)
    from vicinity_b200 import nccl_unique_id

    wd = Path(workdir)
    for ci, case in enumerate(CASES):
        ix, q = _build(rank, case)
        idfile = wd / f"nccl{ci}.id"
        if rank == 0:
            uid = nccl_unique_id()
            tmp = wd / f"nccl{ci}.id.tmp"
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
        np.save(wd / f"rank{rank}_{ci}.npy", np.stack([ids.astype(np.float64), dists.astype(np.float64),
                                                       rids.astype(np.float64), rdists.astype(np.float64)]))
        ix.close()


def test_two_gpu_sharded_search_matches_one_gpu(tmp_path):
    from vicinity_b200 import device_count

    if device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank_main, args=(2, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    for ci, case in enumerate(CASES):
        ix, q = _build(0, case)
        ids, dists = ix.batch_search(q, K)
        rids, rdists = ix.batch_search(q, K, rerank_pool=40)
        ix.close()
        for rank in range(2):
            got = np.load(tmp_path / f"rank{rank}_{ci}.npy")
            assert np.array_equal(got[0].astype(np.int64), ids), f"case {case} rank {rank} ids differ"
            assert np.array_equal(got[1].astype(np.float32).view(np.uint32), dists.view(np.uint32))
            assert np.array_equal(got[2].astype(np.int64), rids), f"case {case} rank {rank} reranked ids differ"
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
