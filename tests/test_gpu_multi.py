"""Multi-GPU list sharding (one process per GPU, NCCL) and its failure path.

After vg_ivfpq_shard every rank keeps only the inverted lists it owns, and
each rank searches a batch of its own.  The ranks all-gather queries, probes
and pruning bounds, seed every query's pruning bound on the rank that owns its
nearest list (that rank's lists of the query's probes, in order, until it holds
k keys; the k-th key travels as an all-reduce min), scan their own lists for
the global batch and
return every query's per-rank top-k to its rank (all-to-all), which merges
them -- the reference's per-shard top-k merge
(examples/large_scale.rs:1969-2025).  Each rank's results must equal, bit for
bit, what one GPU holding the whole index returns for the same queries.
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
# (lists, subspaces, codebook size, queries per rank): a small batch on few
# lists (exact coarse scores), then larger batches on 1024 lists (tensor-core
# probe window) for 8-bit and 4-bit codes
CASES = [(128, 16, 256, 200), (1024, 16, 256, 1500), (1024, 32, 16, 1500)]


def _data(nq):
    from vicinity_b200.synthetic import mixture

    return mixture(N, D, 80, 0.25, seed=21, nq=nq)


def _build(device: int, case, world: int):
    from vicinity_b200 import IVFPQIndex

    lists, m, ks, nq = case
    x, q = _data(nq * world)
    ix = IVFPQIndex(D, num_clusters=lists, num_codebooks=m, codebook_size=ks, nprobe=NPROBE, seed=3, device=device)
    ix.add_items(x)
    ix.build(training_sample_size=12_000, kmeans_max_iter=6)
    return ix, q


def _rank_main(rank: int, world: int, workdir: str):
    os.environ.pop("VICINITY_SCAN_KERNEL", None)
    from vicinity_b200 import VicinityError, nccl_unique_id

    wd = Path(workdir)
    for ci, case in enumerate(CASES):
        ix, q = _build(rank, case, world)
        nq = case[3]
        before = ix.info().device_bytes
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
        after = ix.info().device_bytes
        mine = q[rank * nq:(rank + 1) * nq]
        ix.set_profiling(True)
        ids, dists = ix.batch_search(mine, K)
        prof = ix.profile()
        rids, rdists = ix.batch_search(mine, K, rerank_pool=40)
        try:
            ix.codes()
            partitioned_export = "exported"
        except (VicinityError, ValueError):
            partitioned_export = "refused"
        np.save(wd / f"rank{rank}_{ci}.npy", np.stack([ids.astype(np.float64), dists.astype(np.float64),
                                                       rids.astype(np.float64), rdists.astype(np.float64)]))
        (wd / f"rank{rank}_{ci}.txt").write_text(
            f"{before} {after} {prof['collective_ms']} {partitioned_export}")
        ix.close()


def test_two_gpu_sharded_search_matches_one_gpu(tmp_path):
    from vicinity_b200 import device_count

    if device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    mp.start_processes(_rank_main, args=(world, str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    for ci, case in enumerate(CASES):
        nq = case[3]
        ix, q = _build(0, case, world)
        for rank in range(world):
            mine = q[rank * nq:(rank + 1) * nq]
            ids, dists = ix.batch_search(mine, K)
            rids, rdists = ix.batch_search(mine, K, rerank_pool=40)
            got = np.load(tmp_path / f"rank{rank}_{ci}.npy")
            assert np.array_equal(got[0].astype(np.int64), ids), f"case {case} rank {rank} ids differ"
            assert np.array_equal(got[1].astype(np.float32).view(np.uint32), dists.view(np.uint32))
            assert np.array_equal(got[2].astype(np.int64), rids), f"case {case} rank {rank} reranked ids differ"
            assert np.array_equal(got[3].astype(np.float32).view(np.uint32), rdists.view(np.uint32))
            before, after, coll, exp = (tmp_path / f"rank{rank}_{ci}.txt").read_text().split()
            assert int(after) < int(before), "the shard still holds the whole index"
            assert float(coll) > 0.0 and exp == "refused"
        ix.close()


def test_shard_with_a_peer_that_never_joins_times_out():
    # host-made failure: rank 1 of a 2-rank group never starts, so the
    # bounded communicator set-up must return an error instead of waiting
    from vicinity_b200 import VicinityError, nccl_unique_id

    ix, _ = _build(0, CASES[0], 1)
    t0 = time.time()
    with pytest.raises(VicinityError, match="NCCL"):
        ix.shard(0, 2, nccl_unique_id(), timeout_ms=3000)
    assert time.time() - t0 < 60
    ids, _ = ix.batch_search(np.zeros((1, D), np.float32), K)  # still usable unsharded
    assert ids.shape == (1, K)
