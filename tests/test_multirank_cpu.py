"""Sharded search logic with world_size 2 on CPU (gloo): each rank scans
only the lists the engine's packer gives it, the per-rank top-k are
all-gathered and merged by (distance, id), and the result must equal the
unsharded search.  Ranks run the CPU oracle; the partition comes from the
engine library's host-only vg_shard_assign_lists."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
N, D, L, M, KS, NPROBE, K, NQ = 3000, 16, 24, 4, 16, 6, 10, 40


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((N, D)).astype(np.float32)
    q = rng.standard_normal((NQ, D)).astype(np.float32)
    import oracle as orc

    xn = orc.normalize(x)
    cent = xn[rng.choice(N, L, replace=False)]
    cb = (rng.standard_normal((M, KS, D // M)) * 0.2).astype(np.float32)
    return x, q, cent, cb


def _rank_main(rank, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    import oracle as orc
    from vicinity_b200.ivf_pq import shard_assign_lists

    x, q, cent, cb = _data()
    ix = orc.OracleIndex(D, L, M, KS, NPROBE)
    ix.set_trained(cent, cb)
    ix.add(np.arange(N, dtype=np.uint32), x)  # doc id == internal id
    ix.finalize()
    sizes = np.diff(ix.list_offsets())
    owner = shard_assign_lists(sizes, WORLD)
    # this rank's shard: rebuild with foreign lists emptied (same codes, same
    # probes: centroids stay replicated, only the scanned lists differ)
    assign = ix.assignments()
    mine = owner[assign] == rank
    shard = orc.OracleIndex(D, L, M, KS, NPROBE)
    shard.set_trained(cent, cb)
    shard.add(np.nonzero(mine)[0].astype(np.uint32), x[mine])
    shard.adopt_codes(assign[mine], ix.codes()[mine])
    ids, dists, cnt = shard.search_batch(q, K)
    packed = torch.from_numpy(np.stack([ids.astype(np.int64), dists.view(np.int32).astype(np.int64)], -1))
    gathered = [torch.empty_like(packed) for _ in range(WORLD)]
    dist.all_gather(gathered, packed)
    if rank == 0:
        keys = []
        for g in gathered:
            a = g.numpy()
            keys.append((a[..., 0], a[..., 1].astype(np.int32).view(np.float32)))
        merged = np.empty((NQ, K), np.int64)
        for r in range(NQ):
            cands = []
            for ids_g, d_g in keys:
                for i, dd in zip(ids_g[r], d_g[r]):
                    if i != 0xFFFFFFFF:
                        cands.append((orc.total_order_key(float(dd)), int(i)))
            cands.sort()
            merged[r] = [c[1] for c in cands[:K]]
        full_ids, _, _ = ix.search_batch(q, K)
        np.save(out_path, np.stack([merged, full_ids.astype(np.int64)]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharded_merge_equals_unsharded(tmp_path):
    out = tmp_path / "merged.npy"
    mp.start_processes(_rank_main, args=(_free_port(), str(out)), nprocs=WORLD, start_method="spawn", join=True)
    merged, full = np.load(out)
    assert np.array_equal(merged, full)
