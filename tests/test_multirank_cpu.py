"""The list-sharded search protocol with world_size 2 on CPU (gloo ranks
running the oracle).

Each rank owns the lists the engine's packer gives it and searches a batch of
its own.  The ranks exchange their queries; the rank that owns a query's
nearest list seeds the query's bound: it scores its own lists of the query's
probes in order until it holds k keys, and its k-th key (the minimum over
ranks, the other ranks holding none) bounds the query's k-th key over every
list.  Each rank keeps only keys at or below that bound in its own lists and
routes every query's per-rank top-k back to its rank, which merges them by
(distance, id).  The merged rows must equal the unsharded
search of the same
queries -- the property the engine's NCCL path
(vg_ivfpq_shard / vg_ivfpq_search_batch) relies on.  The partition comes from
the engine library's host-only vg_shard_assign_lists.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
N, D, L, M, KS, NPROBE, K, NQ = 3000, 16, 24, 4, 16, 6, 10, 40  # NQ queries per rank
EMPTY = np.uint64(0xFFFFFFFFFFFFFFFF)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((N, D)).astype(np.float32)
    q = rng.standard_normal((NQ * WORLD, D)).astype(np.float32)
    import oracle as orc

    xn = orc.normalize(x)
    cent = xn[rng.choice(N, L, replace=False)]
    cb = (rng.standard_normal((M, KS, D // M)) * 0.2).astype(np.float32)
    return x, q, cent, cb


def _keys(orc, ids, dists, cnt):
    """(distance order, id) keys of result rows, EMPTY past the count."""
    out = np.full(ids.shape, EMPTY, dtype=np.uint64)
    for r in range(ids.shape[0]):
        for i in range(int(cnt[r])):
            out[r, i] = (np.uint64(orc.total_order_key(float(dists[r, i]))) << np.uint64(32)) | np.uint64(ids[r, i])
    return out


def _rank_main(rank, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    import oracle as orc
    from vicinity_b200.ivf_pq import shard_assign_lists

    x, q_all, cent, cb = _data()
    full = orc.OracleIndex(D, L, M, KS, NPROBE)
    full.set_trained(cent, cb)
    full.add(np.arange(N, dtype=np.uint32), x)  # doc id == internal id
    full.finalize()
    owner = shard_assign_lists(np.diff(full.list_offsets()), WORLD)
    assign = full.assignments()
    mine = owner[assign] == rank
    # this rank's shard: foreign lists emptied (same codes; centroids stay
    # whole, so every rank selects the same probes)
    shard = orc.OracleIndex(D, L, M, KS, NPROBE)
    shard.set_trained(cent, cb)
    shard.add(np.nonzero(mine)[0].astype(np.uint32), x[mine])
    shard.adopt_codes(assign[mine], full.codes()[mine])

    # 1-2. every rank holds the global batch (its own rows at rank * NQ)
    own = torch.from_numpy(np.ascontiguousarray(q_all[rank * NQ:(rank + 1) * NQ]))
    parts = [torch.empty_like(own) for _ in range(WORLD)]
    dist.all_gather(parts, own)
    q = torch.cat(parts).numpy()
    # 3. seed: the owner of a query's nearest list scores its own lists of the
    # query's probes in order until it holds K keys; the minimum over ranks of
    # the seed k-th keys (EMPTY where a rank seeded nothing) is the ceiling
    qn = orc.normalize(q)
    sc_cent = qn @ cent.T
    nearest = np.argmax(sc_cent, axis=1)
    top2 = np.sort(sc_cent, axis=1)[:, -2:]
    assert (top2[:, 1] - top2[:, 0] > 1e-5).all()  # no near-tie for the nearest list
    kth = np.full(q.shape[0], EMPTY, dtype=np.uint64)
    for i in range(q.shape[0]):
        if owner[nearest[i]] != rank:
            continue
        for s in range(1, NPROBE + 1):
            sid, sd, sc = shard.search_batch(q[i:i + 1], K, nprobe=s)
            if sc[0] >= K:
                kth[i] = _keys(orc, sid, sd, sc)[0, K - 1]
                break
    t = torch.from_numpy(kth.view(np.int64).copy())
    parts = [torch.empty_like(t) for _ in range(WORLD)]
    dist.all_gather(parts, t)
    ceiling = np.min(np.stack([p.numpy().view(np.uint64) for p in parts]), axis=0)
    # 4. own lists for the global batch, keys at or below the ceiling only
    ids, dists, cnt = shard.search_batch(q, K)
    keys = _keys(orc, ids, dists, cnt)
    keys[keys > ceiling[:, None]] = EMPTY
    # 5. route every query's keys to its rank and merge
    parts = [torch.empty((NQ * WORLD, K), dtype=torch.int64) for _ in range(WORLD)]
    dist.all_gather(parts, torch.from_numpy(keys.view(np.int64)))
    got = np.concatenate([p.numpy().view(np.uint64)[rank * NQ:(rank + 1) * NQ] for p in parts], axis=1)
    merged = np.sort(got, axis=1)[:, :K]
    fid, fd, fc = full.search_batch(q[rank * NQ:(rank + 1) * NQ], K)
    np.save(f"{out_path}.{rank}.npy", np.stack([merged.view(np.int64), _keys(orc, fid, fd, fc).view(np.int64)]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharded_search_equals_unsharded(tmp_path):
    out = tmp_path / "merged"
    mp.start_processes(_rank_main, args=(_free_port(), str(out)), nprocs=WORLD, start_method="spawn", join=True)
    for rank in range(WORLD):
        merged, full = np.load(f"{out}.{rank}.npy")
        assert np.array_equal(merged, full), f"rank {rank}"
        # the seed bounded every query: at least one key survived per row
        assert (merged[:, 0] != -1).all()
