"""vg_flat_search_ip_noalloc: the exact flat search with its scratch in one
fixed device array, called through the C ABI.

It must return exactly what vg_flat_search_ip and the oracle's exhaustive
scan return, call after call, although every call reuses the same scratch,
and a call must leave the device's free memory unchanged.  The file is named to be collected last and needs
no state from other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20


def _lib():
    from vicinity_b200 import _lib

    return _lib


def _dev(t):
    return C.c_void_p(t.data_ptr())


def _outputs(torch, nq, k):
    return (
        torch.empty((nq, k), dtype=torch.int32, device="cuda:0"),
        torch.empty((nq, k), dtype=torch.float32, device="cuda:0"),
        torch.empty((nq,), dtype=torch.int32, device="cuda:0"),
    )


def _existing(torch, db, q, k):
    lib = _lib()
    ids, dist, cnt = _outputs(torch, q.shape[0], k)
    torch.cuda.synchronize()
    lib.check(lib.load().vg_flat_search_ip(_dev(db), db.shape[0], _dev(q), q.shape[0], q.shape[1], k, 0,
                                           _dev(ids), _dev(dist), _dev(cnt)))
    return ids.cpu().numpy(), dist.cpu().numpy(), cnt.cpu().numpy()


def _noalloc(torch, db, q, k, stream=None):
    lib = _lib()
    ids, dist, cnt = _outputs(torch, q.shape[0], k)
    handle = None
    if stream is not None:
        stream.wait_stream(torch.cuda.current_stream())
        handle = C.c_void_p(stream.cuda_stream)
    lib.check(lib.load().vg_flat_search_ip_noalloc(_dev(db), db.shape[0], _dev(q), q.shape[0], q.shape[1], k, 0,
                                                   handle, _dev(ids), _dev(dist), _dev(cnt)))
    return ids.cpu().numpy(), dist.cpu().numpy(), cnt.cpu().numpy()


def _case(torch, n, nq, d, seed):
    g = np.random.default_rng(seed)
    db = g.standard_normal((n, d), dtype=np.float32)
    q = g.standard_normal((nq, d), dtype=np.float32)
    db[7] = db[3]  # a tie: equal distances resolve to the lower row
    return torch.from_numpy(db).cuda(), torch.from_numpy(q).cuda()


def _same(a, b):
    # the tolerance of the flat-search tests: ids, counts and distance bits equal
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    assert np.array_equal(a[2], b[2])


def test_two_calls_in_a_row_match_the_allocating_entry_point():
    torch = pytest.importorskip("torch")
    # first call: 1024 queries -> 4096-column tiles, 5 tiles over 20000 rows
    db1, q1 = _case(torch, 20_000, 1024, 96, seed=1)
    want1 = _existing(torch, db1, q1, 10)
    got1 = _noalloc(torch, db1, q1, 10)
    _same(got1, want1)
    assert (got1[2] == 10).all()
    # second call reuses the scratch the first one left behind: smaller
    # database, other k, a side stream
    db2, q2 = _case(torch, 3_000, 300, 40, seed=2)
    want2 = _existing(torch, db2, q2, 33)
    got2 = _noalloc(torch, db2, q2, 33, stream=torch.cuda.Stream())
    _same(got2, want2)
    # and the first request once more, bit-identical to its first answer
    _same(_noalloc(torch, db1, q1, 10), want1)


def test_matches_the_oracle():
    # the reference's exhaustive -dot scan (src/distance.rs:125-130) on the host
    torch = pytest.importorskip("torch")
    import oracle as orc

    db, q = _case(torch, 6_000, 200, 64, seed=4)
    got = _noalloc(torch, db, q, 25)
    ri, rd, rc = orc.flat_search_ip(db.cpu().numpy(), q.cpu().numpy(), 25, threads=8)
    _same(got, (ri.astype(np.int32), rd, rc.astype(np.int32)))


def test_empty_database_gives_padding():
    torch = pytest.importorskip("torch")
    db, q = _case(torch, 8, 12, 16, seed=5)  # a placeholder; n = 0 is passed
    lib = _lib()
    ids, dist, cnt = _outputs(torch, 12, 7)
    lib.check(lib.load().vg_flat_search_ip_noalloc(_dev(db), 0, _dev(q), 12, 16, 7, 0, None, _dev(ids), _dev(dist),
                                                   _dev(cnt)))
    got = (ids.cpu().numpy(), dist.cpu().numpy(), cnt.cpu().numpy())
    assert (got[0] == -1).all() and np.isinf(got[1]).all() and (got[2] == 0).all()
    ids2, dist2, cnt2 = _outputs(torch, 12, 7)
    lib.check(lib.load().vg_flat_search_ip(_dev(db), 0, _dev(q), 12, 16, 7, 0, _dev(ids2), _dev(dist2), _dev(cnt2)))
    _same(got, (ids2.cpu().numpy(), dist2.cpu().numpy(), cnt2.cpu().numpy()))


def test_calls_allocate_no_device_memory():
    # after the first call has resolved the scratch address, a call of
    # another size leaves the device's free memory exactly as it was
    torch = pytest.importorskip("torch")
    db, q = _case(torch, 9_000, 500, 48, seed=6)
    _noalloc(torch, db, q, 20)
    db2, q2 = _case(torch, 4_000, 100, 48, seed=7)
    ids, dist, cnt = _outputs(torch, 100, 50)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(0)
    lib = _lib()
    lib.check(lib.load().vg_flat_search_ip_noalloc(_dev(db2), 4_000, _dev(q2), 100, 48, 50, 0, None, _dev(ids),
                                                   _dev(dist), _dev(cnt)))
    free_after, _ = torch.cuda.mem_get_info(0)
    assert free_after == free_before


def test_padding_when_k_exceeds_rows():
    torch = pytest.importorskip("torch")
    db, q = _case(torch, 50, 17, 32, seed=3)
    want = _existing(torch, db, q, 100)
    got = _noalloc(torch, db, q, 100)
    _same(got, want)
    assert (got[2] == 50).all()
    assert (got[0][:, 50:] == -1).all() and np.isinf(got[1][:, 50:]).all()


def test_requests_beyond_the_fixed_scratch_are_rejected():
    torch = pytest.importorskip("torch")
    lib = _lib()
    fn = lib.load().vg_flat_search_ip_noalloc
    # nq above 32768: the 128-column distance tile alone exceeds half the scratch
    nq, d, k = 40_000, 8, 10
    db = torch.zeros((1000, d), dtype=torch.float32, device="cuda:0")
    q = torch.zeros((nq, d), dtype=torch.float32, device="cuda:0")
    ids, dist, cnt = _outputs(torch, nq, k)
    with pytest.raises(ValueError, match="32 MiB"):
        lib.check(fn(_dev(db), 1000, _dev(q), nq, d, k, 0, None, _dev(ids), _dev(dist), _dev(cnt)))
    # 8192 queries over 100000 rows: 196 tiles of keys do not fit
    nq, n = 8192, 100_000
    db = torch.zeros((n, d), dtype=torch.float32, device="cuda:0")
    q = torch.zeros((nq, d), dtype=torch.float32, device="cuda:0")
    ids, dist, cnt = _outputs(torch, nq, k)
    tile = (SCRATCH_BYTES // 2) // (nq * 4) // 128 * 128
    assert nq * tile * 4 + nq * (-(-n // tile)) * k * 8 > SCRATCH_BYTES
    with pytest.raises(ValueError, match="32 MiB"):
        lib.check(fn(_dev(db), n, _dev(q), nq, d, k, 0, None, _dev(ids), _dev(dist), _dev(cnt)))


def test_host_memory_is_rejected():
    torch = pytest.importorskip("torch")
    lib = _lib()
    db = np.zeros((100, 8), np.float32)
    q = np.zeros((4, 8), np.float32)
    ids = np.zeros((4, 5), np.uint32)
    dist = np.zeros((4, 5), np.float32)
    ptr = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    with pytest.raises(ValueError, match="device memory"):
        lib.check(lib.load().vg_flat_search_ip_noalloc(ptr(db), 100, ptr(q), 4, 8, 5, 0, None, ptr(ids),
                                                       ptr(dist), None))
    assert torch.cuda.is_available()
