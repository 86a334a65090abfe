"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (liboracle.so).

The oracle restates the reference IVF-PQ algorithm (vicinity 0.12.0) on the
host; see ivfpq_oracle.h.  Only the tests, the smoke check and the
benchmark's CPU-baseline leg use it, and only as the checker or the timed CPU
baseline -- the engine never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
LIB_PATH = _DIR / "liboracle.so"

_vp, _sz, _i = C.c_void_p, C.c_size_t, C.c_int
_SIGS = {
    "or_normalize": (None, [_vp, _sz, _sz, _vp]),
    "or_adc_table": (_i, [_vp, _sz, _sz, _sz, _vp, _vp]),
    "or_distance_with_table": (C.c_float, [_vp, _sz, _sz, _vp]),
    "or_adc_batch": (None, [_vp, _sz, _sz, _vp, _sz, _vp]),
    "or_pq_quantize": (None, [_vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    "or_pq_reconstruct": (None, [_vp, _sz, _sz, _sz, _vp, _vp]),
    "or_pack_4bit": (None, [_vp, _sz, _sz, _vp]),
    "or_quantize_lut_flat": (None, [_vp, _sz, _vp, _vp, _vp]),
    "or_fastscan_block": (None, [_vp, _vp, _sz, _vp]),
    "or_fastscan_batch_flat": (_i, [_vp, _sz, _sz, _vp, _vp]),
    "or_find_nearest_centroids": (_sz, [_vp, _sz, _vp, _sz, _sz, _vp, _vp]),
    "or_finish_top_k": (_sz, [_vp, _vp, _sz, _sz, _vp, _vp]),
    "or_total_order_key": (C.c_uint32, [C.c_float]),
    "or_assign": (None, [_vp, _sz, _sz, _vp, _sz, _vp]),
    "or_flat_search_ip": (None, [_vp, _sz, _vp, _sz, _sz, _sz, _i, _vp, _vp, _vp]),
    "or_index_new": (_vp, [_sz, _sz, _sz, _sz, _sz]),
    "or_index_free": (None, [_vp]),
    "or_index_set_trained": (_i, [_vp, _vp, _vp]),
    "or_index_add": (_i, [_vp, _vp, _vp, _sz]),
    "or_index_finalize": (_i, [_vp]),
    "or_index_adopt_codes": (_i, [_vp, _vp, _vp]),
    "or_index_adopt_state": (_i, [_vp, _vp, _sz, _vp, _vp]),
    "or_index_set_nprobe": (None, [_vp, _sz]),
    "or_index_set_rotation": (None, [_vp, _vp]),
    "or_index_set_filter": (_i, [_vp, _vp, _vp]),
    "or_index_search_filtered_batch": (_i, [_vp, _vp, _sz, _sz, _i, _i, _vp, _vp, _vp]),
    "or_rotate": (None, [_vp, _vp, _sz, _vp]),
    "or_rotate_t": (None, [_vp, _vp, _sz, _vp]),
    "or_index_num_vectors": (_sz, [_vp]),
    "or_index_get_assignments": (None, [_vp, _vp]),
    "or_index_get_codes": (None, [_vp, _vp]),
    "or_index_get_list_offsets": (None, [_vp, _vp]),
    "or_index_get_list_ids": (None, [_vp, _vp]),
    "or_index_get_vectors": (None, [_vp, _vp]),
    "or_index_reconstruct": (_i, [_vp, _sz, _vp]),
    "or_index_search_batch": (_i, [_vp, _vp, _sz, _sz, _sz, _i, _vp, _vp, _vp]),
    "or_index_search_reranked_batch": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, _i, _vp, _vp, _vp]),
}

_lib = None


def load():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            subprocess.run(["make", "-C", os.fspath(_DIR)], check=True, capture_output=True)
        lib = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def normalize(x) -> np.ndarray:
    x = f32(x)
    out = np.empty_like(x)
    load().or_normalize(_p(x), x.shape[0], x.shape[1], _p(out))
    return out


def adc_table(qres, num_codebooks: int, codebook_size: int, codebooks) -> np.ndarray:
    q = f32(qres)
    cb = f32(codebooks)
    out = np.empty(num_codebooks * codebook_size, dtype=np.float32)
    rc = load().or_adc_table(_p(q), q.size, num_codebooks, codebook_size, _p(cb), _p(out))
    if rc != 0:
        raise ValueError("bad quantizer shape")
    return out


def adc_batch(codes, num_codebooks: int, lut, codebook_size: int) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    t = f32(lut)
    n = c.size // num_codebooks
    out = np.empty(n, dtype=np.float32)
    load().or_adc_batch(_p(c), n, num_codebooks, _p(t), codebook_size, _p(out))
    return out


def distance_with_table(table, num_codebooks: int, codebook_size: int, codes) -> float:
    t = f32(table)
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    return float(load().or_distance_with_table(_p(t), num_codebooks, codebook_size, _p(c)))


def pq_quantize(x, num_codebooks: int, codebook_size: int, codebooks) -> np.ndarray:
    x = f32(x)
    x2 = x.reshape(-1, x.shape[-1])
    cb = f32(codebooks)
    out = np.empty((x2.shape[0], num_codebooks), dtype=np.uint8)
    load().or_pq_quantize(_p(x2), x2.shape[0], x2.shape[1], num_codebooks, codebook_size, _p(cb), _p(out))
    return out


def pq_reconstruct(codes, d: int, num_codebooks: int, codebook_size: int, codebooks) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    cb = f32(codebooks)
    out = np.empty(d, dtype=np.float32)
    load().or_pq_reconstruct(_p(c), d, num_codebooks, codebook_size, _p(cb), _p(out))
    return out


def pack_4bit(codes, n: int, num_codebooks: int) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty(((n + 31) // 32) * num_codebooks * 16, dtype=np.uint8)
    load().or_pack_4bit(_p(c), n, num_codebooks, _p(out))
    return out


def quantize_lut_flat(lut, num_codebooks: int):
    t = f32(lut)
    q = np.empty(num_codebooks * 16, dtype=np.uint8)
    scale = C.c_float()
    offset = C.c_float()
    load().or_quantize_lut_flat(_p(t), num_codebooks, _p(q), C.addressof(scale), C.addressof(offset))
    return q, scale.value, offset.value


def fastscan_block(block, lut_q, num_codebooks: int) -> np.ndarray:
    b = np.ascontiguousarray(block, dtype=np.uint8)
    q = np.ascontiguousarray(lut_q, dtype=np.uint8)
    out = np.empty(32, dtype=np.uint16)
    load().or_fastscan_block(_p(b), _p(q), num_codebooks, _p(out))
    return out


def fastscan_batch_flat(packed, n: int, num_codebooks: int, lut) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    t = f32(lut)
    out = np.empty(n, dtype=np.float32)
    rc = load().or_fastscan_batch_flat(_p(p), n, num_codebooks, _p(t), _p(out))
    if rc != 0:
        raise OverflowError("FastScan accumulates LUT terms in u16: too many codebooks would overflow")
    return out


def rotate(r, v, transpose: bool = False) -> np.ndarray:
    """opq.rs:181-205: R v (or R^T v) with R [d][d] row-major."""
    v = f32(v)
    d = v.shape[0]
    r = f32(r).reshape(d, d)
    out = np.empty(d, np.float32)
    (load().or_rotate_t if transpose else load().or_rotate)(_p(r), _p(v), d, _p(out))
    return out


def find_nearest_centroids(query, centroids, nprobe: int):
    q = f32(query)
    c = f32(centroids)
    ids = np.empty(max(nprobe, 1), dtype=np.uint32)
    d = np.empty(max(nprobe, 1), dtype=np.float32)
    cnt = load().or_find_nearest_centroids(_p(q), q.size, _p(c), c.shape[0], nprobe, _p(ids), _p(d))
    return ids[:cnt], d[:cnt]


def finish_top_k(ids, dists, k: int):
    i = np.ascontiguousarray(ids, dtype=np.uint32)
    d = f32(dists)
    oi = np.empty(max(i.size, 1), dtype=np.uint32)
    od = np.empty(max(i.size, 1), dtype=np.float32)
    cnt = load().or_finish_top_k(_p(i), _p(d), i.size, k, _p(oi), _p(od))
    return oi[:cnt], od[:cnt]


def total_order_key(x: float) -> int:
    return int(load().or_total_order_key(x))


def assign(xn, centroids) -> np.ndarray:
    x = f32(xn)
    c = f32(centroids)
    out = np.empty(x.shape[0], dtype=np.uint32)
    load().or_assign(_p(x), x.shape[0], x.shape[1], _p(c), c.shape[0], _p(out))
    return out


def flat_search_ip(db, queries, k: int, threads: int = 1):
    x = f32(db)
    q = f32(queries)
    nq = q.shape[0]
    ids = np.empty((nq, k), dtype=np.uint32)
    d = np.empty((nq, k), dtype=np.float32)
    cnt = np.empty(nq, dtype=np.uint32)
    load().or_flat_search_ip(_p(x), x.shape[0], _p(q), nq, x.shape[1], k, threads, _p(ids), _p(d), _p(cnt))
    return ids, d, cnt


class OracleIndex:
    """Reference-algorithm IVF-PQ index on the host (search.rs restated)."""

    def __init__(self, d: int, num_clusters: int, num_codebooks: int, codebook_size: int, nprobe: int):
        self._lib = load()
        self._h = self._lib.or_index_new(d, num_clusters, num_codebooks, codebook_size, nprobe)
        if not self._h:
            raise ValueError("invalid IVF-PQ shape")
        self.d, self.M, self.ks, self.L = d, num_codebooks, codebook_size, num_clusters

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.or_index_free(h)
            self._h = None

    def set_trained(self, centroids, codebooks):
        c, cb = f32(centroids), f32(codebooks)
        assert c.shape == (self.L, self.d)
        self._c, self._cb = c, cb
        self._lib.or_index_set_trained(self._h, _p(c), _p(cb))

    def add(self, doc_ids, x):
        ids = np.ascontiguousarray(doc_ids, dtype=np.uint32)
        x = f32(x)
        assert self._lib.or_index_add(self._h, _p(ids), _p(x), x.shape[0]) == 0

    def finalize(self):
        assert self._lib.or_index_finalize(self._h) == 0

    def adopt_codes(self, assignments, codes):
        a = np.ascontiguousarray(assignments, dtype=np.uint32)
        c = np.ascontiguousarray(codes, dtype=np.uint8)
        assert self._lib.or_index_adopt_codes(self._h, _p(a), _p(c)) == 0

    def adopt_state(self, doc_ids, assignments, codes):
        """The built state of a compacted index (no raw vectors): doc ids,
        list assignments and codes (search.rs:901-904)."""
        i = np.ascontiguousarray(doc_ids, dtype=np.uint32)
        a = np.ascontiguousarray(assignments, dtype=np.uint32)
        c = np.ascontiguousarray(codes, dtype=np.uint8)
        assert self._lib.or_index_adopt_state(self._h, _p(i), i.shape[0], _p(a), _p(c)) == 0

    def set_filter(self, category, bitmask=None):
        """Per-vector filter categories (255: none) and per-list bitmasks
        (None: from the categories, as at build); call after finalize."""
        self._cat = np.ascontiguousarray(category, dtype=np.uint8)
        self._mask = None if bitmask is None else np.ascontiguousarray(bitmask, dtype=np.uint64)
        st = self._lib.or_index_set_filter(self._h, _p(self._cat), None if self._mask is None else _p(self._mask))
        if st:
            raise RuntimeError(f"or_index_set_filter failed ({st})")

    def search_filtered_batch(self, queries, k: int, want: int, threads: int = 1):
        q = f32(queries)
        nq = q.shape[0]
        ids = np.empty((nq, k), np.uint32)
        dists = np.empty((nq, k), np.float32)
        counts = np.empty(nq, np.uint32)
        st = self._lib.or_index_search_filtered_batch(self._h, _p(q), nq, k, want, threads, _p(ids), _p(dists),
                                                      _p(counts))
        if st:
            raise RuntimeError(f"or_index_search_filtered_batch failed ({st})")
        return ids, dists, counts

    def set_rotation(self, rotation):
        """OPQ rotation [d][d] (None clears); set before finalize/adopt."""
        if rotation is None:
            self._lib.or_index_set_rotation(self._h, None)
        else:
            self._rot = f32(rotation).reshape(self.d, self.d)
            self._lib.or_index_set_rotation(self._h, _p(self._rot))

    def set_nprobe(self, nprobe: int):
        self._lib.or_index_set_nprobe(self._h, nprobe)

    def __len__(self):
        return int(self._lib.or_index_num_vectors(self._h))

    def assignments(self):
        out = np.empty(len(self), dtype=np.uint32)
        self._lib.or_index_get_assignments(self._h, _p(out))
        return out

    def codes(self):
        out = np.empty((len(self), self.M), dtype=np.uint8)
        self._lib.or_index_get_codes(self._h, _p(out))
        return out

    def list_offsets(self):
        out = np.empty(self.L + 1, dtype=np.uint64)
        self._lib.or_index_get_list_offsets(self._h, _p(out))
        return out

    def list_ids(self):
        out = np.empty(len(self), dtype=np.uint32)
        self._lib.or_index_get_list_ids(self._h, _p(out))
        return out

    def vectors(self):
        out = np.empty((len(self), self.d), dtype=np.float32)
        self._lib.or_index_get_vectors(self._h, _p(out))
        return out

    def reconstruct(self, idx: int):
        out = np.empty(self.d, dtype=np.float32)
        assert self._lib.or_index_reconstruct(self._h, idx, _p(out)) == 0
        return out

    def search_batch(self, queries, k: int, nprobe: int = 0, threads: int = 1, rerank_pool: int = 0):
        q = f32(queries)
        nq = q.shape[0]
        ids = np.empty((nq, k), dtype=np.uint32)
        d = np.empty((nq, k), dtype=np.float32)
        cnt = np.empty(nq, dtype=np.uint32)
        if rerank_pool:
            rc = self._lib.or_index_search_reranked_batch(
                self._h, _p(q), nq, k, rerank_pool, nprobe, threads, _p(ids), _p(d), _p(cnt)
            )
        else:
            rc = self._lib.or_index_search_batch(self._h, _p(q), nq, k, nprobe, threads, _p(ids), _p(d), _p(cnt))
        assert rc == 0, rc
        return ids, d, cnt
