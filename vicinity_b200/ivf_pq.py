"""Python mirror of vicinity's IVF-PQ binding, running on the B200 engine.

`IVFPQIndex` keeps the constructor arguments, methods, return types and
errors of the reference's PyO3 class (vicinity 0.12.0, src/python.rs:523-850)
so code written against ``pyvicinity.IVFPQIndex`` runs unchanged; every
method is a thin call into the C ABI of ``libvicinity_gpu.so``.
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np

from . import _lib

MISSING_LABEL = -1  # src/python.rs:1303
MISSING_DISTANCE = float("inf")  # src/python.rs:1304


def default_ivfpq_codebooks(dim: int) -> int:
    """Largest divisor of ``dim`` up to 8 (src/python.rs:1145-1150)."""
    for m in range(min(8, dim), 0, -1):
        if dim % m == 0:
            return m
    return 1


def _validate_shape(dim, num_clusters, num_codebooks, codebook_size, nprobe):
    """src/python.rs:1152-1179 (validate_ivfpq_shape)."""
    if dim == 0:
        raise ValueError("dim must be greater than 0")
    if num_clusters == 0:
        raise ValueError("num_clusters must be greater than 0")
    if num_codebooks == 0 or dim % num_codebooks != 0:
        raise ValueError(
            f"num_codebooks must be a non-zero divisor of dim (dim={dim}, num_codebooks={num_codebooks})"
        )
    if codebook_size == 0 or codebook_size > 256:
        raise ValueError("codebook_size must be in the range 1..=256")
    if nprobe == 0:
        raise ValueError("nprobe must be greater than 0")


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _metadata_value(v) -> dict:
    """A Python value in the serde form of MetadataValue (filtering/mod.rs)."""
    if isinstance(v, (bool, np.bool_)):
        return {"Bool": bool(v)}
    if isinstance(v, (int, np.integer)):
        return {"Int": int(v)}
    if isinstance(v, (float, np.floating)):
        return {"Float": float(v)}
    if isinstance(v, str):
        return {"Str": v}
    raise TypeError(f"metadata values are int, float, str or bool, got {type(v).__name__}")


class IVFPQIndex:
    """IVF-PQ index on one GPU (or one shard of a multi-GPU group)."""

    def __init__(
        self,
        dim: int,
        num_clusters: int = 256,
        num_codebooks: int | None = None,
        codebook_size: int = 256,
        nprobe: int = 1,
        use_opq: bool = False,
        seed: int = 42,
        device: int = 0,
        filter_field: str | None = None,
    ):
        num_codebooks = default_ivfpq_codebooks(dim) if num_codebooks is None else num_codebooks
        _validate_shape(dim, num_clusters, num_codebooks, codebook_size, nprobe)
        self._lib = _lib.load()
        params = _lib.VgParams(
            num_clusters=num_clusters,
            nprobe=nprobe,
            num_codebooks=num_codebooks,
            codebook_size=codebook_size,
            use_opq=int(bool(use_opq)),
            reserved=0,
            seed=seed,
        )
        handle = C.c_void_p()
        _lib.check(self._lib.vg_ivfpq_create(dim, C.byref(params), device, C.byref(handle)))
        self._h = handle
        self._used_ids: set[int] = set()
        self._id_ranges: list[tuple[int, int]] = []  # ids given by add_device, [lo, hi)
        self._dim = dim
        if filter_field is not None:  # IVFPQIndex::with_filtering (search.rs:414-434)
            _lib.check(self._lib.vg_ivfpq_set_filter_field(self._h, str(filter_field).encode()))

    # -- lifecycle ---------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.vg_ivfpq_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    # -- persistence (src/python.rs:654-681) ------------------------------
    def save(self, path) -> None:
        """Write a directory snapshot in the reference's format
        (IVFPQIndex::save_to_dir): ValueError before build, OSError on I/O."""
        _lib.check(self._lib.vg_ivfpq_save(self._h, os.fsencode(os.fspath(path))))

    @staticmethod
    def load(path, device: int = 0) -> "IVFPQIndex":
        """Load a directory snapshot written by ``save`` or by the reference
        (IVFPQIndex::load_from_dir): FileNotFoundError when it is missing,
        RuntimeError when it is malformed."""
        lib = _lib.load()
        handle = C.c_void_p()
        _lib.check(lib.vg_ivfpq_load(os.fsencode(os.fspath(path)), device, C.byref(handle)))
        return IVFPQIndex._adopt(lib, handle)

    def save_generation(self, path) -> None:
        """Save this index as one published generation below ``path``
        (IVFPQIndex::save_to_generation): ``path/generations/<id>`` plus an
        atomically replaced ``path/CURRENT``; earlier generations stay."""
        _lib.check(self._lib.vg_ivfpq_save_generation(self._h, os.fsencode(os.fspath(path))))

    @staticmethod
    def load_generation(path, device: int = 0) -> "IVFPQIndex":
        """Load the generation named by ``path/CURRENT``
        (IVFPQIndex::load_from_generation)."""
        lib = _lib.load()
        handle = C.c_void_p()
        _lib.check(lib.vg_ivfpq_load_generation(os.fsencode(os.fspath(path)), device, C.byref(handle)))
        return IVFPQIndex._adopt(lib, handle)

    @staticmethod
    def _adopt(lib, handle) -> "IVFPQIndex":
        ix = IVFPQIndex.__new__(IVFPQIndex)
        ix._lib = lib
        ix._h = handle
        ix._used_ids = set()
        ix._id_ranges = []
        ix._dim = int(ix.info().dimension)
        return ix

    # -- construction --------------------------------------------------------
    def add_items(self, vectors, ids=None) -> None:
        """src/python.rs:581-620: rows are normalised on insertion; ids are
        unique u32 values, sequential from ``len(self)`` when omitted."""
        x = np.ascontiguousarray(vectors, dtype=np.float32)
        if x.ndim != 2:
            raise ValueError("vectors must be a 2-D array")
        n, d = x.shape
        if d != self._dim:
            raise ValueError(f"dimension mismatch: index expects {self._dim}, got {d}")
        if ids is None:
            base = len(self)
            if base + n - 1 <= 0xFFFFFFFF and not any(base <= u < base + n for u in self._used_ids
                                                       if u >= base):
                id_u32 = np.arange(base, base + n, dtype=np.uint32)
            else:  # src/python.rs:1209-1229 (sequential_ids_avoiding)
                out = []
                cand = base
                while len(out) < n:
                    if cand > 0xFFFFFFFF:
                        raise ValueError("implicit IDs exceed the u32 ID limit")
                    if cand not in self._used_ids:
                        out.append(cand)
                    cand += 1
                id_u32 = np.asarray(out, dtype=np.uint32)
        else:
            ids = np.asarray(ids, dtype=np.int64)
            if ids.shape != (n,):
                raise ValueError(f"ids length {ids.size} != vectors rows {n}")
            batch: set[int] = set()
            for i, v in enumerate(ids.tolist()):
                if not 0 <= v <= 0xFFFFFFFF:
                    raise ValueError(
                        f"ids[{i}] = {v} out of range [0, 2**32); pyvicinity stores IDs as u32 internally"
                    )
                if v in self._used_ids or v in batch or any(lo <= v < hi for lo, hi in self._id_ranges):
                    raise ValueError(f"duplicate doc_id {v} (IDs must be unique within an index)")
                batch.add(v)
            id_u32 = ids.astype(np.uint32)
        if n == 0:
            return
        _lib.check(self._lib.vg_ivfpq_add(self._h, _ptr(id_u32), _ptr(x), n))
        self._used_ids.update(id_u32.tolist())

    def add_device(self, x_ptr: int, n: int) -> None:
        """Add n rows [n][dim] f32 at address x_ptr (device or host memory)
        with the implicit sequential ids len(self) .. len(self) + n - 1, as
        add_items assigns them.  Rows generated on the GPU stay there: nothing
        passes through host memory but the ids."""
        base = len(self)
        if n <= 0:
            return
        if base + n - 1 > 0xFFFFFFFF:
            raise ValueError("implicit IDs exceed the u32 ID limit")
        if any(base <= u < base + n for u in self._used_ids):
            raise ValueError("implicit IDs collide with explicit ones; use add_items")
        ids = np.arange(base, base + n, dtype=np.uint32)
        _lib.check(self._lib.vg_ivfpq_add(self._h, _ptr(ids), x_ptr, n))
        self._id_ranges.append((base, base + n))

    def set_trained(self, centroids, codebooks, rotation=None) -> None:
        """Adopt coarse centroids [nc][dim] and PQ codebooks [M][ks][dsub]
        (and, for OPQ, the rotation [dim][dim])."""
        if rotation is not None:
            self.set_rotation(rotation)
        c = np.ascontiguousarray(centroids, dtype=np.float32)
        cb = np.ascontiguousarray(codebooks, dtype=np.float32)
        info = self.info()
        expect = info.num_codebooks * info.codebook_size * info.subvector_dim
        if cb.size != expect:
            raise ValueError(f"codebooks must hold {expect} floats, got {cb.size}")
        if c.ndim != 2 or c.shape[1] != self._dim:
            raise ValueError("centroids must be [num_centroids, dim]")
        _lib.check(self._lib.vg_ivfpq_set_trained(self._h, _ptr(c), c.shape[0], _ptr(cb)))

    def set_rotation(self, rotation) -> None:
        """OPQ rotation [dim][dim], row-major (opq.rs:31-41); None removes it."""
        if rotation is None:
            _lib.check(self._lib.vg_ivfpq_set_rotation(self._h, None))
            return
        r = np.ascontiguousarray(rotation, dtype=np.float32)
        if r.shape != (self._dim, self._dim):
            raise ValueError(f"rotation must be [{self._dim}, {self._dim}]")
        _lib.check(self._lib.vg_ivfpq_set_rotation(self._h, _ptr(r)))

    def build(self, training_sample_size: int | None = None, kmeans_max_iter: int = 100) -> None:
        """src/python.rs:622-637 (build_with_training_options)."""
        if training_sample_size is not None and training_sample_size == 0:
            raise ValueError("invalid config `training_sample_size`: must be greater than 0")
        _lib.check(self._lib.vg_ivfpq_build(self._h, training_sample_size or 0, kmeans_max_iter))

    def set_nprobe(self, nprobe: int) -> None:
        _lib.check(self._lib.vg_ivfpq_set_nprobe(self._h, nprobe))

    def set_stream(self, stream: int | None) -> None:
        """Run device work on a caller's cudaStream_t (None: the index's own)."""
        _lib.check(self._lib.vg_ivfpq_set_stream(self._h, stream or None))

    def set_coarse_tile_rows(self, rows: int) -> None:
        """Query rows per tile of the coarse stage (0: automatic); a tuning
        knob that leaves results unchanged."""
        _lib.check(self._lib.vg_ivfpq_set_coarse_tile_rows(self._h, int(rows)))

    def compact(self) -> None:
        if not self.info().built:
            raise ValueError("index must be built before compact")
        _lib.check(self._lib.vg_ivfpq_compact(self._h))

    # -- search --------------------------------------------------------------
    def _search_rows(self, q: np.ndarray, k: int, nprobe, rerank_pool):
        nq = q.shape[0]
        ids = np.empty((nq, k), dtype=np.uint32)
        dists = np.empty((nq, k), dtype=np.float32)
        counts = np.empty(nq, dtype=np.uint32)
        np_ = 0 if nprobe is None else int(nprobe)
        if nprobe is not None and np_ == 0:
            raise ValueError("nprobe must be greater than 0")
        if rerank_pool is None:
            st = self._lib.vg_ivfpq_search_batch(
                self._h, _ptr(q), nq, k, np_, _ptr(ids), _ptr(dists), _ptr(counts)
            )
        else:
            st = self._lib.vg_ivfpq_search_batch_reranked(
                self._h, _ptr(q), nq, k, int(rerank_pool), np_, _ptr(ids), _ptr(dists), _ptr(counts)
            )
        _lib.check(st)
        return ids, dists, counts

    # -- metadata filtering (search.rs:414-475, 1407-1549) ---------------------
    def add_metadata(self, doc_id: int, metadata: dict) -> None:
        """Attach metadata to a document: {field: int | float | str | bool};
        the filter field's value must be an int in 0..63."""
        body = json.dumps({str(k): _metadata_value(v) for k, v in metadata.items()})
        _lib.check(self._lib.vg_ivfpq_add_metadata(self._h, int(doc_id), body.encode()))

    def _filtered_rows(self, q: np.ndarray, k: int, field: str, value):
        nq = q.shape[0]
        ids = np.empty((nq, k), dtype=np.uint32)
        dists = np.empty((nq, k), dtype=np.float32)
        counts = np.empty(nq, dtype=np.uint32)
        _lib.check(self._lib.vg_ivfpq_search_filtered_batch(
            self._h, _ptr(q), nq, k, str(field).encode(), json.dumps(_metadata_value(value)).encode(),
            _ptr(ids), _ptr(dists), _ptr(counts)))
        return ids, dists, counts

    def search_with_filter(self, query, k: int, field: str, value):
        """Nearest documents with metadata `field == value` (an int category
        in 0..63): (doc ids int64, distances float32), ascending."""
        q = np.ascontiguousarray(query, dtype=np.float32)
        if q.ndim != 1 or q.shape[0] != self._dim:
            raise ValueError(f"query dimension mismatch: index expects {self._dim}")
        ids, dists, counts = self._filtered_rows(q.reshape(1, -1), k, field, value)
        c = int(counts[0])
        return ids[0, :c].astype(np.int64), dists[0, :c].copy()

    def batch_search_with_filter(self, queries, k: int, field: str, value):
        """search_with_filter over rows, padded like batch_search."""
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self._dim:
            raise ValueError(f"queries dimension mismatch: index expects {self._dim}")
        ids, dists, counts = self._filtered_rows(q, k, field, value)
        out = ids.astype(np.int64)
        out[np.arange(k)[None, :] >= counts.astype(np.int64)[:, None]] = MISSING_LABEL
        return out, dists

    def search(self, query, k: int, nprobe=None, rerank_pool=None):
        """src/python.rs:683-718: (ids int64, distances float32), ascending."""
        q = np.ascontiguousarray(query, dtype=np.float32)
        if q.ndim != 1 or q.shape[0] != self._dim:
            raise ValueError(
                f"query dimension mismatch: index expects {self._dim}, got {q.shape[-1] if q.ndim else 0}"
            )
        ids, dists, counts = self._search_rows(q.reshape(1, -1), k, nprobe, rerank_pool)
        c = int(counts[0])
        return ids[0, :c].astype(np.int64), dists[0, :c].copy()

    def batch_search(self, queries, k: int, nprobe=None, rerank_pool=None):
        """src/python.rs:720-795: [nq, k] arrays padded with MISSING_LABEL /
        MISSING_DISTANCE."""
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self._dim:
            raise ValueError(
                f"queries dimension mismatch: index expects {self._dim}, got {q.shape[-1] if q.ndim else 0}"
            )
        ids, dists, counts = self._search_rows(q, k, nprobe, rerank_pool)
        out = ids.astype(np.int64)
        out[np.arange(k)[None, :] >= counts.astype(np.int64)[:, None]] = MISSING_LABEL
        return out, dists

    def nearest_lists(self, queries, nprobe=None):
        """search.rs:1602-1617 (find_nearest_centroids) for each normalised
        query row: ([nq, p] list ids, [nq, p] distances 1 - q.c), nearest
        first, p = min(nprobe or the index default, number of centroids)."""
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self._dim:
            raise ValueError(
                f"queries dimension mismatch: index expects {self._dim}, got {q.shape[-1] if q.ndim else 0}"
            )
        np_ = 0 if nprobe is None else int(nprobe)
        if nprobe is not None and np_ == 0:
            raise ValueError("nprobe must be greater than 0")
        info = self.info()
        p = min(np_ or info.nprobe, info.num_centroids)
        lists = np.empty((q.shape[0], p), dtype=np.uint32)
        dists = np.empty((q.shape[0], p), dtype=np.float32)
        _lib.check(self._lib.vg_ivfpq_nearest_lists(self._h, _ptr(q), q.shape[0], np_, _ptr(lists), _ptr(dists)))
        return lists.astype(np.int64), dists

    def search_raw(self, q_ptr: int, nq: int, k: int, nprobe: int, ids_ptr: int, dist_ptr: int,
                   count_ptr: int = 0, rerank_pool: int = 0) -> None:
        """Search with caller-provided buffers (host or device addresses)."""
        if rerank_pool:
            st = self._lib.vg_ivfpq_search_batch_reranked(
                self._h, q_ptr, nq, k, rerank_pool, nprobe, ids_ptr, dist_ptr, count_ptr or None
            )
        else:
            st = self._lib.vg_ivfpq_search_batch(
                self._h, q_ptr, nq, k, nprobe, ids_ptr, dist_ptr, count_ptr or None
            )
        _lib.check(st)

    # -- state -----------------------------------------------------------------
    def info(self) -> _lib.VgInfo:
        info = _lib.VgInfo()
        _lib.check(self._lib.vg_ivfpq_get_info(self._h, C.byref(info)))
        return info

    def _export(self, what: int, dtype, shape) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        _lib.check(self._lib.vg_ivfpq_export(self._h, what, _ptr(out), out.nbytes))
        return out

    def centroids(self) -> np.ndarray:
        i = self.info()
        return self._export(_lib.EXPORT_CENTROIDS, np.float32, (i.num_centroids, i.dimension))

    def codebooks(self) -> np.ndarray:
        i = self.info()
        return self._export(
            _lib.EXPORT_CODEBOOKS, np.float32, (i.num_codebooks, i.codebook_size, i.subvector_dim)
        )

    def rotation(self) -> np.ndarray | None:
        """OPQ rotation [dim][dim] (None for plain PQ)."""
        try:
            return self._export(_lib.EXPORT_ROTATION, np.float32, (self._dim, self._dim))
        except ValueError:
            return None

    def assignments(self) -> np.ndarray:
        return self._export(_lib.EXPORT_ASSIGNMENTS, np.uint32, (len(self),))

    def codes(self) -> np.ndarray:
        i = self.info()
        return self._export(_lib.EXPORT_CODES, np.uint8, (len(self), i.num_codebooks))

    def list_offsets(self) -> np.ndarray:
        return self._export(_lib.EXPORT_LIST_OFFSETS, np.uint64, (self.info().num_centroids + 1,))

    def list_ids(self) -> np.ndarray:
        return self._export(_lib.EXPORT_LIST_IDS, np.uint32, (len(self),))

    def doc_ids(self) -> np.ndarray:
        return self._export(_lib.EXPORT_DOC_IDS, np.uint32, (len(self),))

    def vectors(self) -> np.ndarray:
        return self._export(_lib.EXPORT_VECTORS, np.float32, (len(self), self._dim))

    def reconstruct(self, idx: int) -> np.ndarray:
        out = np.empty(self._dim, dtype=np.float32)
        _lib.check(self._lib.vg_ivfpq_reconstruct(self._h, idx, _ptr(out)))
        return out

    # -- profiling ---------------------------------------------------------------
    def set_profiling(self, on: bool) -> None:
        _lib.check(self._lib.vg_ivfpq_set_profiling(self._h, int(bool(on))))

    def reset_profile(self) -> None:
        _lib.check(self._lib.vg_ivfpq_reset_profile(self._h))

    def profile(self) -> dict:
        p = _lib.VgProfile()
        _lib.check(self._lib.vg_ivfpq_get_profile(self._h, C.byref(p)))
        return {name: getattr(p, name) for name, _ in p._fields_}

    # -- sharding ----------------------------------------------------------------
    def shard(self, rank: int, world_size: int, nccl_id: bytes, timeout_ms: int = 60000) -> None:
        """Make this built index rank ``rank`` of a list-sharded group: the
        device keeps only this rank's inverted lists (greedy size-balanced
        packing).  Afterwards every rank searches batches of its own -- the
        same size on every rank, every search called on all ranks -- and gets
        the results of its own queries; the ranks exchange queries, probes,
        a pruning seed and per-rank top-k over NCCL."""
        if len(nccl_id) != 128:
            raise ValueError("nccl_id must be 128 bytes")
        buf = (C.c_uint8 * 128).from_buffer_copy(nccl_id)
        _lib.check(self._lib.vg_ivfpq_shard(self._h, rank, world_size, buf, timeout_ms))

    # -- getters (src/python.rs:797-846) ------------------------------------------
    @property
    def num_vectors(self) -> int:
        return self.info().num_vectors

    @property
    def dimension(self) -> int:
        return self._dim

    @property
    def num_clusters(self) -> int:
        return self.info().num_clusters

    @property
    def num_codebooks(self) -> int:
        return self.info().num_codebooks

    @property
    def codebook_size(self) -> int:
        return self.info().codebook_size

    @property
    def nprobe(self) -> int:
        return self.info().nprobe

    @property
    def use_opq(self) -> bool:
        return bool(self.info().use_opq)

    def __len__(self) -> int:
        return self.info().num_vectors

    def __repr__(self) -> str:
        i = self.info()
        return (
            f"IVFPQIndex(dim={i.dimension}, n={i.num_vectors}, num_clusters={i.num_clusters}, "
            f"num_codebooks={i.num_codebooks}, codebook_size={i.codebook_size}, nprobe={i.nprobe}, "
            f"use_opq={'True' if i.use_opq else 'False'})"
        )


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    _lib.check(_lib.load().vg_nccl_unique_id(buf))
    return bytes(buf)


def selftest_bounded_wait(limit_us: int = 20_000, device: int = 0) -> bool:
    """Run the tensor-core kernels' bounded-wait path on its own: a device
    wait of at most ``limit_us`` on a barrier nothing completes.  True when
    it expired and was reported through the device error flag."""
    out = C.c_int(0)
    _lib.check(_lib.load().vg_selftest_bounded_wait(device, limit_us, C.byref(out)))
    return bool(out.value)


def shard_assign_lists(sizes, world_size: int) -> np.ndarray:
    """Owner rank of every list (greedy size-balanced packing, host only)."""
    s = np.ascontiguousarray(sizes, dtype=np.uint64)
    out = np.empty(s.shape[0], dtype=np.int32)
    _lib.check(_lib.load().vg_shard_assign_lists(_ptr(s), s.shape[0], world_size, _ptr(out)))
    return out


def flat_search_ip(db, queries, k: int, device: int = 0):
    """Exact inner-product top-k (distance -dot, ascending): (ids int64 padded
    with MISSING_LABEL, distances float32)."""
    x = np.ascontiguousarray(db, dtype=np.float32)
    q = np.ascontiguousarray(queries, dtype=np.float32)
    if x.ndim != 2 or q.ndim != 2 or x.shape[1] != q.shape[1]:
        raise ValueError("db and queries must be 2-D with the same dimension")
    nq = q.shape[0]
    ids = np.empty((nq, k), dtype=np.uint32)
    dists = np.empty((nq, k), dtype=np.float32)
    counts = np.empty(nq, dtype=np.uint32)
    _lib.check(
        _lib.load().vg_flat_search_ip(
            _ptr(x), x.shape[0], _ptr(q), nq, x.shape[1], k, device, _ptr(ids), _ptr(dists), _ptr(counts)
        )
    )
    out = ids.astype(np.int64)
    out[np.arange(k)[None, :] >= counts.astype(np.int64)[:, None]] = MISSING_LABEL
    return out, dists


class FlatIndex:
    """Exhaustive inner-product index over f32 rows (vg_flat_create): the
    exact top-k by distance -dot (src/distance.rs:125-130), ascending, ties to
    the lower row -- the ground truth of src/benchmark/evaluation.rs:250-268.
    Host rows are copied to the device once; a device pointer (``from_device``)
    is used in place and must outlive the index."""

    def __init__(self, db=None, device: int = 0, *, _ptr_rows=None):
        self._lib = _lib.load()
        self._h = C.c_void_p()
        self.device = device
        if _ptr_rows is not None:
            ptr, n, d = _ptr_rows
            self._keep = None
        else:
            x = np.ascontiguousarray(db, dtype=np.float32)
            if x.ndim != 2:
                raise ValueError("db must be 2-D")
            ptr, (n, d) = _ptr(x), x.shape
            self._keep = x
        self.n, self.dim = int(n), int(d)
        _lib.check(self._lib.vg_flat_create(ptr, self.n, self.dim, device, C.byref(self._h)))
        self._keep = None  # host rows were copied

    @classmethod
    def from_device(cls, ptr: int, n: int, dim: int, device: int = 0) -> "FlatIndex":
        return cls(device=device, _ptr_rows=(ptr, n, dim))

    def close(self) -> None:
        if self._h:
            self._lib.vg_flat_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def search(self, queries, k: int):
        """(ids int64 padded with MISSING_LABEL, distances float32) of every query row."""
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self.dim:
            raise ValueError(f"queries must be 2-D with dimension {self.dim}")
        nq = q.shape[0]
        ids = np.empty((nq, k), dtype=np.uint32)
        dists = np.empty((nq, k), dtype=np.float32)
        counts = np.empty(nq, dtype=np.uint32)
        _lib.check(self._lib.vg_flat_search(self._h, _ptr(q), nq, k, None, _ptr(ids), _ptr(dists), _ptr(counts)))
        out = ids.astype(np.int64)
        out[np.arange(k)[None, :] >= counts.astype(np.int64)[:, None]] = MISSING_LABEL
        return out, dists

    def search_raw(self, q_ptr: int, nq: int, k: int, stream: int | None, ids_ptr: int, dist_ptr: int,
                   count_ptr: int | None) -> None:
        """vg_flat_search on raw host or device pointers, on a cudaStream_t handle."""
        _lib.check(self._lib.vg_flat_search(self._h, q_ptr, nq, k, stream or None, ids_ptr, dist_ptr,
                                            count_ptr or None))

    def set_profiling(self, on: bool) -> None:
        _lib.check(self._lib.vg_flat_set_profiling(self._h, 1 if on else 0))

    def profile(self) -> dict:
        p = _lib.VgProfile()
        _lib.check(self._lib.vg_flat_get_profile(self._h, C.byref(p)))
        return {name: getattr(p, name) for name, _ in p._fields_}


def current_generation(root) -> str:
    """The directory ``root/CURRENT`` names (persistence/generation.rs:191-205)."""
    lib = _lib.load()
    buf = C.create_string_buffer(4096)
    _lib.check(lib.vg_generation_current(os.fsencode(os.fspath(root)), buf, len(buf)))
    return os.fsdecode(buf.value)


def verify_generation(path) -> None:
    """Check every file of a generation against its GENERATION.json inventory
    (persistence/generation.rs:285-365): RuntimeError on any mismatch."""
    lib = _lib.load()
    _lib.check(lib.vg_verify_generation(os.fsencode(os.fspath(path))))


class IVFPQFileSearcher:
    """Search-only handle over a snapshot (IVFPQFileSearcher, search.rs:1620-1860;
    Python binding python.rs:857-1110).  The reference reads codes and raw
    vectors from the snapshot files through a block cache; here the snapshot
    is loaded into device memory once and searched there, with the same
    results."""

    def __init__(self, index: IVFPQIndex):
        self._ix = index

    @staticmethod
    def load(path, mmap=None, device: int = 0) -> "IVFPQFileSearcher":
        if mmap is not None:
            import warnings

            warnings.warn("IVFPQFileSearcher.load(mmap=...) is deprecated and ignored", DeprecationWarning,
                          stacklevel=2)
        return IVFPQFileSearcher(IVFPQIndex.load(path, device=device))

    @staticmethod
    def load_generation(path, device: int = 0) -> "IVFPQFileSearcher":
        return IVFPQFileSearcher(IVFPQIndex.load_generation(path, device=device))

    def set_nprobe(self, nprobe: int) -> None:
        self._ix.set_nprobe(nprobe)

    def search(self, query, k: int, nprobe=None, rerank_pool=None):
        return self._ix.search(query, k, nprobe=nprobe, rerank_pool=rerank_pool)

    def batch_search(self, queries, k: int, nprobe=None, rerank_pool=None):
        return self._ix.batch_search(queries, k, nprobe=nprobe, rerank_pool=rerank_pool)

    @property
    def num_vectors(self) -> int:
        return len(self._ix)

    @property
    def dimension(self) -> int:
        return int(self._ix.info().dimension)

    @property
    def num_clusters(self) -> int:
        return int(self._ix.info().num_centroids)

    @property
    def num_codebooks(self) -> int:
        return self._ix.num_codebooks

    @property
    def codebook_size(self) -> int:
        return self._ix.codebook_size

    @property
    def nprobe(self) -> int:
        return self._ix.nprobe

    def __len__(self) -> int:
        return self.num_vectors

    def __repr__(self) -> str:
        return (f"IVFPQFileSearcher(dim={self.dimension}, n={self.num_vectors}, num_clusters={self.num_clusters}, "
                f"num_codebooks={self.num_codebooks}, codebook_size={self.codebook_size}, nprobe={self.nprobe})")
