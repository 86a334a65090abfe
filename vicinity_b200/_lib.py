"""ctypes binding of the engine's C ABI (include/vicinity_gpu.h).

The shared library is built in-tree by ``vicinity_b200.build``.  Loading fails
loudly when it is missing: there is no CPU implementation behind this API.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvicinity_gpu.so"

VG_OK = 0
VG_ERR_EMPTY_INDEX = -1
VG_ERR_INVALID_PARAMETER = -2
VG_ERR_INVALID_CONFIG = -3
VG_ERR_NOT_BUILT = -4
VG_ERR_ALREADY_BUILT = -5
VG_ERR_UNSUPPORTED = -6
VG_ERR_DIMENSION_MISMATCH = -7
VG_ERR_IO = -8
VG_ERR_FORMAT = -9
VG_ERR_CUDA = -10
VG_ERR_NCCL = -11
VG_ERR_OUT_OF_MEMORY = -12
VG_ERR_OTHER = -13
VG_ERR_NOT_FOUND = -14

EXPORT_CENTROIDS = 0
EXPORT_CODEBOOKS = 1
EXPORT_ASSIGNMENTS = 2
EXPORT_CODES = 3
EXPORT_LIST_OFFSETS = 4
EXPORT_LIST_IDS = 5
EXPORT_DOC_IDS = 6
EXPORT_VECTORS = 7
EXPORT_ROTATION = 8


class VgParams(C.Structure):
    _fields_ = [
        ("num_clusters", C.c_uint64),
        ("nprobe", C.c_uint64),
        ("num_codebooks", C.c_uint64),
        ("codebook_size", C.c_uint64),
        ("use_opq", C.c_int32),
        ("reserved", C.c_int32),
        ("seed", C.c_uint64),
    ]


class VgInfo(C.Structure):
    _fields_ = [
        ("dimension", C.c_uint64),
        ("num_vectors", C.c_uint64),
        ("num_clusters", C.c_uint64),
        ("num_centroids", C.c_uint64),
        ("nprobe", C.c_uint64),
        ("num_codebooks", C.c_uint64),
        ("codebook_size", C.c_uint64),
        ("subvector_dim", C.c_uint64),
        ("built", C.c_int32),
        ("trained", C.c_int32),
        ("compacted", C.c_int32),
        ("use_opq", C.c_int32),
        ("device", C.c_int32),
        ("shard_rank", C.c_int32),
        ("shard_world", C.c_int32),
        ("reserved", C.c_int32),
        ("device_bytes", C.c_uint64),
    ]


class VgProfile(C.Structure):
    _fields_ = [
        (name, C.c_double)
        for name in (
            "h2d_ms",
            "normalize_ms",
            "coarse_ms",
            "select_ms",
            "pairs_ms",
            "scan_ms",
            "merge_ms",
            "collective_ms",
            "d2h_ms",
            "total_ms",
        )
    ] + [
        (name, C.c_uint64)
        for name in (
            "calls",
            "queries",
            "probed_pairs",
            "scanned_vectors",
            "scanned_code_bytes",
            "kernel_launches",
            "scan_launches",
            "scored_lists",
            "scored_vectors",
            "tables_built",
            "code_groups",
            "seed_scored_lists",
            "seed_scored_vectors",
            "seed_tables_built",
            "seed_code_groups",
        )
    ]


_vp = C.c_void_p
_sz = C.c_size_t
_i = C.c_int

# name -> (restype, argtypes); every declaration of include/vicinity_gpu.h.
SIGNATURES = {
    "vg_last_error": (_i, [C.c_char_p, _sz]),
    "vg_version": (C.c_char_p, []),
    "vg_device_count": (_i, [C.POINTER(_i)]),
    "vg_selftest_bounded_wait": (_i, [_i, C.c_uint32, C.POINTER(_i)]),
    "vg_ivfpq_create": (_i, [_sz, C.POINTER(VgParams), _i, C.POINTER(_vp)]),
    "vg_ivfpq_destroy": (_i, [_vp]),
    "vg_ivfpq_add": (_i, [_vp, _vp, _vp, _sz]),
    "vg_ivfpq_set_trained": (_i, [_vp, _vp, _sz, _vp]),
    "vg_ivfpq_set_rotation": (_i, [_vp, _vp]),
    "vg_ivfpq_build": (_i, [_vp, _sz, _sz]),
    "vg_ivfpq_set_nprobe": (_i, [_vp, _sz]),
    "vg_ivfpq_set_stream": (_i, [_vp, _vp]),
    "vg_ivfpq_set_coarse_tile_rows": (_i, [_vp, _sz]),
    "vg_ivfpq_get_info": (_i, [_vp, C.POINTER(VgInfo)]),
    "vg_ivfpq_search_batch": (_i, [_vp, _vp, _sz, _sz, _sz, _vp, _vp, _vp]),
    "vg_ivfpq_search_batch_reranked": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, _vp]),
    "vg_ivfpq_nearest_lists": (_i, [_vp, _vp, _sz, _sz, _vp, _vp]),
    "vg_ivfpq_set_filter_field": (_i, [_vp, C.c_char_p]),
    "vg_ivfpq_add_metadata": (_i, [_vp, C.c_uint32, C.c_char_p]),
    "vg_ivfpq_search_filtered_batch": (_i, [_vp, _vp, _sz, _sz, C.c_char_p, C.c_char_p, _vp, _vp, _vp]),
    "vg_ivfpq_reconstruct": (_i, [_vp, _sz, _vp]),
    "vg_ivfpq_compact": (_i, [_vp]),
    "vg_ivfpq_export": (_i, [_vp, _i, _vp, _sz]),
    "vg_ivfpq_set_profiling": (_i, [_vp, _i]),
    "vg_ivfpq_get_profile": (_i, [_vp, C.POINTER(VgProfile)]),
    "vg_ivfpq_reset_profile": (_i, [_vp]),
    "vg_nccl_unique_id": (_i, [_vp]),
    "vg_ivfpq_shard": (_i, [_vp, _i, _i, _vp, _i]),
    "vg_shard_assign_lists": (_i, [_vp, _sz, _i, _vp]),
    "vg_flat_search_ip": (_i, [_vp, _sz, _vp, _sz, _sz, _sz, _i, _vp, _vp, _vp]),
    "vg_flat_create": (_i, [_vp, _sz, _sz, _i, C.POINTER(_vp)]),
    "vg_flat_destroy": (_i, [_vp]),
    "vg_flat_search": (_i, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp]),
    "vg_flat_set_profiling": (_i, [_vp, _i]),
    "vg_flat_get_profile": (_i, [_vp, C.POINTER(VgProfile)]),
    "vg_ivfpq_save": (_i, [_vp, C.c_char_p]),
    "vg_ivfpq_load": (_i, [C.c_char_p, _i, C.POINTER(_vp)]),
    "vg_ivfpq_save_generation": (_i, [_vp, C.c_char_p]),
    "vg_ivfpq_load_generation": (_i, [C.c_char_p, C.c_int, C.POINTER(_vp)]),
    "vg_generation_current": (_i, [C.c_char_p, C.c_char_p, _sz]),
    "vg_verify_generation": (_i, [C.c_char_p]),
    "vg_flat_search_ip_noalloc": (_i, [_vp, _sz, _vp, _sz, _sz, _sz, _i, _vp, _vp, _vp, _vp]),
}

_lib: C.CDLL | None = None


def _preload_torch_libs() -> None:
    """Load the NCCL and cuBLAS that PyTorch in this environment ships (the
    nvidia-nccl and nvidia-cublas wheels), when there are any, before the
    engine library.

    The engine links libnccl.so.2 and libcublas.so.12 by soname.  Were the
    system copies loaded first, a later `import torch` would bind to them as
    well (and fail on symbols only torch's newer NCCL exports) or load a
    second cuBLAS; with torch's copies loaded first both share them (NCCL and
    cuBLAS keep their C APIs backward compatible within a major version).
    """
    import importlib.util

    for pkg, names in (("nvidia.nccl", ("libnccl.so.2",)), ("nvidia.cublas", ("libcublasLt.so.12", "libcublas.so.12"))):
        try:
            spec = importlib.util.find_spec(pkg)
        except (ImportError, ValueError):
            continue
        for base in (spec.submodule_search_locations or []) if spec else []:
            paths = [Path(base) / "lib" / n for n in names]
            if all(path.exists() for path in paths):
                for path in paths:
                    C.CDLL(os.fspath(path), mode=C.RTLD_GLOBAL)
                break


def load() -> C.CDLL:
    """Load (once) and return the engine library with typed signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing; build it with `python -m vicinity_b200.build` "
            "(the engine has no CPU fallback)"
        )
    _preload_torch_libs()
    lib = C.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class VicinityError(Exception):
    """Engine failure that has no closer Python equivalent."""


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().vg_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    """Raise the Python exception a reference binding raises for `status`."""
    if status == VG_OK:
        return
    msg = last_error()
    if status == VG_ERR_NOT_FOUND:
        raise FileNotFoundError(msg)
    if status == VG_ERR_IO:
        raise OSError(msg)
    if status == VG_ERR_FORMAT:  # persistence format errors (python.rs:67-70)
        raise RuntimeError(msg)
    if status in (VG_ERR_CUDA, VG_ERR_NCCL, VG_ERR_OUT_OF_MEMORY):
        raise VicinityError(f"[{status}] {msg}")
    raise ValueError(msg)


def device_count() -> int:
    n = C.c_int(0)
    check(load().vg_device_count(C.byref(n)))
    return n.value
