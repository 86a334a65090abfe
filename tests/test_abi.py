"""The C-ABI library loads, exports every declared entry point, and its
host-only logic (validation, list sharding) behaves -- no GPU needed."""
from __future__ import annotations

import ctypes as C
import re
import subprocess

import numpy as np
import pytest

from tests.conftest import ROOT
from vicinity_b200 import _lib
from vicinity_b200.ivf_pq import IVFPQIndex, default_ivfpq_codebooks, shard_assign_lists

HEADER = ROOT / "include" / "vicinity_gpu.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(vg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), f"{name} declared in vicinity_gpu.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (vg_[a-z0-9_]+)", out.stdout))
    assert set(names) <= exported


def test_torch_imports_after_the_engine_library():
    # both link libnccl.so.2 by soname; loading the engine first must not pin
    # an NCCL that torch cannot use
    code = "from vicinity_b200 import _lib; _lib.load(); import torch; print('ok')"
    out = subprocess.run(["python", "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]


def test_version_string():
    assert b"sm_100a" in _lib.load().vg_version()


def test_create_rejects_bad_shapes_before_touching_a_device():
    lib = _lib.load()
    h = C.c_void_p()
    bad = [
        (0, dict(num_clusters=4, nprobe=1, num_codebooks=2, codebook_size=16), _lib.VG_ERR_INVALID_CONFIG),
        (8, dict(num_clusters=4, nprobe=1, num_codebooks=3, codebook_size=16), _lib.VG_ERR_INVALID_CONFIG),
        (8, dict(num_clusters=4, nprobe=1, num_codebooks=2, codebook_size=257), _lib.VG_ERR_INVALID_CONFIG),
    ]
    for dim, kw, code in bad:
        p = _lib.VgParams(use_opq=0, reserved=0, seed=42, **kw)
        assert lib.vg_ivfpq_create(dim, C.byref(p), 0, C.byref(h)) == code
        assert _lib.last_error()


def test_create_without_a_device_fails_loudly():
    if _lib.device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(_lib.VicinityError, match="no CPU path"):
        IVFPQIndex(dim=8, num_clusters=8, num_codebooks=4, codebook_size=8)


def test_python_binding_validation_mirrors_reference():
    # src/python.rs:1152-1179
    with pytest.raises(ValueError, match="dim must be greater than 0"):
        IVFPQIndex(dim=0)
    with pytest.raises(ValueError, match="num_codebooks must be a non-zero divisor"):
        IVFPQIndex(dim=8, num_codebooks=3)
    with pytest.raises(ValueError, match="codebook_size must be in the range"):
        IVFPQIndex(dim=8, num_codebooks=2, codebook_size=257)
    with pytest.raises(ValueError, match="nprobe must be greater than 0"):
        IVFPQIndex(dim=8, num_codebooks=2, nprobe=0)
    with pytest.raises(ValueError, match="num_clusters must be greater than 0"):
        IVFPQIndex(dim=8, num_clusters=0)


def test_default_codebooks(kats):
    kat = kats["default_codebooks"]
    assert default_ivfpq_codebooks(kat["dim"]) == kat["expected"]
    assert default_ivfpq_codebooks(96) == 8 and default_ivfpq_codebooks(7) == 7


def test_shard_assignment_is_balanced_and_deterministic():
    rng = np.random.default_rng(0)
    sizes = rng.integers(0, 2000, size=4096).astype(np.uint64)
    for world in (1, 2, 4, 8):
        owner = shard_assign_lists(sizes, world)
        assert owner.min() >= 0 and owner.max() < world
        assert np.array_equal(owner, shard_assign_lists(sizes, world))
        loads = np.bincount(owner, weights=sizes.astype(np.float64), minlength=world)
        # greedy largest-first packing: spread bounded by the largest list
        assert loads.max() - loads.min() <= sizes.max()
    # ties: equal sizes go round-robin by list id
    assert shard_assign_lists(np.ones(6, np.uint64), 3).tolist() == [0, 1, 2, 0, 1, 2]
