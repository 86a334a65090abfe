"""Generation snapshots (persistence/generation.rs, search.rs:916-943):
root/generations/<id>/ directories with a GENERATION.json inventory (length
and CRC-32 of every file, paths sorted) and a root/CURRENT pointer.  The
inventory's CRC-32 is pinned to zlib's (the same IEEE polynomial); the
resolution and verification rules follow generation.rs:191-205, 285-365.
"""
from __future__ import annotations

import json
import os
import zlib
from pathlib import Path

import numpy as np
import pytest

from oracle import snapshot as osnap
from vicinity_b200 import IVFPQFileSearcher, IVFPQIndex, current_generation, verify_generation
from vicinity_b200.synthetic import mixture


def _inventory(gen: Path) -> dict:
    files = []
    for path in sorted(p for p in gen.rglob("*") if p.is_file() and p.name != "GENERATION.json"):
        data = path.read_bytes()
        files.append({"path": path.relative_to(gen).as_posix(), "length": len(data), "crc32": zlib.crc32(data)})
    files.sort(key=lambda f: f["path"])
    return {"version": 1, "files": files}


def _hand_made(root: Path, gid: str = "g1") -> Path:
    gen = root / "generations" / gid
    (gen / "sub").mkdir(parents=True)
    (gen / "a.bin").write_bytes(bytes(range(256)) * 3)
    (gen / "sub" / "b.bin").write_bytes(b"vicinity")
    (gen / "GENERATION.json").write_text(json.dumps(_inventory(gen), indent=2))
    (root / "CURRENT").write_text(gid + "\n")
    return gen


# ---- host only --------------------------------------------------------------

def test_current_and_verify_accept_a_consistent_generation(tmp_path):
    gen = _hand_made(tmp_path)
    assert Path(current_generation(tmp_path)) == gen
    verify_generation(gen)


@pytest.mark.parametrize("damage", ["byte", "extra", "missing", "unsorted", "no_inventory"])
def test_verify_rejects_damage(tmp_path, damage):
    gen = _hand_made(tmp_path)
    if damage == "byte":
        data = bytearray((gen / "a.bin").read_bytes())
        data[5] ^= 1
        (gen / "a.bin").write_bytes(bytes(data))
    elif damage == "extra":
        (gen / "c.bin").write_bytes(b"x")
    elif damage == "missing":
        (gen / "sub" / "b.bin").unlink()
    elif damage == "unsorted":
        inv = json.loads((gen / "GENERATION.json").read_text())
        inv["files"].reverse()
        (gen / "GENERATION.json").write_text(json.dumps(inv))
    else:
        (gen / "GENERATION.json").unlink()
    with pytest.raises(RuntimeError):
        verify_generation(gen)


def test_current_rejects_unsafe_pointers(tmp_path):
    with pytest.raises(FileNotFoundError):
        current_generation(tmp_path)
    _hand_made(tmp_path)
    (tmp_path / "CURRENT").write_text("../elsewhere\n")
    with pytest.raises(RuntimeError, match="safe generation basename"):
        current_generation(tmp_path)
    os.symlink(tmp_path / "generations" / "g1", tmp_path / "generations" / "link")
    (tmp_path / "CURRENT").write_text("link")
    with pytest.raises(RuntimeError, match="not a directory"):
        current_generation(tmp_path)


# ---- GPU --------------------------------------------------------------------

@pytest.mark.gpu
def test_save_and_load_generations(tmp_path):
    # search.rs:2740-2785: two publications; CURRENT moves, the first stays
    x, q = mixture(3000, 32, 20, 0.3, seed=31, nq=20)
    ix = IVFPQIndex(32, num_clusters=16, num_codebooks=8, codebook_size=256, nprobe=4, seed=5)
    ix.add_items(x)
    ix.build(kmeans_max_iter=4)
    before = ix.batch_search(q, 5)
    root = tmp_path / "root"
    ix.save_generation(root)
    first = (root / "CURRENT").read_text().strip()
    gen = Path(current_generation(root))
    assert gen == root / "generations" / first
    man = json.loads((gen / "manifest.json").read_text())
    assert man["generation_components"] == ["centroids.bin", "clusters.bin", "codes.bin", "doc_ids.bin",
                                            "list_codes.bin", "list_offsets.bin", "raw_vectors.bin"]
    assert json.loads((gen / "GENERATION.json").read_text()) == _inventory(gen)
    verify_generation(gen)
    assert osnap.read_snapshot(gen)["manifest"]["num_vectors"] == 3000  # the independent reader agrees
    loaded = IVFPQIndex.load_generation(root)
    after = loaded.batch_search(q, 5)
    assert np.array_equal(before[0], after[0]) and np.array_equal(before[1].view(np.uint32), after[1].view(np.uint32))
    searcher = IVFPQFileSearcher.load_generation(root)
    ids, dists = searcher.search(q[0], 5)
    assert np.array_equal(ids, before[0][0]) and len(searcher) == 3000 and searcher.num_clusters == 16
    assert "IVFPQFileSearcher(dim=32, n=3000" in repr(searcher)
    ix.save_generation(root)
    second = (root / "CURRENT").read_text().strip()
    assert second != first and (root / "generations" / first).is_dir()
    assert not [p for p in (root / "generations").iterdir() if p.name.startswith(".staging-")]
    # a plain directory snapshot still loads, without a component inventory
    ix.save(tmp_path / "flat")
    assert "generation_components" not in json.loads((tmp_path / "flat" / "manifest.json").read_text())
    flat = IVFPQFileSearcher.load(tmp_path / "flat")
    assert np.array_equal(flat.batch_search(q, 5)[0], before[0])
