"""Build step for the engine's shared library and the CPU oracle.

Compiles every ``csrc/*.cu`` for sm_100a with nvcc (in parallel) and links
``vicinity_b200/libvicinity_gpu.so`` against NCCL; the CUDA runtime is linked
statically so the library does not depend on which ``libcudart`` a host
process has already loaded.  Also runs ``make`` in ``oracle/`` (the checker
used by the tests and the benchmark's CPU leg).

Usage: ``python -m vicinity_b200.build [--force]``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libvicinity_gpu.so"
ORACLE_DIR = ROOT / "oracle"
ORACLE_LIB = ORACLE_DIR / "liboracle.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-Wall",
    f"-I{ROOT / 'include'}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the engine has no CPU build")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_engine(force: bool = False, jobs: int | None = None) -> Path:
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    todo = []
    objs = []
    for src in sources:
        obj = OBJ / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return src.name

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(compile_one, todo))
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lnccl", "-Xlinker", "--no-undefined"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def build_oracle(force: bool = False) -> Path:
    args = ["make", "-C", str(ORACLE_DIR)]
    if force:
        args.insert(1, "-B")
    res = subprocess.run(args, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    return ORACLE_LIB


def main(argv: list[str]) -> int:
    force = "--force" in argv
    print(build_engine(force))
    print(build_oracle(force))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
