"""Build ``libconvrot_b200.so`` in-tree with nvcc for sm_100a.

    python -m convrot_mlx_b200.build [--force] [--jobs N]

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (in parallel),
then linked into ``convrot_mlx_b200/libconvrot_b200.so``.  A source newer than
the library (or a changed header) triggers a rebuild.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libconvrot_b200.so"
HEADERS = [ROOT / "include" / "convrot_b200.h", *sorted(CSRC.glob("*.cuh"))]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O2",
    "-I", str(ROOT / "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    sources = sorted(CSRC.glob("*.cu"))
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objects = []
    todo = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *HEADERS]):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return src.name

    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as pool:
            for name in pool.map(compile_one, todo):
                if verbose:
                    print(f"compiled {name}", flush=True)
    if force or todo or _stale(LIB, objects):
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB), *map(str, objects)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    sys.exit(main())
