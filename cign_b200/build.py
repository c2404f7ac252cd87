"""Build libcign_sm100.so (the C-ABI kernel library) in-tree for sm_100a.

    python -m cign_b200.build            # incremental
    python -m cign_b200.build --force    # rebuild everything

Every .cu under cign_b200/csrc is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` into an object
under cign_b200/_build/ (git-ignored), then linked into
cign_b200/libcign_sm100.so with the CUDA runtime linked statically, so the
library has no dependency on a particular libcudart in the process.
No GPU is needed to build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_DIR = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
INCLUDE_DIR = PKG_DIR.parent / "include"
LIB_PATH = PKG_DIR / "libcign_sm100.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE_DIR}",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")
    return cand


def _sources():
    return sorted(SRC_DIR.glob("*.cu"))


def _headers():
    return sorted(SRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool):
    cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if jobs:
        workers = max(1, min(len(jobs), os.cpu_count() or 1))
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose) for s, o in jobs]
            for f in futs:
                f.result()
    if force or jobs or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
