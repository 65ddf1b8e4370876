"""Build ``libpack3d_b200.so`` in-tree from ``csrc/*.cu`` with nvcc for sm_100a.

    python -m pack3d_b200.build            # incremental
    python -m pack3d_b200.build --force    # rebuild everything

Objects go to ``pack3d_b200/_build/`` and the library to ``pack3d_b200/lib/``.
nvcc cross-compiles, so this runs on machines without a GPU.
"""
import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libpack3d_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE)]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build pack3d_b200")
    return exe


def _headers():
    return [*SRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(source, obj, verbose):
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    run = subprocess.run(cmd, capture_output=True, text=True)
    if run.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{run.stderr}")
    return run.stderr


def build(force=False, verbose=False, jobs=None):
    """Compile every CUDA source for sm_100a and link the shared library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(SRC.glob("*.cu"))
    headers = _headers()
    todo = []
    objects = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            todo.append((src, obj))
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        logs = list(pool.map(lambda so: (so[0].name, _compile(so[0], so[1], verbose)), todo))
    if verbose:
        for name, log in logs:
            print(f"== {name}\n{log}")
    if force or todo or _stale(LIB, objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objects)]
        run = subprocess.run(cmd, capture_output=True, text=True)
        if run.returncode != 0:
            raise RuntimeError(f"link failed:\n{run.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    sys.exit(0)
