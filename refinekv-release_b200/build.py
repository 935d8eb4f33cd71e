"""Build ``refinekv_b200/_lib/librefinekv_b200.so`` in-tree with nvcc for sm_100a.

    python refinekv-release_b200/build.py [--force] [--jobs N]

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (in parallel),
then linked into one shared library that exports only the ``rkv_*`` C ABI of
``include/refinekv_b200.h``.  The CUDA runtime is linked statically and its
symbols are kept private, so the library coexists with the runtime that
PyTorch loads.  Targets only ``sm_100a`` (B200); nvcc cross-compiles it
without a GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"
LIB = HERE / "refinekv_b200" / "_lib" / "librefinekv_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not pathlib.Path(path).exists():
        raise RuntimeError("nvcc not found; install the CUDA 12.9 toolkit")
    return path


def _inputs():
    return sorted(CSRC.glob("*.cu")), sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        INCLUDE / "refinekv_b200.h", pathlib.Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    sources, headers = _inputs()
    newest = max(p.stat().st_mtime for p in sources + headers)
    return LIB.stat().st_mtime >= newest


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> pathlib.Path:
    """Compile and link the library unless it is newer than every source."""
    if not force and up_to_date():
        return LIB
    sources, _ = _inputs()
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    compiler = nvcc()

    def compile_one(src: pathlib.Path) -> pathlib.Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [compiler, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose:
            sys.stderr.write(res.stderr)
        return obj

    jobs = jobs or min(len(sources), os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as pool:
        objects = list(pool.map(compile_one, sources))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [compiler, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-Xlinker", "--exclude-libs,ALL",
           *map(str, objects), "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    main()
