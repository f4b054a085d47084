"""Builds libiron_b200.so from iron_b200/csrc/*.cu with nvcc for sm_100a.

The library is built in-tree (iron_b200/libiron_b200.so) so that it travels with
the source tree; there is no JIT cache. Each .cu compiles to an object under
iron_b200/_build/ in parallel, then one shared library is linked. Objects are
rebuilt when their source or any header under csrc/ or include/ is newer.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libiron_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
    f"-I{INCLUDE}",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile_one(nvcc: str, src: Path, obj: Path) -> str:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    # ptxas -v resource lines, kept for inspection
    (obj.with_suffix(".ptxas.txt")).write_text(res.stderr)
    return src.name


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel source for sm_100a and link libiron_b200.so."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    hdr_time = _newest(_headers())
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_time):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile_one, nvcc, s, o) for s, o in jobs]
            for f in futs:
                name = f.result()
                if verbose:
                    print(f"[iron_b200] compiled {name}")
    if force or jobs or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < _newest(objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
        if verbose:
            print(f"[iron_b200] linked {LIB_PATH}")
    return LIB_PATH


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv, verbose=True)
