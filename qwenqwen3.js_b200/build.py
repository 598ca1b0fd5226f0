"""Build the native parts of the package in-tree.

* ``libqq3cuda.so``  -- the sm_100a CUDA backend behind include/qq3.h (nvcc, cross-compiles
  without a GPU);
* ``libqq3synth.so`` -- the seeded synthetic-weight generator (gcc + OpenMP).

Both land next to this file so that they travel with the repository snapshot.
"""
from __future__ import annotations

import concurrent.futures as _cf
import glob
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
CUDA_LIB = PKG_DIR / "libqq3cuda.so"
SYNTH_LIB = PKG_DIR / "libqq3synth.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
                           f"-I{REPO_DIR / 'include'}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libqq3cuda.so")


def _gomp() -> str:
    cands = sorted(glob.glob("/usr/lib/gcc/x86_64-linux-gnu/*/libgomp.so")) + ["/usr/lib/x86_64-linux-gnu/libgomp.so.1"]
    for c in cands:
        if Path(c).exists():
            return c
    raise RuntimeError("libgomp not found")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_cuda(force: bool = False) -> Path:
    cus = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO_DIR / "include" / "qq3.h"]
    if not force and not _stale(CUDA_LIB, cus + headers):
        return CUDA_LIB
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    jobs = []
    with _cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cu in cus:
            obj = BUILD_DIR / (cu.stem + ".o")
            objs.append(obj)
            if force or _stale(obj, [cu] + headers):
                jobs.append(ex.submit(_run, [nvcc, *NVCC_FLAGS, "-c", str(cu), "-o", str(obj)]))
        for j in jobs:
            j.result()
    tmp = CUDA_LIB.with_suffix(".so.tmp")
    _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)])
    os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_synth(force: bool = False) -> Path:
    src = CSRC / "synth.c"
    if not force and not _stale(SYNTH_LIB, [src]):
        return SYNTH_LIB
    BUILD_DIR.mkdir(exist_ok=True)
    cc = shutil.which("gcc") or "gcc"
    obj = BUILD_DIR / "synth.o"
    _run([cc, "-O2", "-fPIC", "-fopenmp", "-std=c11", "-c", str(src), "-o", str(obj)])
    tmp = SYNTH_LIB.with_suffix(".so.tmp")
    _run([cc, "-shared", "-o", str(tmp), str(obj), _gomp(), "-lm"])
    os.replace(tmp, SYNTH_LIB)
    return SYNTH_LIB


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_cuda(force)


if __name__ == "__main__":
    build_all(force=True)
    print(CUDA_LIB, SYNTH_LIB)
