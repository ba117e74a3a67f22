"""Build ``libdevproc_b200.so`` from the ``.cu`` sources in this folder.

Every source is compiled for sm_100a only (``-gencode arch=compute_100a,
code=sm_100a``) with relocatable device code, then device-linked into one
shared library next to the package.  nvcc cross-compiles, so this runs on a
machine without a GPU.  Objects are rebuilt only when a source or header is
newer than them.

Usage: python -m devproc_b200.csrc.build [--force] [--jobs N]
"""

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
INCLUDE = ROOT / "include"
OBJ_DIR = PKG / "_build"
LIB = PKG / "libdevproc_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
                     f"-I{INCLUDE}", f"-I{HERE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def _sources():
    return sorted(HERE.glob("*.cu"))


def _headers():
    return sorted(list(HERE.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    headers = _headers()
    todo = [s for s in _sources() if force or _stale(OBJ_DIR / (s.stem + ".o"), [s, *headers])]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
            list(ex.map(lambda s: _compile(s, verbose_ptxas), todo))
    objs = [OBJ_DIR / (s.stem + ".o") for s in _sources()]
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objs),
               "-o", str(LIB), "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--ptxas-v", action="store_true", help="print register / spill / smem usage")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.ptxas_v))
