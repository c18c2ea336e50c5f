"""Build the sm_100a shared library in-tree: trifuse_b200/lib/libtrifuse_b200.so.

    python -m trifuse_b200.build [--force]

Each ``csrc/*.cu`` compiles to an object with
``-gencode arch=compute_100a,code=sm_100a`` in parallel, then one link.
Objects are rebuilt only when their source or a header is newer.
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
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = PKG / "_build"
LIB = LIB_DIR / "libtrifuse_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-O3", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and not shutil.which(cand):
        raise RuntimeError("nvcc not found; set NVCC")
    return cand


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, force: bool, extra: list[str]) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
            and obj.stat().st_mtime >= _deps_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if "-v" in extra:
        print(f"== {src.name}\n{r.stderr}", end="")
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force or ptxas_info, extra), sources))
    if (force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs)):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs),
               "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args(argv)
    build(force=a.force, verbose=True, ptxas_info=a.ptxas_info)


if __name__ == "__main__":
    sys.exit(main())
