"""Build libmoeb200.so in-tree with nvcc for sm_100a (no JIT cache, no pip install).

    python moe-offload-lab_b200/moeb200/build.py [--force]

Objects go to moe-offload-lab_b200/_build/, the shared library next to this file, so the built
library travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG.parent / "csrc"
INC = PKG.parent.parent / "include"
BUILD = PKG.parent / "_build"
LIB = PKG / "libmoeb200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-DNDEBUG"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the moeb200 CUDA library cannot be built")


def _deps() -> list[Path]:
    return sorted(SRC.glob("*.cu")) + sorted(SRC.glob("*.cuh")) + sorted(INC.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu to an object and link libmoeb200.so. Returns the library path."""
    BUILD.mkdir(exist_ok=True)
    headers = sorted(SRC.glob("*.cuh")) + sorted(INC.glob("*.h"))
    cc = nvcc()
    jobs = []
    for cu in sorted(SRC.glob("*.cu")):
        obj = BUILD / (cu.stem + ".o")
        if force or _stale(obj, [cu] + headers):
            jobs.append([cc, *ARCH, *FLAGS, f"-I{INC}", "-c", str(cu), "-o", str(obj)])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    objs = [str(BUILD / (cu.stem + ".o")) for cu in sorted(SRC.glob("*.cu"))]
    if force or jobs or _stale(LIB, [Path(o) for o in objs]):
        tmp = LIB.with_suffix(".so.tmp")
        run([cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs, "-lcudart_static", "-lrt",
             "-lpthread", "-ldl"])
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
