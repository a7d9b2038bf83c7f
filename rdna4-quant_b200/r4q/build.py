"""Build ``libr4q.so`` (all of csrc/*.cu) in-tree with nvcc for sm_100a.

    python -m r4q.build        (from the rdna4-quant_b200 folder)

Objects go to ``_build/``; the shared library lands next to the Python
modules so that it travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
CSRC = PKG / "csrc"
OUT = PKG / "libr4q.so"
BUILD = PKG / "_build"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path, headers) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    nvcc = _nvcc()
    jobs = []
    objs = []
    for s in sources():
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, s, headers):
            jobs.append([nvcc, *ARCH, *FLAGS, "-c", str(s), "-o", str(o)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(run, jobs))
    if jobs or force or not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        run([nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"])
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
