"""Build libpim_b200.so (sm_100a) in place next to this file.

    python flagos-pim-compiler_b200/csrc/build.py [--verbose] [--ptxas]

Each .cu compiles to an object in ``_build/`` (parallel nvcc), then one shared
library is linked.  Objects are rebuilt only when a source or header changed.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
LIB = HERE / "libpim_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include"), "-I", str(HERE)]


def _sources() -> list[Path]:
    return sorted(HERE.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(HERE.glob("*.cuh")) + list(HERE.glob("*.h")) + list((ROOT / "include").glob("*.h")))


def build(verbose: bool = False, extra: list[str] | None = None, force: bool = False) -> Path:
    out = HERE / "_build"
    out.mkdir(exist_ok=True)
    newest_header = max((p.stat().st_mtime for p in _headers()), default=0)
    jobs = []
    for src in _sources():
        obj = out / (src.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            jobs.append((src, [NVCC, *ARCH, *FLAGS, *(extra or []), "-c", str(src), "-o", str(obj)]))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, flush=True)

    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(run, jobs))
    objs = [str(out / (s.stem + ".o")) for s in _sources()]
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(Path(o).stat().st_mtime for o in objs):
        r = subprocess.run([NVCC, *ARCH, "-shared", "-o", str(LIB), *objs, "-lcudart"], capture_output=True,
                           text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ptx = "--ptxas" in sys.argv
    print(build(verbose="--verbose" in sys.argv or ptx, extra=["-Xptxas", "-v"] if ptx else None, force=ptx))
