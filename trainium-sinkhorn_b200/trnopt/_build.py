"""Build libtrnopt_cuda.so in-tree with nvcc for sm_100a (B200).

    python trainium-sinkhorn_b200/trnopt/_build.py     # or __graft_entry__.build()

Every .cu file under csrc/ is compiled to an object in parallel, then linked into one shared library with the CUDA
runtime linked statically (the library then needs only the driver at load time). Objects go to
trainium-sinkhorn_b200/_build/; the library lands next to this file, where trnopt._capi loads it from.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
PROJECT = PKG.parent
CSRC = PROJECT / "csrc"
BUILD = PROJECT / "_build"
LIB = PKG / "libtrnopt_cuda.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit's bin/ on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_v: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((PROJECT.parent / "include").glob("*.h"))
    cc = nvcc()
    jobs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_v:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for src, r in ex.map(run, jobs):
            if verbose or ptxas_v or r.returncode != 0:
                sys.stderr.write(f"--- {src.name}\n{r.stdout}{r.stderr}")
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}")
    objs = [BUILD / (s.stem + ".o") for s in sources()]
    if force or jobs or _stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc link failed")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_v="--ptxas-v" in sys.argv, force="--force" in sys.argv)
    print(LIB)
