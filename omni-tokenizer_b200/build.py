"""Build the sm_100a shared libraries of this package in-tree.

    python omni-tokenizer_b200/build.py          # builds libomni_b200.so

Every CUDA source under csrc/ is compiled by nvcc for
`-gencode arch=compute_100a,code=sm_100a` (B200 only) into object files under
_build/, then linked into omni-tokenizer_b200/libomni_b200.so.  The CUDA
runtime is linked statically and the driver's cuTensorMapEncodeTiled is looked
up at run time, so the library loads on machines without a GPU driver.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libomni_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    objs = []
    jobs = []
    for src in _sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers + [Path(__file__)]):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [nvcc()] + ARCH + FLAGS + ["-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
        if verbose:
            print(r.stderr, end="")
        return src.name

    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for name in ex.map(compile_one, jobs):
                if verbose:
                    print("compiled", name)
    if force or jobs or _stale(LIB, objs):
        # cuBLAS (the encoder graphs' linears) is linked dynamically from the CUDA
        # toolkit the library was built with.
        cuda_lib = Path(nvcc()).resolve().parent.parent / "lib64"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + [
            "-L", str(cuda_lib), "-lcublas", "-lcublasLt", "-Xlinker", f"-rpath={cuda_lib}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
