"""Builds the engine library pyodide-llm_b200/b200fwd/libb200fwd.so for sm_100a, in-tree (the built library travels
with the repository to the GPU boxes; it is git-ignored).

    python pyodide-llm_b200/build.py [--force] [-v]

nvcc compiles every csrc/*.cu with -gencode arch=compute_100a,code=sm_100a and --fmad=false (the exact kernels round
every multiply and add on its own, as the reference's WASM does), and links them with the CUDA runtime.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "b200fwd" / "libb200fwd.so"
BUILD = HERE / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default",
         "--expt-relaxed-constexpr"]


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "b200fwd.h"]


def stale():
    if not OUT.exists():
        return True
    built = OUT.stat().st_mtime
    return any(p.stat().st_mtime > built for p in sources() + headers() + [Path(__file__)])


def build(force=False, verbose=False):
    if not force and not stale():
        return OUT
    BUILD.mkdir(exist_ok=True)

    def compile_one(src):
        obj = BUILD / (src.stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-I", str(HERE.parent / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, sources()))
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
