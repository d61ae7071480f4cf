"""TEST INFRASTRUCTURE: builds the oracle (oracle.cpp, a C++ restatement of the reference's CPU path) into
oracle/liboracle.so. Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline load it.

    python oracle/build_oracle.py

-ffp-contract=off keeps every multiply and add rounded on its own, as WASM's f32 operations are. x86-64-v2 keeps
the library runnable on any x86-64 host the GPU boxes have (the build runs in one container, the tests in another).
"""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "liboracle.so"


def build(verbose=False):
    src = HERE / "oracle.cpp"
    if OUT.exists() and OUT.stat().st_mtime >= max(src.stat().st_mtime, (HERE.parent / "include" / "b200fwd.h").stat().st_mtime):
        return OUT
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-march=x86-64-v2", "-pthread", str(src), "-o", str(OUT)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
