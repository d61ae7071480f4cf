"""TEST INFRASTRUCTURE: builds the oracle (oracle.cpp, a C++ restatement of the reference's CPU path) into
oracle/liboracle.so. Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline load it.

    python oracle/build_oracle.py [--native]

-ffp-contract=off keeps every multiply and add rounded on its own, as WASM's f32 operations are. x86-64-v2 keeps
the library runnable on any x86-64 host the GPU boxes have (the build runs in one container, the tests in another).
--native builds oracle/_native/liboracle.so for the CPU it is built on (-march=native), on the host that runs it:
the timed CPU baseline. The numbers are the same (no contraction, no reassociation either way).
"""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "liboracle.so"


NATIVE = HERE / "_native" / "liboracle.so"


def build(verbose=False, native=False):
    src = HERE / "oracle.cpp"
    out = NATIVE if native else OUT
    newest = max(src.stat().st_mtime, (HERE.parent / "include" / "b200fwd.h").stat().st_mtime)
    if out.exists() and out.stat().st_mtime >= newest and not native:
        return out
    out.parent.mkdir(exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-march=native" if native else "-march=x86-64-v2", "-pthread", str(src), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(out)
    return out


def cpu_model():
    """the host CPU's model name (/proc/cpuinfo), for the baseline's line"""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


if __name__ == "__main__":
    build(verbose=True, native="--native" in sys.argv)
    sys.exit(0)
