"""Build the sm_100a shared library in place: drama3_b200/libdrama3_b200.so.

    python comfyui-drama3_b200/build.py [--force]

nvcc cross-compiles for sm_100a on a machine without a GPU. The library is rebuilt when a source under csrc/ or the
public header is newer than it.
"""
import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = [HERE / "csrc" / "drama3_b200.cu", HERE / "csrc" / "pack.cpp"]
DEPENDS = sorted((HERE / "csrc").glob("*.c*")) + [ROOT / "include" / "drama3_b200.h"]
OUTPUT = HERE / "drama3_b200" / "libdrama3_b200.so"
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-shared", "-Xptxas", "-warn-spills", "-diag-suppress", "177,128"]


def nvcc():
    for candidate in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if candidate and (os.path.sep not in candidate or Path(candidate).exists()):
            return candidate
    raise RuntimeError("nvcc not found")


def stale():
    if not OUTPUT.exists():
        return True
    built = OUTPUT.stat().st_mtime
    return any(p.stat().st_mtime > built for p in DEPENDS)


def build(force=False, verbose=False):
    """Compile the library if it is missing or older than its sources; returns its path."""
    if not force and not stale():
        return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=HERE)
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True))
    sys.exit(0)
