"""Build recipe of the engine library (``libnitro_engine.so``), compiled in-tree for
sm_100a with nvcc so that the shared object travels with the source tree."""
from __future__ import annotations

import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libnitro_engine.so")
SERVER = os.path.join(PKG, "nitro_server")        # the inference server process
SERVER_SRC = os.path.join(PKG, "nitro_server.cc")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-Wall",
    "-shared",
]


def sources() -> list[str]:
    csrc = os.path.join(PKG, "csrc")
    return sorted(glob.glob(os.path.join(csrc, "*.cu")) + glob.glob(os.path.join(csrc, "*.cpp")))


def headers() -> list[str]:
    csrc = os.path.join(PKG, "csrc")
    return sorted(glob.glob(os.path.join(csrc, "*.h")) + glob.glob(os.path.join(csrc, "*.cuh"))
                  + glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in sources() + headers())


def build(force: bool = False, verbose: bool = False) -> str:
    nvcc = os.environ.get("NVCC", "nvcc")
    if force or not up_to_date():
        cmd = [nvcc, *NVCC_FLAGS, "-o", LIB, *sources()]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True, cwd=ROOT)
    if force or not os.path.exists(SERVER) or os.path.getmtime(SERVER) < max(
            os.path.getmtime(LIB), os.path.getmtime(SERVER_SRC)):
        # host-only executable linked against the library, found next to it at run time
        cmd = [os.environ.get("CXX_HOST", "g++"), "-O2", "-std=c++17", "-Wall", "-o", SERVER, SERVER_SRC,
               "-L", PKG, "-lnitro_engine", "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True, cwd=ROOT)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
