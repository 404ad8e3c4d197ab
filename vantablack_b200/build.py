"""Builds the backend's shared library, in-tree, for sm_100a.

``python -m vantablack_b200.build`` (or ``__graft_entry__.build()``) runs
nvcc on csrc/libvtbcuda.cu and writes vantablack_b200/libvtbcuda.so.  The
library links only the CUDA runtime (and NCCL for tensor parallelism); it
has no PyTorch dependency.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libvtbcuda.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    """NCCL headers and library: the copy PyTorch ships (same library torch
    loads in-process), else the system one."""
    try:
        import nvidia.nccl as n
        base = list(n.__path__)[0]
        if os.path.exists(os.path.join(base, "include", "nccl.h")):
            return os.path.join(base, "include"), os.path.join(base, "lib")
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h")))


def up_to_date() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(os.path.join(HERE, "libvtbbridgeloop.so")):
        return False
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(ROOT, "include", "vtb_cuda.h"), os.path.join(HERE, "native", "bridge_loop.c")]
    return all(os.path.getmtime(s) <= t for s in deps if os.path.exists(s))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-shared", "-o", LIB + ".tmp",
           os.path.join(CSRC, "libvtbcuda.cu"), "-lcudart"]
    inc, libdir = nccl_dirs()
    cmd += ["-I" + inc, "-L" + libdir, "-l:libnccl.so.2", "-Xlinker", "-rpath," + libdir]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    build_bridge_loop()
    return LIB


BRIDGE_LOOP = os.path.join(HERE, "libvtbbridgeloop.so")


def build_bridge_loop() -> str:
    """native/bridge_loop.c: a compiled caller of the C ABI (bench.py's
    end-to-end measurement), linked against libvtbcuda.so."""
    src = os.path.join(HERE, "native", "bridge_loop.c")
    subprocess.run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-o", BRIDGE_LOOP, src,
                    "-L" + HERE, "-l:libvtbcuda.so", "-Wl,-rpath,$ORIGIN"], check=True)
    return BRIDGE_LOOP


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
