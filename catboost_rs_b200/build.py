"""Build libcbgpu.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m catboost_rs_b200.build

The shared library lands next to this file so it travels with the source tree;
no JIT cache is involved.  -fmad=false keeps every f64 operation separately
rounded (the reference's arithmetic); bit-exact paths also use explicit
round-to-nearest intrinsics.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libcbgpu.so")
SOURCES = ["kernels.cu", "session.cu", "noalloc.cu", "borders.cu", "apply.cu", "multi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def nccl_flags():
    inc = ["/usr/include"]
    libdirs = ["/usr/lib/x86_64-linux-gnu"]
    return [f"-I{d}" for d in inc if os.path.exists(os.path.join(d, "nccl.h"))], \
           [f"-L{d}" for d in libdirs] + ["-lnccl"]


def build(verbose: bool = False, force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "cbgpu.h"))
    if not force and os.path.exists(OUT):
        newest = max(os.path.getmtime(d) for d in deps)
        if os.path.getmtime(OUT) >= newest:
            return OUT
    inc, libs = nccl_flags()
    cmd = [nvcc_path(), "-std=c++17", "-O3", "-lineinfo", "-fmad=false", *ARCH,
           "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-ccbin", shutil.which("g++") or "g++",
           f"-I{os.path.join(os.path.dirname(HERE), 'include')}", *inc,
           "-o", OUT + ".tmp", *srcs, *libs, "-Xlinker", "-rpath=/usr/lib/x86_64-linux-gnu"]
    if verbose:
        cmd.insert(3, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force=True))
