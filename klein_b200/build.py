"""Builds libklein_b200.so in-tree with nvcc for sm_100a (the only target).

    python -m klein_b200.build          # or klein_b200.build.build()

Objects go to klein_b200/_build/, the library to klein_b200/libklein_b200.so. The CUDA runtime is linked
statically and the driver API is reached through cudaGetDriverEntryPointByVersion, so the library loads
on a machine without a GPU driver (its symbols can be inspected there) and needs nothing but the driver
on a GPU machine.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libklein_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                     "-I" + os.path.join(HERE, "..", "include")]


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(HERE, "..", "include", "*.h"))
    newest_header = max((os.path.getmtime(h) for h in headers), default=0.0)
    jobs = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), newest_header):
            continue
        flags = list(NVCC_FLAGS)
        if ptxas_info and s.endswith(".cu"):
            flags += ["-Xptxas", "-v"]
        jobs.append([NVCC] + flags + ["-c", s, "-o", o])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for out in ex.map(_run, jobs):
            logs.append(out)
    if jobs or not os.path.exists(LIB):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-ldl", "-lpthread", "-lrt"])
    if verbose:
        for l in logs:
            if l.strip():
                print(l)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
    print(LIB)
