"""Build libsemicrf.so (the sm_100a CUDA kernels behind include/semicrf.h) in-tree.

    python -m torch_semimarkov_b200.build_ext

nvcc cross-compiles for sm_100a without a GPU.  The shared library is written
next to this file so that it travels with the source tree.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libsemicrf.so")
# device-rate probes for bench.py's roofline denominators (not part of the scan)
PROBE_LIB = os.path.join(HERE, "libsemicrf_probe.so")
PROBE_SOURCES = ["probe.cu"]
SOURCES = ["api.cu", "chain.cu", "lchain.cu", "lchain_ws.cu", "lchain_fix.cu", "lchain_cl.cu", "lchunk.cu", "lmarg.cu", "marginals.cu", "viterbi.cu", "vchain.cu", "kcc.cu", "kblk.cu", "escan.cu", "gold.cu",
           "noalloc.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xptxas", "-warn-spills"]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(HERE, "..", "include", "semicrf.h"))
    return [h for h in hs if os.path.exists(h)]


def _newer(target: str, deps) -> bool:
    """True when target is missing or older than any of deps."""
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, jobs: int = 0) -> str:
    """Compile each stale object (its .cu or a shared header is newer), in
    parallel, then link the library when any object is newer than it."""
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = _headers()
    objs, todo = [], []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _newer(obj, [path, *headers]):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj + ".tmp"]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            todo.append((cmd, obj))
    jobs = jobs or max(1, min(len(todo), os.cpu_count() or 1))
    running = []
    failed = None
    for cmd, obj in todo:
        if verbose:
            print(" ".join(cmd), flush=True)
        running.append((subprocess.Popen(cmd), cmd, obj))
        while len(running) >= jobs:
            failed = _reap(running) or failed
    while running:
        failed = _reap(running) or failed
    if failed:
        raise subprocess.CalledProcessError(1, failed)
    if force or todo or _newer(LIB, objs):
        tmp = LIB + ".tmp"
        subprocess.run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"], check=True)
        os.replace(tmp, LIB)
    srcs = [os.path.join(CSRC, f) for f in PROBE_SOURCES]
    if force or _newer(PROBE_LIB, srcs):
        tmp = PROBE_LIB + ".tmp"
        subprocess.run([NVCC, *ARCH, *FLAGS, "-shared", "-o", tmp, *srcs, "-lcudart"],
                       check=True)
        os.replace(tmp, PROBE_LIB)
    return LIB


def _reap(running):
    """Wait for the oldest compile; returns its command when it failed."""
    proc, cmd, obj = running.pop(0)
    if proc.wait() != 0:
        return cmd
    os.replace(obj + ".tmp", obj)
    return None


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
