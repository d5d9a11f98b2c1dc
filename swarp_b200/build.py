"""Build the sm_100a shared library ``swarp_b200/libswarp_b200.so`` in-tree with nvcc.

``python -m swarp_b200.build`` (or ``__graft_entry__.build()``). Rebuilds only when a
source is newer than the library. The library is a plain C ABI (include/swarp_b200.h)
linked against the CUDA runtime; Python loads it with ctypes.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libswarp_b200.so")
SOURCES = ["capi.cu", "noalloc.cu", "k_fwd_f32.cu", "k_fwd_f64.cu", "k_bwd_f32.cu",
           "k_bwd_f64.cu", "k_fwd_f32_rk4.cu", "k_fwd_f64_rk4.cu", "k_bwd_f32_rk4.cu",
           "k_bwd_f64_rk4.cu", "k_x2_f32.cu", "k_fwd_f32_box.cu", "k_fwd_f64_box.cu",
           "k_bwd_f32_box.cu", "k_bwd_f64_box.cu", "k_fwd_f32_drone.cu", "k_fwd_f64_drone.cu",
           "k_bwd_f32_drone.cu", "k_bwd_f64_drone.cu", "k_cl_fwd_f32.cu", "k_cl_fwd_f64.cu",
           "k_cl_bwd_f32.cu", "k_cl_bwd_f64.cu"]
# headers every translation unit includes, and those only some include
COMMON_HEADERS = ["launch.cuh", "rollout.cuh", "physics.cuh", "bodies.cuh", "boxes.cuh",
                  "boxes_vjp.cuh", "drone.cuh"]
EXTRA_HEADERS = {"k_x2_f32.cu": ["rollout_x2.cuh"], "capi.cu": ["rollout_cluster.cuh"],
                 **{f"k_cl_{d}_{t}.cu": ["k_cl.cuh", "rollout_cluster.cuh"]
                    for d in ("fwd", "bwd") for t in ("f32", "f64")}}
DEPS = [*SOURCES, *COMMON_HEADERS, "rollout_x2.cuh", "k_cl.cuh", "rollout_cluster.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -ftz=true: float32 arithmetic flushes subnormal inputs and results to zero (float64 is
# unaffected); every float kernel is built the same way, so the kernels that must agree bit
# for bit (forward and adjoint recomputation, paired and one-agent, cluster and one-CTA)
# still do
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--extended-lambda", "-fmad=false", "-ftz=true",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"]
LINK = ["--shared", "-cudart", "shared"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build swarp_b200")
    return cand


def _stale(lib: str, deps: list[str]) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    hdr = os.path.join(ROOT, "include", "swarp_b200.h")
    # this file holds the compiler flags: a change to it rebuilds everything
    return any(os.path.getmtime(p) > t for p in [*deps, hdr, os.path.abspath(__file__)])


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    deps = [os.path.join(CSRC, d) for d in DEPS]
    if not force and not _stale(LIB, deps):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs, procs = [], []
    # a translation unit is rebuilt when it, a common header or one of its own headers
    # changed (or when forced or given extra flags)
    headers = [os.path.join(CSRC, d) for d in COMMON_HEADERS]
    headers.append(os.path.join(ROOT, "include", "swarp_b200.h"))
    headers.append(os.path.abspath(__file__))
    newest_hdr = max(os.path.getmtime(h) for h in headers)
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        path = os.path.join(CSRC, src)
        own = [os.path.getmtime(os.path.join(CSRC, h)) for h in EXTRA_HEADERS.get(src, [])]
        if (not force and not extra and os.path.exists(obj)
                and os.path.getmtime(obj) > max(newest_hdr, os.path.getmtime(path), *own)):
            continue
        cmd = [nvcc(), *ARCH, *FLAGS, *(extra or []), "-c", "-o", obj, path]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append(subprocess.Popen(cmd))
    failed = [p.args[-1] for p in procs if p.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed on {failed}")
    cmd = [nvcc(), *ARCH, *LINK, "-o", LIB + ".tmp", *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None))
