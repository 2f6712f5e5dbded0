"""Build recipe for libqi8.so (in-tree, sm_100a only).

``python -m convert_to_quant_quip_int8_b200.build`` compiles every ``csrc/*.cu``
with nvcc for ``-gencode arch=compute_100a,code=sm_100a`` into
``convert_to_quant_quip_int8_b200/libqi8.so``.  No fast-math: the kernels rely
on IEEE division, reciprocal and round-half-even for bit-exact parity.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libqi8.so")
BUILD_DIR = os.path.join(PKG, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-std=c++17", "-O3", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(objs_and_srcs, lib) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(os.path.dirname(PKG), "include", "qi8.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile libqi8.so if any source is newer than it; returns its path."""
    srcs = sources()
    if not force and not _stale(srcs, LIB):
        return LIB
    nvcc = nvcc_path()
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    headers.append(os.path.join(os.path.dirname(PKG), "include", "qi8.h"))
    newest_header = max(os.path.getmtime(h) for h in headers if os.path.exists(h))
    for src in srcs:
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        # an object newer than its source and every shared header is current
        if (not force and not ptxas_verbose and os.path.exists(obj)
                and os.path.getmtime(obj) > max(os.path.getmtime(src), newest_header)):
            objs.append(obj)
            continue
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", os.path.join(os.path.dirname(PKG), "include"),
               "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
           *objs, "-ldl", "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv))
