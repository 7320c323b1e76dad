"""Build libfreeml_cuda.so (all CUDA sources under csrc/) for sm_100a, in-tree.

    python -m freeml_b200.build          # or: python freeml_b200/build.py

nvcc cross-compiles without a GPU; the .so lands next to this file so that it
travels with the source tree.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfreeml_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _needs(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _needs(obj, [src] + headers) or ptxas_info:
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            if verbose:
                print(" ".join(cmd))
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0 or (out and (verbose or ptxas_info)):
            sys.stdout.write(out)
        if p.returncode != 0:
            failed = True
            print(f"nvcc failed on {src}", file=sys.stderr)
    if failed:
        raise RuntimeError("CUDA build failed")
    if _needs(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-lcuda", "-lnccl"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return LIB


DROPIN_SRC = os.path.join(HERE, "dropin", "nanollm_dropin.cpp")
DROPIN_BIN = os.path.join(BUILD, "nanollm_dropin")


def freeml_root() -> str | None:
    """The FreeML source tree the drop-in example compiles against: the
    FREEML_ROOT environment variable, else a checkout named `reference` next
    to this repository.  None when neither holds FreeML (a machine that only
    runs the prebuilt binaries)."""
    env = os.environ.get("FREEML_ROOT")
    cands = [env] if env else [os.path.join(os.path.dirname(os.path.realpath(ROOT)), "reference")]
    for cand in cands:
        if cand and os.path.exists(os.path.join(cand, "ModelLibrary", "Model.h")):
            return cand
    if env:
        raise RuntimeError(f"FREEML_ROOT={env} does not hold a FreeML tree (ModelLibrary/Model.h is missing)")
    return None


def build_dropin(verbose: bool = False) -> str | None:
    """Compile the Model<float, MatrixCUDA<float>> example (needs the FreeML
    headers; skipped when the tree is absent, e.g. on a machine that only
    runs the prebuilt binary)."""
    root = freeml_root()
    if root is None:
        return None
    inc = os.path.join(ROOT, "include")
    deps = [DROPIN_SRC, LIB] + glob.glob(os.path.join(inc, "freeml_b200", "*.h")) + [os.path.join(inc, "freeml_cuda.h")]
    if _needs(DROPIN_BIN, deps):
        os.makedirs(BUILD, exist_ok=True)
        # -O3 -march=x86-64-v3: the flags the reference CPU build uses.  FreeML
        # draws its weights through libstdc++'s normal_distribution, which is
        # instantiated in this translation unit, and FMA contraction there
        # changes the last bit of the draws -- same flags, same weights.
        cmd = [os.environ.get("CXX", "g++"), "-std=c++20", "-O3", "-march=x86-64-v3", "-w",
               "-I" + os.path.join(inc, "freeml_b200", "gcc_compat"), "-I" + root, "-I" + inc,
               "-o", DROPIN_BIN, DROPIN_SRC, "-L" + HERE, "-lfreeml_cuda", "-Wl,-rpath,$ORIGIN/.."]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
    return DROPIN_BIN


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
    print(build_dropin(verbose="-v" in sys.argv))
