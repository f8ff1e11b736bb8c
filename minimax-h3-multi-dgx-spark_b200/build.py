"""Build libh3b.so (sm_100a only) in-tree.

    python minimax-h3-multi-dgx-spark_b200/build.py [--verbose]

Each csrc/*.cu is compiled by nvcc for `-gencode arch=compute_100a,code=sm_100a`
(SASS only, no PTX fallback) and the objects are linked into
h3b/libh3b.so with the CUDA runtime linked statically, so the library only
needs the GPU driver at run time and loads (without a GPU) for symbol checks.
The exported C ABI is declared in include/h3b.h at the repository root.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "h3b")
LIB = os.path.join(OUT_DIR, "libh3b.so")
OBJ_DIR = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-I", os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "h3b.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, force=False):
    os.makedirs(OBJ_DIR, exist_ok=True)
    objs = []
    hdrs = headers()
    for src in sources():
        obj = os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + hdrs):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB + ".tmp", *objs]
        subprocess.run(cmd, check=True)
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
