"""Builds libdtts.so in this folder from csrc/ (nvcc for sm_100a + g++).

    python build.py            # incremental
    python build.py --clean    # from scratch

Objects go to _build/ beside this file; the shared library lands next to
this file so it travels with the repository snapshot.  cudart is linked
statically; the driver API is reached through cudaGetDriverEntryPoint, so no
libcuda link is needed at build time."""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "libdtts.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
# the system g++ (an alternative toolchain earlier on PATH may lack pieces)
CXX = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-ccbin", CXX,
                     "-Xptxas", "-warn-spills", "-I" + os.path.join(HERE, "..", "include")]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function", "-I" + os.path.join(CUDA, "include"),
             "-I" + os.path.join(HERE, "..", "include")]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(HERE, "..", "include", "*.h"))


def _stale(obj, src, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in [src] + deps)


def _compile(src):
    base = os.path.splitext(os.path.basename(src))[0]
    obj = os.path.join(BUILD, base + ".o")
    if src.endswith(".cu"):
        cmd = [NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj]
    else:
        cmd = [CXX] + CXX_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    spills = [l for l in r.stderr.splitlines() if "spill" in l.lower() and " 0 bytes" not in l]
    return obj, spills


def build(clean: bool = False, verbose: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    deps = _headers()
    todo = [s for s in srcs if _stale(os.path.join(BUILD, os.path.splitext(os.path.basename(s))[0] + ".o"), s, deps)]
    objs = [os.path.join(BUILD, os.path.splitext(os.path.basename(s))[0] + ".o") for s in srcs]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, spills in ex.map(_compile, todo):
                if verbose:
                    print("built", os.path.basename(obj))
                for s in spills:
                    print("warning:", s, file=sys.stderr)
    if todo or not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-ccbin", CXX, "-o", OUT] + objs + ["-cudart", "static", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    a = ap.parse_args()
    print(build(clean=a.clean, verbose=True))
