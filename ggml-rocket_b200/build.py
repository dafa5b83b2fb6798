"""Build libggml-b200.so (CUDA kernels for sm_100a + the C++ backend layer) in-tree.

    python ggml-rocket_b200/build.py            # incremental
    python ggml-rocket_b200/build.py --clean
    GGML_DIR=/path/to/llama.cpp python ggml-rocket_b200/build.py   # + the ggml plugin

Every .cu under csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a), every .cpp by g++; the objects go to _build/ and
the shared library to lib/. No GPU is needed to build.
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libggml-b200.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INCLUDES = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nccl_include():
    try:
        import nvidia.nccl  # noqa: F401  (torch's bundled NCCL)
        base = os.path.dirname(nvidia.nccl.__file__)
        inc = os.path.join(base, "include")
        lib = os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return None, None


def run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def newer(src, dst, deps):
    if not os.path.exists(dst):
        return True
    t = os.path.getmtime(dst)
    return any(os.path.getmtime(p) > t for p in [src] + deps)


def build(verbose_ptxas=False, jobs=8):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    objs, cmds = [], []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if newer(src, obj, headers):
            cmd = [NVCC] + ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                                   "--expt-relaxed-constexpr"] + INCLUDES + ["-c", src, "-o", obj]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            cmds.append(cmd)
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cpp"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if newer(src, obj, headers):
            cmds.append(["g++", "-O2", "-std=c++20", "-fPIC", "-Wall", "-Wextra", "-I" + os.path.join(CUDA_HOME, "include")]
                        + INCLUDES + ["-c", src, "-o", obj])
    # compile in parallel
    procs = []
    for cmd in cmds:
        print(" ".join(cmd), flush=True)
        procs.append(subprocess.Popen(cmd))
        if len(procs) >= jobs:
            if procs.pop(0).wait() != 0:
                raise SystemExit("compile failed")
    for p in procs:
        if p.wait() != 0:
            raise SystemExit("compile failed")
    stale = not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs)
    if cmds or stale:
        link = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        run(link)
    return LIB


def build_plugin(ggml_dir, ggml_lib=None):
    """The ggml plugin (csrc/ggml/ggml-b200-plugin.cpp -> lib/libggml-b200-plugin.so), compiled against a
    host's ggml: ggml_dir is a llama.cpp or ggml checkout (its ggml/include and ggml/src, where the private
    ggml-backend-impl.h lives), ggml_lib the directory holding libggml-base.so (default: its build/bin).
    The plugin links libggml-b200.so beside it; a host loads it with GGML_BACKEND_PATH or
    ggml_backend_load."""
    lib = build()
    root = ggml_dir
    inc = [os.path.join(root, "ggml", "include"), os.path.join(root, "ggml", "src"), os.path.join(root, "include"),
           os.path.join(root, "src")]
    inc = [d for d in inc if os.path.isdir(d)]
    if not any(os.path.exists(os.path.join(d, "ggml-backend-impl.h")) for d in inc):
        raise SystemExit(f"{ggml_dir}: no ggml-backend-impl.h under ggml/src or src")
    ggml_lib = ggml_lib or os.path.join(root, "build", "bin")
    out = os.path.join(LIBDIR, "libggml-b200-plugin.so")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-I" + os.path.join(CUDA_HOME, "include")] + \
        INCLUDES + ["-I" + d for d in inc] + [os.path.join(CSRC, "ggml", "ggml-b200-plugin.cpp"), "-o", out,
                                             "-L" + LIBDIR, "-lggml-b200", "-L" + ggml_lib, "-lggml-base",
                                             "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart",
                                             "-Wl,-rpath,$ORIGIN"]
    run(cmd)
    return out


def clean():
    for d in (BUILD, LIBDIR):
        if os.path.isdir(d):
            shutil.rmtree(d)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", action="store_true", help="ptxas -v")
    ap.add_argument("--ggml", default=os.environ.get("GGML_DIR"),
                    help="also build the ggml plugin against this llama.cpp / ggml checkout (default: $GGML_DIR)")
    ap.add_argument("--ggml-lib", default=os.environ.get("GGML_LIB_DIR"), help="directory of libggml-base.so")
    a = ap.parse_args()
    if a.clean:
        clean()
    ok = build(verbose_ptxas=a.v)
    if a.ggml:
        build_plugin(a.ggml, a.ggml_lib)
    sys.exit(0 if ok else 1)
