"""Builds libltx_b200.so (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python ltx-rust_b200/build.py [--force] [--jobs N]

Objects go to ltx-rust_b200/_build/, the library to
ltx-rust_b200/ltx_b200/libltx_b200.so (git-ignored, shipped with the tree).
nvcc cross-compiles here without a GPU.  cudart is linked statically so the
library does not depend on which CUDA runtime the host process loaded.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "ltx_b200", "libltx_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
                     "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]
CXX_FLAGS = ["-O3", "-std=c++17", "-ffp-contract=off", "-fPIC", "-Wall", "-Wextra", "-I" + os.path.join(CUDA, "include"),
             "-I" + os.path.join(ROOT, "include")]


def headers_mtime():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0)


def compile_one(src, force, extra):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest_input = max(os.path.getmtime(src), headers_mtime(), os.path.getmtime(__file__))
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest_input:
        return obj, None
    if src.endswith(".cu"):
        cmd = [NVCC] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    else:
        cmd = [os.environ.get("CXX", "g++")] + CXX_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    if extra and r.stderr:
        print(r.stderr, end="")   # -Xptxas -v: registers, spills, shared memory
    return obj, None


def build(force=False, jobs=8, verbose_ptxas=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    objs, errors = [], []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, err in ex.map(lambda s: compile_one(s, force, extra), srcs):
            objs.append(obj)
            if err:
                errors.append(err)
    if errors:
        raise RuntimeError("build failed:\n" + "\n".join(errors))
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(o) for o in objs):
        return OUT
    cmd = [NVCC] + ARCH + ["-shared", "-o", OUT] + objs + ["-cudart", "static", "-lrt", "-lpthread", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    try:
        print(build(a.force, a.jobs, a.ptxas_v))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
