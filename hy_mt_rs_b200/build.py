"""Build libhyq.so (the C-ABI CUDA library) in-tree for sm_100a.

    python hy_mt_rs_b200/build.py [--force] [-v]

(run it by path: importing the package loads the library it builds)

Each csrc/*.cu is compiled with nvcc for sm_100a only and linked into
hy_mt_rs_b200/lib/libhyq.so.  Objects go to hy_mt_rs_b200/_build/.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libhyq.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-I" + INCLUDE, "-I" + CSRC]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr}")
    return obj, res.stderr


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    todo = [s for s in srcs
            if force or _stale(os.path.join(BUILD, os.path.basename(s) + ".o"), [s, *hdrs])]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
                logs.append(log)
    objs = [os.path.join(BUILD, os.path.basename(s) + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
        subprocess.check_call(cmd)
        os.replace(tmp, LIB)
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
