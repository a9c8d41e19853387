"""Builds libqlin.so (sm_100a) in-tree: mac-kernels-public_b200/qlin/libqlin.so.

    python mac-kernels-public_b200/build.py [--jobs N] [--verbose] [--checks]

--checks builds the same library with -DQLIN_CHECKS (bounds checks on every plain global access
and computed shared-memory index, recorded and read back with qlin_bounds_check) as
qlin/libqlin_checked.so, from objects in _build/checks/; select it with QLIN_LIB.

Each csrc/*.cu is compiled with nvcc for `-gencode arch=compute_100a,code=sm_100a` into
_build/, then linked into one shared library with the CUDA runtime linked statically, so the
library does not depend on which libcudart the host process (PyTorch) loaded.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "qlin", "libqlin.so")
OUT_CHECKED = os.path.join(HERE, "qlin", "libqlin_checked.so")
BUILD = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-v" if os.environ.get("QLIN_PTXAS_V") else "-O3"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def compile_one(src, verbose=False, checks=False):
    obj = os.path.join(BUILD, "checks" if checks else "", os.path.basename(src) + ".o")
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(HERE, "..", "include", "qlin.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, *(["-DQLIN_CHECKS"] if checks else []), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr) if verbose else ""


def build(jobs=None, verbose=False, checks=False):
    out = OUT_CHECKED if checks else OUT
    os.makedirs(os.path.join(BUILD, "checks") if checks else BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose, checks), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log)
    newest = max(os.path.getmtime(o) for o in objs)
    if not os.path.exists(out) or os.path.getmtime(out) < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", out, *objs, "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--checks", action="store_true")
    a = ap.parse_args()
    try:
        print(build(a.jobs, a.verbose, a.checks))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
