"""Build libspo_cuda.so in-tree for sm_100a (B200) with nvcc.

Every .cu under csrc/ is compiled to an object in parallel, then linked into
spo_mojo_b200/libspo_cuda.so with the CUDA runtime linked statically and NCCL
(the pip-installed nvidia-nccl-cu12 that torch also loads) found through an rpath.

    python -m spo_mojo_b200.build          # incremental
    python -m spo_mojo_b200.build --force  # rebuild everything
    python -m spo_mojo_b200.build --trace  # libspo_cuda_trace.so: the small step's phase trace
"""

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
LIB = os.path.join(HERE, "libspo_cuda.so")
# the same library with the one-launch small step's phase marks compiled in
TRACE_BUILD = os.path.join(HERE, "_build_trace")
TRACE_LIB = os.path.join(HERE, "libspo_cuda_trace.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-Xcompiler", "-Wall,-Wextra",
          "--expt-relaxed-constexpr"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def nccl_dir():
    try:
        import nvidia.nccl as n  # noqa: F401
        base = list(n.__path__)[0]
        if os.path.exists(os.path.join(base, "include", "nccl.h")):
            return base
    except Exception:
        pass
    raise RuntimeError("NCCL headers (nvidia-nccl-cu12) not found")


def _deps_newer(obj, src):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, trace=False):
    BUILD, LIB = (TRACE_BUILD, TRACE_LIB) if trace else (globals()["BUILD"], globals()["LIB"])
    flags = CFLAGS + (["-DSPO_SMALL_TRACE"] if trace else [])
    os.makedirs(BUILD, exist_ok=True)
    nv = nvcc()
    nccl = nccl_dir()
    inc = ["-I" + os.path.join(nccl, "include"), "-I" + os.path.join(ROOT, "include")]
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if force or _deps_newer(obj, src):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [nv] + ARCH + flags + inc + ["-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r

    failed = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            for src, r in ex.map(compile_one, jobs):
                if r.returncode != 0:
                    failed.append((src, r.stderr))
                elif verbose:
                    sys.stderr.write(r.stderr)
    if failed:
        for src, err in failed:
            sys.stderr.write(f"--- {src}\n{err}\n")
        raise RuntimeError("nvcc failed for " + ", ".join(os.path.basename(s) for s, _ in failed))
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or not os.path.exists(LIB) or any(
            os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        ncl = os.path.join(nccl, "lib")
        cmd = [nv] + ARCH + ["-shared", "-o", LIB] + objs + [
            "-L" + ncl, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + ncl, "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, trace=a.trace))
