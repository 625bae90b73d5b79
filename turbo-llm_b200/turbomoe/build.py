"""Build libturbomoe.so in-tree with nvcc for sm_100a.

    python -m turbomoe.build            (from turbo-llm_b200/)
    python turbo-llm_b200/turbomoe/build.py [--trace]

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (skipped when the
object is newer than the source and every header), then linked into
``turbomoe/libturbomoe.so`` next to this file.  ``trace=True`` (``--trace``)
builds a debugging variant instead: every source compiled with -DTM_TRACE into
``_build/trace/`` and linked as ``turbomoe/libturbomoe_trace.so``; its kernels
record per-CTA (kernel, event, globaltimer, clock64) marks into a region of
the workspace whose layout ``tm_common.cuh`` documents (TM_TRACE).  The
product never loads it and ships no reader for the marks.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)               # turbo-llm_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG_DIR, "libturbomoe.so")
TRACE_LIB = os.path.join(PKG_DIR, "libturbomoe_trace.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I" + os.path.join(REPO, "include")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))


def _stale(obj, src, deps):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *deps])


def build(verbose: bool = False, ptxas_info: bool = False, jobs: int | None = None, trace: bool = False) -> str:
    out_dir = os.path.join(BUILD, "trace") if trace else BUILD
    lib_path = TRACE_LIB if trace else LIB
    defs = ["-DTM_TRACE"] if trace else []
    os.makedirs(out_dir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = _headers()
    cc = nvcc()
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(out_dir, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if _stale(o, s, deps) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            todo.append([cc, *ARCH, *NVCC_FLAGS, *defs, *extra, "-c", s, "-o", o])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        for cmd, r in ex.map(run, todo):
            if verbose or ptxas_info or r.returncode:
                sys.stdout.write(r.stdout)
                sys.stderr.write(r.stderr)
            if r.returncode:
                failed.append(cmd[-3])
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    if todo or not os.path.exists(lib_path) or any(os.path.getmtime(o) > os.path.getmtime(lib_path) for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", lib_path, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"link of {os.path.basename(lib_path)} failed")
    return lib_path


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="-v" in sys.argv, trace="--trace" in sys.argv))
