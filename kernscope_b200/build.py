"""Build the in-tree native libraries for sm_100a.

    python -m kernscope_b200.build [--jobs N] [--force]

* ``kernscope_b200/lib/libkernscope_b200.so`` -- the CUDA kernels and their
  C ABI (``include/kernscope_b200.h``), compiled with
  ``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and the CUDA
  runtime linked statically (no dependency on the toolkit being installed
  where the library is loaded).
* ``kernscope_b200/lib/libkernscope_tune.so`` and
  ``kernscope_b200/lib/kernscope-tune`` -- the C++20 tuner (config spaces,
  pre-screen, arch/occupancy/roofline models, bench, db + tunecache, driver,
  CLI), linked against the kernel library;
* ``kernscope_b200/lib/kernscope-bench`` -- the roofline peak measurement
  CLI (HBM, bf16 tensor, fp32, shared memory);
* ``kernscope_b200/lib/ks-template-runner`` -- runs one kernel on raw host
  buffers (the gate runner of the reference's template flow).

Objects are rebuilt only when a source or header is newer than the object.
"""

from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(ROOT, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]

KERNEL_LIB = os.path.join(LIBDIR, "libkernscope_b200.so")
TUNE_LIB = os.path.join(LIBDIR, "libkernscope_tune.so")
TUNE_CLI = os.path.join(LIBDIR, "kernscope-tune")
BENCH_CLI = os.path.join(LIBDIR, "kernscope-bench")
RUNNER_CLI = os.path.join(LIBDIR, "ks-template-runner")


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build_kernels(jobs: int, force: bool, verbose_ptxas: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(INCLUDE, "kernscope_b200.h")]
    objs = []
    cmds = []
    for s in srcs:
        o = os.path.join(OBJDIR, os.path.basename(s) + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            cmd = [NVCC, *GENCODE, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-rdc=false", "-I", INCLUDE, "-I", CSRC, "-c", s, "-o", o]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            cmds.append(cmd)
    log = []
    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for out in ex.map(_run, cmds):
            log.append(out)
    if force or cmds or _newer(KERNEL_LIB, objs):
        _run([NVCC, *GENCODE, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", *objs,
              "-o", KERNEL_LIB, "-ldl", "-lpthread", "-lrt"])
    return "\n".join(log)


def build_tuner(force: bool) -> None:
    srcs = sorted(glob.glob(os.path.join(HOST, "*.cpp")))
    if not srcs:
        return
    hdrs = sorted(glob.glob(os.path.join(HOST, "*.h"))) + [os.path.join(INCLUDE, "kernscope_b200.h")]
    clis = ("tune_cli.cpp", "bench_cli.cpp", "runner_cli.cpp")
    lib_srcs = [s for s in srcs if not s.endswith(clis)]
    cli_src = [s for s in srcs if s.endswith("tune_cli.cpp")]
    bench_src = [s for s in srcs if s.endswith("bench_cli.cpp")]
    runner_src = [s for s in srcs if s.endswith("runner_cli.cpp")]
    # The system g++ (nvcc's host compiler): both libraries must share one
    # dynamic libstdc++ (a toolchain that links libstdc++ statically would put
    # a second copy in the process next to the one the kernel library uses).
    cxx = os.environ.get("KS_CXX", "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++")
    common = ["-std=c++20", "-O2", "-fPIC", "-Wall", "-I", INCLUDE, "-I", HOST]
    rpath = "-Wl,-rpath,$ORIGIN"
    if force or _newer(TUNE_LIB, lib_srcs + hdrs + [KERNEL_LIB]):
        _run([cxx, *common, "-shared", *lib_srcs, "-o", TUNE_LIB, "-L", LIBDIR, "-lkernscope_b200",
              rpath, "-ldl", "-lpthread"])
    for src, out in ((cli_src, TUNE_CLI), (bench_src, BENCH_CLI), (runner_src, RUNNER_CLI)):
        if src and (force or _newer(out, src + hdrs + [TUNE_LIB])):
            _run([cxx, *common, *src, "-o", out, "-L", LIBDIR, "-lkernscope_tune", "-lkernscope_b200",
                  rpath, "-ldl", "-lpthread"])


def build(jobs: int = 8, force: bool = False, verbose_ptxas: bool = False) -> str:
    log = build_kernels(jobs, force, verbose_ptxas)
    build_tuner(force)
    return log


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    p.add_argument("--force", action="store_true")
    p.add_argument("--ptxas-v", action="store_true", help="print registers/spills/smem per kernel")
    a = p.parse_args()
    log = build(a.jobs, a.force, a.ptxas_v)
    if a.ptxas_v:
        print(log)
    print(KERNEL_LIB)
    return 0


if __name__ == "__main__":
    sys.exit(main())
