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

Every output is rebuilt when the content hash of its inputs changes: the
sources, the headers, the compiler's version line and the exact command line
(flags included).  The hash sits in a ``.stamp`` file beside each output, so
a prebuilt tree whose stamps do not match the sources is rebuilt whatever
the files' mtimes say.  The kernel library also carries the hash of its
sources and flags in ``ks_build_info()`` ("src <hex>"), which
``source_hash()`` recomputes: a loaded library that reports another hash was
not built from these sources.
"""

from __future__ import annotations

import argparse
import glob
import hashlib
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


def _digest(parts) -> str:
    h = hashlib.sha256()
    for p in parts:
        h.update(p if isinstance(p, bytes) else str(p).encode())
        h.update(b"\0")
    return h.hexdigest()


def _file_digest(paths) -> str:
    parts = []
    for p in paths:
        parts.append(os.path.relpath(p, ROOT))
        with open(p, "rb") as fh:
            parts.append(fh.read())
    return _digest(parts)


_VERSIONS: dict = {}


def _tool_version(tool: str) -> str:
    if tool not in _VERSIONS:
        try:
            r = subprocess.run([tool, "--version"], capture_output=True, text=True)
            _VERSIONS[tool] = r.stdout.strip().splitlines()[-1] if r.stdout.strip() else tool
        except OSError:
            _VERSIONS[tool] = tool
    return _VERSIONS[tool]


def _stale(target: str, key: str) -> bool:
    """True unless `target` exists and its stamp records `key`."""
    stamp = target + ".stamp"
    if not os.path.exists(target) or not os.path.exists(stamp):
        return True
    with open(stamp) as fh:
        return fh.read().strip() != key


def _stamp(target: str, key: str) -> None:
    with open(target + ".stamp", "w") as fh:
        fh.write(key + "\n")


def _kernel_sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(INCLUDE, "kernscope_b200.h")]
    return srcs, hdrs


def _compile_flags():
    return [*GENCODE, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-rdc=false", "-I", INCLUDE,
            "-I", CSRC]


def source_hash() -> str:
    """Hash of the kernel library's sources, headers, nvcc flags and nvcc
    version: the value the library built from them reports in
    ``ks_build_info()``."""
    srcs, hdrs = _kernel_sources()
    return _digest([_file_digest(srcs + hdrs), " ".join(_compile_flags()), _tool_version(NVCC)])[:16]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build_kernels(jobs: int, force: bool, verbose_ptxas: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    srcs, hdrs = _kernel_sources()
    src_hash = source_hash()
    hdr_digest = _file_digest(hdrs)
    objs, keys, cmds = [], [], []
    for s in srcs:
        o = os.path.join(OBJDIR, os.path.basename(s) + ".o")
        cmd = [NVCC, *_compile_flags(), f"-DKS_SOURCE_HASH=\"{src_hash}\"", "-c", s, "-o", o]
        key = _digest([_file_digest([s]), hdr_digest, " ".join(cmd), _tool_version(NVCC)])
        objs.append(o)
        keys.append(key)
        if force or _stale(o, key):
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            cmds.append((cmd, o, key))
    log = []

    def one(job):
        cmd, o, key = job
        out = _run(cmd)
        _stamp(o, key)
        return out

    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for out in ex.map(one, cmds):
            log.append(out)
    link = [NVCC, *GENCODE, "-shared", "-cudart", "static", "-Xcompiler", "-fPIC", *objs, "-o", KERNEL_LIB, "-ldl",
            "-lpthread", "-lrt"]
    lkey = _digest([*keys, " ".join(link)])
    if force or cmds or _stale(KERNEL_LIB, lkey):
        _run(link)
        _stamp(KERNEL_LIB, lkey)
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
    hdr_digest = _file_digest(hdrs)
    with open(KERNEL_LIB + ".stamp") as fh:
        kernel_key = fh.read().strip()
    lib_cmd = [cxx, *common, "-shared", *lib_srcs, "-o", TUNE_LIB, "-L", LIBDIR, "-lkernscope_b200", rpath, "-ldl",
               "-lpthread"]
    lib_key = _digest([_file_digest(lib_srcs), hdr_digest, kernel_key, " ".join(lib_cmd), _tool_version(cxx)])
    if force or _stale(TUNE_LIB, lib_key):
        _run(lib_cmd)
        _stamp(TUNE_LIB, lib_key)
    for src, out in ((cli_src, TUNE_CLI), (bench_src, BENCH_CLI), (runner_src, RUNNER_CLI)):
        if not src:
            continue
        cmd = [cxx, *common, *src, "-o", out, "-L", LIBDIR, "-lkernscope_tune", "-lkernscope_b200", rpath, "-ldl",
               "-lpthread"]
        key = _digest([_file_digest(src), hdr_digest, lib_key, " ".join(cmd), _tool_version(cxx)])
        if force or _stale(out, key):
            _run(cmd)
            _stamp(out, key)


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
