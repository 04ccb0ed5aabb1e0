"""Test infrastructure: build the reference generator's own CUDA kernels.

For every config of the reference tuner's bounded "auto" grid at the
benchmark shapes, `oracle/_ref/ref_tune_check gen` (the reference generator
API: validate_config, launch_geometry, kernel_symbol, generate_to_file)
writes the kernel source, and nvcc compiles it with `ref_launch.cu` into one
small shared library per config under `oracle/_ref/kernels/`. The index
`oracle/_ref/kernels/index.json` records each config's geometry, its library
or the reason it was rejected (by the reference validator, or by nvcc: the
reference kernels keep their tiles in static shared memory, which CUDA caps
at 48 KB).

Only `bench.py --impl reference` and the GPU tests load these libraries, to
time the reference's kernels on the same GPU beside this repository's.

    python oracle/ref_tune/build_ref_kernels.py <reference checkout> [-j N]

The auto grids follow the reference driver's enumerate() functions:
matmul tools/tune/src/driver_matmul.cpp:98-114, flash_attention
tools/tune/src/driver_flash.cpp:81-94, softmax and layernorm
tools/tune/src/driver_elem.cpp:185-196 and :259-270, bias_gelu
tools/tune/src/driver_elem.cpp:107-116.
"""

from __future__ import annotations

import argparse
import itertools
import json
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(ROOT, "oracle", "_ref", "kernels")
CHECK = os.path.join(ROOT, "oracle", "_ref", "ref_tune_check")
ARCH = "sm_100"  # the reference arch table's Blackwell row

# benchmark shapes (BASELINE configs C2-C5), in each generator's shape convention
SHAPES = {
    "matmul": [8192, 8192, 8192],           # M, N, K
    "flash_attention": [8192, 8192, 128],   # Nq, Nk, d: one (batch, head) slice
    "softmax": [4096, 8192],                # rows, cols
    "layernorm": [16384, 4096],
    "bias_gelu": [16384, 16384],
}


def auto_grid(family: str) -> list[dict]:
    if family == "matmul":
        return [dict(tile_m=bm, tile_n=bn, tile_k=bk, warps=w, stages=st, vec_width=1, smem_layout="padding", unroll=1)
                for (bm, bn), bk, w, st in itertools.product([(64, 64), (128, 128)], [16, 32], [1, 2, 4], [1, 2])]
    if family == "flash_attention":
        return [dict(tile_m=br, tile_n=bc, stages=st, vec_width=v, smem_layout="padding", causal=1)
                for br, bc, st, v in itertools.product([32, 64], [32, 64], [1, 2], [1, 2, 4])]
    if family in ("softmax", "layernorm"):
        return [dict(block=b, vec_width=v, mode=m)
                for b, v, m in itertools.product([128, 256, 512, 1024], [1, 2, 4], ["onepass", "twopass"])]
    if family == "bias_gelu":
        return [dict(block=b, vec_width=v) for b, v in itertools.product([128, 256, 512, 1024], [1, 2, 4])]
    raise ValueError(family)


def build_one(ref: str, family: str, idx: int, cfg: dict) -> dict:
    shape = SHAPES[family]
    d = os.path.join(OUT, family)
    src = os.path.join(d, f"{idx:02d}.cu")
    args = [CHECK, "gen", family, ARCH, ",".join(map(str, shape)), src] + [f"{k}={v}" for k, v in cfg.items()]
    g = json.loads(subprocess.run(args, capture_output=True, text=True, check=True).stdout)
    entry = dict(family=family, shape=shape, config=cfg, valid=g["valid"], symbol=g["symbol"], grid=g["grid"],
                 block=g["block"])
    if not g["valid"]:
        entry["rejected"] = "validator: " + g["reason"]
        return entry
    lib = os.path.join(d, f"{idx:02d}.so")
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-Xcompiler", "-fPIC", "-shared",
           "-cudart", "shared", "-I", os.path.join(ref, "kernels", "templates", "include"), "-include", src,
           f"-DKS_REF_SYMBOL={g['symbol']}", os.path.join(HERE, "ref_launch.cu"), "-o", lib]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        first = next((ln for ln in r.stderr.splitlines() if "error" in ln), r.stderr.strip()[:200])
        entry["rejected"] = "nvcc: " + first.split("error", 1)[-1].strip(": ")
        return entry
    entry["lib"] = os.path.relpath(lib, os.path.join(ROOT, "oracle", "_ref"))
    return entry


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("reference")
    ap.add_argument("-j", type=int, default=os.cpu_count() or 8)
    a = ap.parse_args()
    if not os.access(CHECK, os.X_OK):
        print("build_ref_kernels: oracle/_ref/ref_tune_check is not built", file=sys.stderr)
        return 1
    jobs = []
    for family in SHAPES:
        os.makedirs(os.path.join(OUT, family), exist_ok=True)
        jobs += [(family, i, c) for i, c in enumerate(auto_grid(family))]
    with ThreadPoolExecutor(a.j) as ex:
        entries = list(ex.map(lambda t: build_one(a.reference, *t), jobs))
    with open(os.path.join(OUT, "index.json"), "w") as f:
        json.dump(entries, f, indent=1)
    for family in SHAPES:
        es = [e for e in entries if e["family"] == family]
        print(f"{family:16s} {sum('lib' in e for e in es):2d} of {len(es)} built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
