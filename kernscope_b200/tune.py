"""ctypes binding of the C++20 tuner (``lib/libkernscope_tune.so``).

``run(**options)`` runs ``kernscope::tune::tune`` (pre-screen, gate, bench,
db + tunecache) and returns its JSON evidence as a dict together with the
CLI exit code; ``query(op, **kw)`` exposes the host model (shape hashes,
config spaces, validation, occupancy, roofline, db round trips).
``CLI`` is the path of the ``kernscope-tune`` executable.
"""

from __future__ import annotations

import ctypes as C
import json
import os

from . import native  # noqa: F401  (loads libkernscope_b200.so first, as the tuner links it)

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libkernscope_tune.so")
CLI = os.path.join(PKG, "lib", "kernscope-tune")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python -m kernscope_b200.build`")
lib = C.CDLL(LIB_PATH)
for _name in ("ks_tune_run_json", "ks_tune_query_json"):
    _fn = getattr(lib, _name)
    _fn.restype = C.c_int
    _fn.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]


def _call(fn, payload: dict):
    req = json.dumps(payload).encode()
    need = C.c_size_t(0)
    cap = 1 << 16
    while True:
        buf = C.create_string_buffer(cap)
        rc = fn(req, buf, cap, C.byref(need))
        if rc != -1:
            return rc, json.loads(buf.value.decode())
        cap = int(need.value) + 1


def run(**options) -> tuple[int, dict]:
    """Run the tuning pipeline.  Keys: kernel_family, shape, arch, grid, db,
    cache, min_occupancy, live_bench, use_cache, gate_shape, causal, gelu,
    device, warmup_ms, rep_ms, seed, inject_gate_failure, emit_repro."""
    return _call(lib.ks_tune_run_json, options)


def query(op: str, **kw):
    rc, out = _call(lib.ks_tune_query_json, {"op": op, **kw})
    if rc != 0:
        raise ValueError(out.get("error", out))
    return out["result"]
