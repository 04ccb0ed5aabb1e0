"""Write the golden fixtures in this folder from the REFERENCE harness itself.

Run once in a checkout that has the kernscope reference tree next to it:

    python tests/golden/make_fixtures.py --reference <kernscope>/tests/golden

It imports the reference's own ``kernscope_golden`` package (inputs.py,
refs.py), generates seeded inputs and expected outputs for every family at
the reference's own test shapes (``tests/golden/test_golden.py:33-40``) and at
the tuner's gate shapes (``tools/tune/tests/*_gen_test.cpp``), and saves them
as ``<family>_<shape>_s<seed>[_causal].npz`` with bf16 arrays stored as raw
uint16 bit patterns.  The fixtures travel with the repository; the reference
tree does not, so nothing at test time imports it.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (family, shape, seed, causal)
CASES = [
    # reference unit-test shapes (test_golden.py:33-40)
    ("matmul", (16, 16, 16), 0, False),
    ("bias_gelu", (16, 32), 0, False),
    ("softmax", (16, 32), 0, False),
    ("layernorm", (16, 32), 0, False),
    ("reduction", (32, 16), 0, False),
    ("attention", (8, 8, 16), 0, False),
    ("attention", (8, 8, 16), 0, True),
    # tuner gate shapes (matmul 64^3, flash 64,64,32, elem gates)
    ("matmul", (64, 64, 64), 0, False),
    ("attention", (64, 64, 32), 0, False),
    ("attention", (64, 64, 32), 0, True),
    ("softmax", (32, 512), 0, False),
    ("layernorm", (32, 512), 0, False),
    ("bias_gelu", (64, 256), 0, False),
    ("reduction", (256, 256), 0, False),
    # ragged / non-tile-multiple shapes and another seed
    ("matmul", (72, 40, 24), 7, False),
    ("softmax", (5, 200), 7, False),
    ("layernorm", (3, 1000), 7, False),
    ("bias_gelu", (7, 24), 7, False),
    ("reduction", (33, 40), 7, False),
    ("attention", (128, 128, 128), 3, True),
]


def fixture_name(family, shape, seed, causal) -> str:
    s = "x".join(str(v) for v in shape)
    return f"{family}_{s}_s{seed}{'_causal' if causal else ''}.npz"


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--reference", required=True,
                   help="path to the reference's tests/golden directory")
    args = p.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    from kernscope_golden import inputs as kin  # the reference harness

    for family, shape, seed, causal in CASES:
        inp = kin.generate_inputs(family, shape, seed=seed)
        exp = kin.reference_output(family, inp, causal=causal)
        arrays = {k: np.asarray(v).view(np.uint16) for k, v in inp.items()}
        arrays["expected"] = np.asarray(exp).view(np.uint16)
        arrays["shape"] = np.asarray(shape, dtype=np.int64)
        arrays["seed"] = np.asarray(seed, dtype=np.int64)
        arrays["causal"] = np.asarray(int(causal), dtype=np.int64)
        out = os.path.join(HERE, fixture_name(family, shape, seed, causal))
        np.savez_compressed(out, **arrays)
        print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
