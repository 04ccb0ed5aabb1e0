"""CPU oracle for the six kernscope-tune kernel families -- TEST INFRASTRUCTURE.

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path (``kernscope_b200``)
never imports it and has no CPU fallback.

It restates, in NumPy + ml_dtypes, the reference golden harness of
kernscope (``tests/golden/kernscope_golden``):

* ``refs``    -- the per-family reference math (``refs.py:57-153``) plus the
  extensions the B200 build needs (tanh GELU, full fp32 sum in fp64,
  batched multi-head causal attention);
* ``inputs``  -- seeded input generation (``inputs.py:73-132``), bit-identical
  to the reference for the reference profile, plus the ``baseline`` profile
  whose distributions follow the benchmark configurations;
* ``metrics`` -- the reference verdict (cosine / max_rel_err / pcc,
  ``metrics.py:29-116``) and the floor-guarded relative error used for the
  benchmark tolerances.

Parity is pinned: ``tests/golden/make_fixtures.py`` imported the reference
harness itself to write ``tests/golden/*.npz`` (inputs + expected outputs);
``tests/test_oracle_pins.py`` checks this restatement against them bit for bit.
"""

from . import inputs, metrics, refs  # noqa: F401

__all__ = ["inputs", "metrics", "refs"]
