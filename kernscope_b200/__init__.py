"""kernscope_b200 -- B200 (sm_100a) kernels for the six kernscope-tune families.

* ``native``  -- ctypes binding of the C ABI (``include/kernscope_b200.h``)
  exported by ``lib/libkernscope_b200.so``;
* ``ops``     -- torch-tensor front end of that ABI (device memory / streams);
* ``tune``    -- binding of the C++20 tuner (``lib/libkernscope_tune.so``):
  config spaces, pre-screen, roofline, bench, db + tunecache, driver;
* ``build``   -- compiles both libraries in-tree for sm_100a.

Importing the package does not load the native library; ``native`` does, and
raises if it has not been built.
"""

__all__ = ["native", "ops", "build"]
