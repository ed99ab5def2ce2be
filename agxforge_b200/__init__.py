"""agxforge_b200 — the native half of the B200 decode path: the CUDA sources (csrc/), the built library
(lib/libagxcuda.so, ``python -m agxforge_b200.build``) and its ctypes binding (_native). The Python API that mirrors
the reference's modules lives in the ``agxforge`` package beside this one."""
__version__ = "0.2.0"
