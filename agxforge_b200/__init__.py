"""agxforge_b200 — AGXForge's quantized LLM decode path, rebuilt for NVIDIA B200 (sm_100a).

The package keeps the reference's Python module layout for this path:

    agxforge_b200.kernels      qmv (affine group-64 packs, the GEMV family), attention, norm, argmax, numerics
    agxforge_b200.inference    models (shapes), catalog (which kernel form each role runs), assemble (the layer
                               builder: a model's weights, KV cache and decode graph on the device), execute (the
                               decode loop and its report)

Every computation runs in libagxcuda.so (hand-written CUDA for sm_100a, built in-tree by
``python -m agxforge_b200.build``) through the C ABI in include/agxc.h. There is no CPU fallback.
"""
__version__ = "0.1.0"
