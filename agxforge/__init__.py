"""agxforge — the reference's Python API for the quantized LLM decode path, running on NVIDIA B200 (sm_100a).

This package keeps the reference's module paths for the decode path, so code written against them imports unchanged:

    agxforge.kernels      qmv (affine group-64 packs, the GEMV family), attention, norm, argmax, qmm (the batched
                          tensor-core GEMM)
    agxforge.inference    models (shapes), catalog (which kernel form and launch plan each role runs), assemble (the
                          layer builder: weights, KV cache and decode graph on the device), execute (the decode loop
                          and its report), checkpoint (MLX-format packs from safetensors files), encoder, tp

Every computation runs in libagxcuda.so (hand-written CUDA for sm_100a, built in-tree by
``python -m agxforge_b200.build``) through the C ABI declared in include/agxc.h and bound by agxforge_b200._native.
There is no CPU fallback: without the library a call raises FileNotFoundError, without a GPU RuntimeError.
"""
__version__ = "0.2.0"
