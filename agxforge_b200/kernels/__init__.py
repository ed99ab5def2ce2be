"""The decode kernels (the reference's agxforge/kernels/__init__.py:1-25 module layout), each a thin host wrapper
over libagxcuda.so:

    qmv        the affine group-64 weight pack (quantize, device pack, unpack, dequant) and the GEMV family with its
               fused RMSNorm prologue and residual / SwiGLU epilogues
    attention  split-KV decode attention with the log-sum-exp merge
    norm       the standalone RMSNorm
    argmax     the first-maximum rule and the generation step's token choice
    numerics   the shared constants (the base-2 softmax scale, RoPE tables)
"""
