"""The decode kernels (the reference's agxforge/kernels/__init__.py:1-25 module layout), each a host wrapper over
libagxcuda.so:

    qmv        the affine group-64 weight pack (quantize, device pack, unpack, dequant), the GEMV family with its
               fused RMSNorm prologue and residual / SwiGLU epilogues, and the reference's layout records and
               per-kernel functions (qmv_layout, qmv2_ksplit_reference, qmv_swiglu_reference, residual_reference, ...)
    attention  split-KV decode attention with the log-sum-exp merge; attn_layout, attn_reference, attn_rope_reference
    norm       the standalone RMSNorm; rmsnorm_wide_reference
    argmax     the first-maximum rule; argmax_reference
    qmm        the batched tensor-core GEMM (32..256 activation rows)

The reference's numerics module models Apple G17 fp32 arithmetic (flush-to-zero, a software exp2, midpoint-tested
rsqrt) for its bit-exact references; the B200 kernels use IEEE fp32, so it has no counterpart here.
"""
