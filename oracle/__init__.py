"""CPU oracle for the quantized decode path — TEST INFRASTRUCTURE, NOT PRODUCT CODE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this package, and only as
the checker (or, for the baseline, as the timed CPU port). The product path (``agxforge_b200``) never imports it and
fails loudly when its CUDA library is missing.

It restates, in numpy, the reference's CPU implementation of AGXForge's quantized decode path:

    pack        MLX-style affine group-64 quantisation, low-field-first packing, unpack and the fp32 dequant
                (agxforge/kernels/qmv.py:1854-1880, agxforge/inference/assemble.py:834-840, qmv.py:1699-1750)
    decoder     the decoder in FP64 (no intermediate rounding) and in "half transport" FP64 (fp16 rounding at the
                storage points the GPU has), following tools/g17decodestep.py:213-273,459-489 and the per-dispatch
                order of agxforge/inference/assemble.py:852-931; a batched causal forward over a teacher-forced token
                sequence, so a whole history is one pass
    cpu_decode  the reference's CPU decode step (dequant + fp32 matvec chained in QSim order) as a numpy FP32 port,
                timed as the CPU baseline

Parity is pinned by golden vectors produced by the reference's own importable kernel references
(tests/golden/make_golden.py writes tests/golden/ref_kernels.npz; tests/test_oracle_golden.py checks this oracle
against them).
"""
