"""Batched quantized GEMM for 32..256 activation rows on the B200 tensor cores (the reference's tensor-unit path:
agxforge/kernels/qmm.py and tools/g17qsm.py:1-21; assemble.layer_ops_qsm agxforge/inference/assemble.py:368-426).

    qmm(pack, x, ksplit=0) -> y fp32 [B, N]

x fp16 [B, K] (B a multiple of 16 in 32..256), pack a plain `qmv.Pack` with N a multiple of 128. The weights are
dequantised once to fp16 (w = fp16(q * s + b), one rounding) and multiplied by tcgen05 MMAs with fp32 accumulation
in tensor memory; `ksplit` splits K over CTAs (0 = the library's choice).
"""
from __future__ import annotations

import ctypes as C

from agxforge_b200 import _native as N
from agxforge.kernels import qmv as _qmv


def qmm(pack, x, ksplit=0, out=None):
    import torch
    if x.dim() != 2 or x.shape[1] != pack.K:
        raise ValueError("qmm: x is [B, K] with K = %d" % pack.K)
    B = x.shape[0]
    if B < 32 or B > 256 or B % 16:
        raise ValueError("qmm: 32 to 256 activation rows, a multiple of 16")
    if pack.N % 128:
        raise ValueError("qmm: N must be a multiple of 128")
    if pack.gateup:
        raise ValueError("qmm: a plain pack")
    x = x.to(torch.float16).contiguous()
    if out is None:
        out = torch.empty((B, pack.N), dtype=torch.float32, device=x.device)
    N.check(N.lib().agxc_qmm(N.context(pack.device), pack.handle, N.ptr(x), B, N.ptr(out), pack.N, int(ksplit),
                             _qmv._stream(torch)), "qmm")
    return out
