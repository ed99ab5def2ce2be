"""RMSNorm for decode (the reference's agxforge/kernels/norm.py:42-155 build_rmsnorm_wide): one row per CTA,
y = fp16(x * rsqrt(mean(x^2) + eps) * g). Inside the decode step the norm is fused into the GEMV that consumes it
(qmv.qmv(..., norm_gain=g)); this standalone form is the final norm's reference shape and a test surface.

    rmsnorm(x, g, eps)                              device tensors in and out
    rmsnorm_wide_reference(v, g, spec, tpg, seed)   the reference's name (norm.py:185-203): numpy in, fp16 numpy out;
                                                    eps from spec.norm_eps; `tpg` and `seed` choose among the
                                                    reference's G17 code forms and are accepted unused
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from agxforge_b200 import _native as N
from agxforge.kernels import qmv as _qmv


def rmsnorm(x, g, eps=1e-6, device=0):
    import torch
    if x.dim() == 1:
        x = x[None]
    nb, d = x.shape
    if g.shape[-1] != d or g.dtype != torch.float16:
        raise ValueError("rmsnorm: gain fp16 [d]")
    if x.dtype not in (torch.float16, torch.float32):
        raise ValueError("rmsnorm: x fp16 or fp32")
    x, g = x.contiguous(), g.contiguous()
    out = torch.empty((nb, d), dtype=torch.float16, device=x.device)
    N.check(N.lib().agxc_rmsnorm_dev(N.context(device), N.ptr(x), int(x.dtype == torch.float32), nb, d, N.ptr(g),
                                     float(eps), N.ptr(out), _qmv._stream(torch)),
            "rmsnorm")
    return out


def rmsnorm_wide_reference(v, g, spec, tpg=1024, seed=False):
    """y fp16 [d] = fp16(v * rsqrt(mean(v^2) + eps) * g) of one row (norm.py:185-203), by the B200 kernel."""
    import torch
    eps = float(getattr(spec, "norm_eps", getattr(spec, "EPS", 1e-5)))
    va = np.asarray(v)
    x = torch.as_tensor(va.astype(np.float16 if va.dtype == np.float16 else np.float32)).cuda()
    gt = torch.as_tensor(np.asarray(g, np.float32).astype(np.float16)).cuda()
    y = rmsnorm(x, gt, eps)
    torch.cuda.synchronize()
    return y.cpu().numpy()[0]
