"""Argmax and the device-resident generation step (the reference's agxforge/kernels/argmax.py).

In the decode step the argmax is fused into the vocabulary GEMV (each CTA keeps the first maximum of its rows, the
last CTA to finish reduces the CTAs' pairs) and the generation step runs in that same last CTA: token = the pending
forced token, else the logged prompt token at q0 + 1, else the first maximum; the token is logged at q0 + 1, its
embedding row becomes the next x, and q0 advances, clamped to cap - 1 (argmax.py:133-215; assemble.py:918-930).

    TOKEN_UNSET             a free log entry (0xFFFFFFFF)
    argmax(logits)          the first maximum of a device row (torch tensor) as an int
    argmax_reference(l)     the reference's name (argmax.py:287-288): the same, for numpy input
"""
from __future__ import annotations

import numpy as np

from agxforge_b200 import _native as N
from agxforge_b200._native import TOKEN_UNSET  # noqa: F401  (re-exported: the token log's free marker)
from agxforge.kernels import qmv as _qmv


def argmax(logits, device=0):
    """The smallest index of the largest value of an fp32 row (NaN-free), by one device reduction."""
    import torch
    x = logits.reshape(-1).to(torch.float32).contiguous()
    if x.numel() == 0:
        raise ValueError("argmax: an empty row")
    out = torch.empty(1, dtype=torch.int32, device=x.device)
    N.check(N.lib().agxc_argmax_dev(N.context(device), N.ptr(x), x.numel(), N.ptr(out), _qmv._stream(torch)), "argmax")
    return int(out.item())


def argmax_reference(logits):
    """int(np.argmax(logits)) (argmax.py:287-288), computed on the B200."""
    import torch
    return argmax(torch.as_tensor(np.asarray(logits, np.float32)).cuda())
