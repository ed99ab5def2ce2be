"""agxc_qmv_noalloc (the GEMV entry point that takes its split-K scratch from static device memory) against agxc_qmv.

Both run the same kernels with the same launch plan and sum the split-K partials in the same order, so the outputs
must agree bit for bit; they are also held to the FP64 GEMV bound of the kernel tests. Each case calls the no-alloc
entry point twice in a row (the second call finds the counters the first one left) and between other entry points.
Collected last (file name) so it also runs after every other GPU test; it needs nothing from them.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import pack as P

pytestmark = pytest.mark.gpu

EPS32 = np.finfo(np.float32).eps
STATIC_PART_FLOATS = 1 << 20


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _case(torch, bits, N_, K, nb, seed):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N_, K)) * 0.02).astype(np.float32)
    packed, s16, b16, _ = Q.quantize(W, bits=bits, scale_dtype="fp16")
    pk = Q.Pack(packed, s16, b16, N_, K, bits=bits)
    W64 = P.dequant64(P.unpack(packed, bits, N_, K), s16, b16, "fp16")
    x16 = rng.standard_normal((nb, K)).astype(np.float16)
    return pk, x16, W64


def _noalloc(torch, pk, x, epi="f32", res=None, splits=0):
    """agxc_qmv_noalloc through the C-ABI with the argument block agxc_qmv takes."""
    from agxforge_b200 import _native as N
    from agxforge.kernels import qmv as Q
    nb, K = x.shape
    nout = pk.N
    dt = torch.float32 if epi in ("f32", "add16") else torch.float16
    out = torch.full((nb, nout), float("nan"), dtype=dt, device=x.device)
    a = N.QmvArgs(pk.handle, nb, N.ptr(x), 0, K, None, 1e-6, Q.EPILOGUES[epi], N.ptr(out), nout, N.ptr(res),
                  pk.N if res is not None else 0, int(splits), 0, 0, 0)
    N.check(N.lib().agxc_qmv_noalloc(N.context(pk.device), C.byref(a), Q._stream(torch)), "qmv_noalloc")
    return out


def _bound(x16, W64):
    x = x16.astype(np.float64)
    return x @ W64.T, 32 * EPS32 * (np.abs(x) @ np.abs(W64).T) + 1e-7


@pytest.mark.parametrize("bits,N_,K,nb,splits", [
    (4, 2048, 4096, 4, 4),     # split K asked for
    (4, 1024, 8192, 8, 2),     # 8 rows of 8,192 columns, K split in two (an explicit plan, independent of the planner)
    (8, 512, 2048, 2, 8),
    (4, 768, 1024, 1, 1),      # no split: the static block is not touched
])
def test_noalloc_matches_qmv_twice(torch, bits, N_, K, nb, splits):
    from agxforge.kernels import qmv as Q
    pk, x16, W64 = _case(torch, bits, N_, K, nb, seed=N_ + K + nb + bits)
    x = torch.from_numpy(x16).cuda()
    y_ref = Q.qmv(pk, x, splits=splits)
    y1 = _noalloc(torch, pk, x, splits=splits)
    y2 = _noalloc(torch, pk, x, splits=splits)
    torch.cuda.synchronize()
    assert torch.equal(y1, y_ref)
    assert torch.equal(y2, y_ref)
    ref, bound = _bound(x16, W64)
    assert np.all(np.abs(y1.cpu().numpy().astype(np.float64) - ref) <= bound)


def test_noalloc_residual_epilogue_and_interleaving(torch):
    """add32_to16 with split K, interleaved with agxc_qmv calls of another shape on the same stream."""
    from agxforge.kernels import qmv as Q
    pk, x16, W64 = _case(torch, 4, 1536, 4096, 3, seed=11)
    pk2, x16b, _ = _case(torch, 4, 256, 2048, 2, seed=12)
    x = torch.from_numpy(x16).cuda()
    xb = torch.from_numpy(x16b).cuda()
    res = torch.randn((3, 1536), dtype=torch.float32, device="cuda")
    y_ref = Q.qmv(pk, x, epi="add32_to16", res=res, splits=8)
    outs = []
    for _ in range(2):
        outs.append(_noalloc(torch, pk, x, epi="add32_to16", res=res, splits=8))
        Q.qmv(pk2, xb, splits=4)
        outs.append(_noalloc(torch, pk2, xb, splits=4))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], y_ref) and torch.equal(outs[2], y_ref)
    assert torch.equal(outs[1], outs[3])
    assert torch.equal(outs[1], Q.qmv(pk2, xb, splits=4))


def test_noalloc_rejects_oversize_plan(torch):
    """splits x N x nb above the static block's 1,048,576 partials is refused before any launch."""
    pk, x16, _ = _case(torch, 4, 16384, 4096, 8, seed=13)
    x = torch.from_numpy(x16).cuda()
    assert 16 * 16384 * 8 > STATIC_PART_FLOATS
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(torch, pk, x, splits=16)
    # the same pack with a plan that fits still runs and agrees with agxc_qmv
    from agxforge.kernels import qmv as Q
    y = _noalloc(torch, pk, x, splits=4)
    assert torch.equal(y, Q.qmv(pk, x, splits=4))
