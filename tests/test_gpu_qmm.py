"""The batched GEMM on the tensor cores (tcgen05 + TMEM) against the FP64 GEMM of the same pack.

The weights are dequantised once to fp16 (w16 = fp16(q * s + b)) as the reference's tensor-unit path does
(tools/g17qsm.py), then multiplied with fp32 accumulation: |y - x W^T| <= 2^-10 * sum|x||w| + 1e-6 per entry (fp16
rounding of w, relative 2^-11, plus the fp32 sums)."""
import numpy as np
import pytest

from oracle import pack as P

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _case(torch, bits, N_, K, B, sdt="fp16", seed=0):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N_, K)) * 0.02).astype(np.float32)
    packed, s16, b16, _ = Q.quantize(W, bits=bits, scale_dtype=sdt)
    pk = Q.Pack(packed, s16, b16, N_, K, bits=bits, scale_dtype=sdt)
    W64 = P.dequant64(P.unpack(packed, bits, N_, K), s16, b16, sdt)
    x16 = rng.standard_normal((B, K)).astype(np.float16)
    return pk, x16, W64


def _check(y, x16, W64):
    x = x16.astype(np.float64)
    ref = x @ W64.T
    bound = 2.0 ** -10 * (np.abs(x) @ np.abs(W64).T) + 1e-6
    err = np.abs(y.astype(np.float64) - ref)
    assert np.all(err <= bound), (err.max(), float((err / bound).max()))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("B", [32, 64, 128, 256])
def test_qmm_against_fp64(torch, bits, B):
    from agxforge.kernels.qmm import qmm
    pk, x16, W64 = _case(torch, bits, 256, 1024, B, seed=B + bits)
    y = qmm(pk, torch.from_numpy(x16).cuda(), ksplit=1).cpu().numpy()
    _check(y, x16, W64)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("groups,B", [(7, 32), (7, 128), (6, 64), (14, 256), (3, 48)])
def test_qmm_chunk_shapes(torch, bits, groups, B):
    """K ranges of an odd number of 64-groups (one-group chunks: four dequant warps share a group's k) and of 2 mod 4
    groups (two-group chunks), as the tensor-parallel shards produce (the 7B down projection at 8 ranks: 7 groups)."""
    from agxforge.kernels.qmm import qmm
    pk, x16, W64 = _case(torch, bits, 256, 64 * groups, B, seed=groups * 10 + bits)
    y = qmm(pk, torch.from_numpy(x16).cuda(), ksplit=1).cpu().numpy()
    _check(y, x16, W64)


@pytest.mark.parametrize("ksplit", [1, 2, 4, 0])
def test_qmm_k_split(torch, ksplit):
    from agxforge.kernels.qmm import qmm
    pk, x16, W64 = _case(torch, 4, 384, 2048, 48, seed=7)
    y = qmm(pk, torch.from_numpy(x16).cuda(), ksplit=ksplit).cpu().numpy()
    _check(y, x16, W64)


def test_qmm_bf16_scales_and_wide_n(torch):
    from agxforge.kernels.qmm import qmm
    pk, x16, W64 = _case(torch, 4, 2048, 512, 32, sdt="bf16", seed=9)
    y = qmm(pk, torch.from_numpy(x16).cuda()).cpu().numpy()
    _check(y, x16, W64)


def test_qmm_agrees_with_gemv_rows(torch):
    """The first 8 activation rows through the CUDA-core GEMV (exact factorised form) and through the tensor-core
    GEMM (fp16 weights) agree within the fp16 weight rounding."""
    from agxforge.kernels import qmv as Q
    from agxforge.kernels.qmm import qmm
    pk, x16, W64 = _case(torch, 8, 512, 1024, 32, seed=13)
    x = torch.from_numpy(x16).cuda()
    y_mm = qmm(pk, x).cpu().numpy()[:8].astype(np.float64)
    y_mv = Q.qmv(pk, x[:8]).cpu().numpy().astype(np.float64)
    bound = 2.0 ** -10 * (np.abs(x16[:8].astype(np.float64)) @ np.abs(W64).T) + 1e-5
    assert np.all(np.abs(y_mm - y_mv) <= bound)


def test_qmm_rejects_bad_shapes(torch):
    from agxforge.kernels.qmm import qmm
    pk, x16, _ = _case(torch, 4, 256, 512, 32, seed=1)
    with pytest.raises(ValueError):
        qmm(pk, torch.zeros((24, 512), dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        qmm(pk, torch.zeros((32, 256), dtype=torch.float16, device="cuda"))
