"""Affine group-wise weight packs: quantise, pack, unpack, dequantise (numpy; oracle / test infrastructure).

Restates the reference's MLX-style affine quantisation (agxforge/kernels/qmv.py:1854-1871 ``quantize``), its 16-bit
scale/bias conversions (qmv.py:1874-1880 ``_to_bf16`` / ``_from_bf16``), the simulator's field unpack
(agxforge/inference/assemble.py:834-840 ``_unpack``) and the dequantise-once contract ``w = fma(q, s, b)`` rounded once
to fp32 (qmv.py:1699-1750 ``qmv_dq_reference``; agxforge/kernels/qmm.py:75).

Format (the reference's, qmv.py:17-18): per row n and group g of 64 consecutive k,
``scale = (max - min) / (2^bits - 1)`` (1.0 for a constant group), ``bias = min``, both rounded to a 16-bit float;
``q = clip(rint((w - bias) / scale), 0, 2^bits - 1)`` with the ROUNDED scale and bias; packed little-endian into
uint32 words [N, K*bits/32], element k in bits [bits*(k % (32/bits)), ...) of word k // (32/bits) — low field first.
The reference stores bf16 scale/bias (MLX); the synthetic configs of this build store fp16 (``scale_dtype``).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
SCALE_DTYPES = ("fp16", "bf16")


def to_bf16(x):
    """fp32 -> bf16 bit pattern, round to nearest even (qmv.py:1874-1876)."""
    u = np.asarray(x, F32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def from_bf16(h):
    """bf16 bit pattern -> fp32 value (exact) (qmv.py:1879-1880)."""
    return (np.asarray(h, np.uint32) << 16).view(F32)


def to_16(x, scale_dtype):
    """fp32 -> the 16-bit storage pattern (uint16) of ``scale_dtype``, RNE."""
    if scale_dtype == "bf16":
        return to_bf16(x)
    if scale_dtype == "fp16":
        with np.errstate(over="ignore"):
            return np.asarray(x, F32).astype(np.float16).view(np.uint16)
    raise ValueError("scale_dtype must be one of %s" % (SCALE_DTYPES,))


def from_16(h, scale_dtype):
    """16-bit storage pattern -> exact fp32 value."""
    if scale_dtype == "bf16":
        return from_bf16(h)
    if scale_dtype == "fp16":
        return np.asarray(h, np.uint16).view(np.float16).astype(F32)
    raise ValueError("scale_dtype must be one of %s" % (SCALE_DTYPES,))


def check_shape(N, K, bits, group=64):
    """The pack's admissible shapes; raises ValueError naming the violated constraint (the reference's convention,
    qmv.py:74-80)."""
    if bits not in (4, 8):
        raise ValueError("pack: 4- or 8-bit weights")
    if group != 64:
        raise ValueError("pack: group 64 only")
    if K % group:
        raise ValueError("pack: K (%d) must be a multiple of the group (%d)" % (K, group))
    if N < 1:
        raise ValueError("pack: N must be positive")


def quantize(Wf, bits=4, group=64, scale_dtype="bf16"):
    """Affine quantisation of fp32 weights [N, K] -> (packed uint32 [N, K*bits/32], scales uint16 [N, K/group],
    biases uint16 [N, K/group], q uint8/uint16-valued uint32 [N, K]). Restates qmv.py:1854-1871 with the 16-bit type
    selectable; with scale_dtype="bf16" it is the reference's quantize bit for bit."""
    Wf = np.asarray(Wf, F32)
    N, K = Wf.shape
    check_shape(N, K, bits, group)
    g = Wf.reshape(N, K // group, group)
    lo, hi = g.min(-1), g.max(-1)
    levels = (1 << bits) - 1
    scale = np.where(hi > lo, (hi - lo) / F32(levels), F32(1.0)).astype(F32)
    s16 = to_16(scale, scale_dtype)
    b16 = to_16(lo.astype(F32), scale_dtype)
    s32, b32 = from_16(s16, scale_dtype), from_16(b16, scale_dtype)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        qf = np.rint((g - b32[..., None]) / s32[..., None])
    q = np.clip(qf, 0, levels).astype(np.uint32).reshape(N, K)
    return pack(q, bits), s16, b16, q


def pack(q, bits):
    """Fields [N, K] (values < 2^bits) -> uint32 words [N, K*bits/32], low field first."""
    q = np.asarray(q, np.uint32)
    N, K = q.shape
    pw = 32 // bits
    qw = q.reshape(N, K // pw, pw)
    packed = np.zeros((N, K // pw), np.uint32)
    for j in range(pw):
        packed |= qw[:, :, j] << np.uint32(bits * j)
    return packed


def unpack(packed, bits, N, K):
    """uint32 words -> fields uint8 [N, K] (assemble.py:834-840)."""
    per = 32 // bits
    w = np.asarray(packed).reshape(N, K // per).astype(np.uint32, copy=False)
    sh = (bits * np.arange(per)).astype(np.uint32)
    out = np.empty((N, K), np.uint8)

    def block(r0, r1):
        out[r0:r1] = ((w[r0:r1, :, None] >> sh) & np.uint32((1 << bits) - 1)).astype(np.uint8).reshape(r1 - r0, K)
    parallel_rows(N, block)
    return out


def fma32(a, b, c):
    """fp32 fused multiply-add, one rounding of the exact a*b + c, vectorised: a*b is exact in float64 (two fp32
    significands), a*b + c is rounded to ODD in float64 (TwoSum's error decides the sticky bit), then rounded to
    fp32; rounding to odd with 53 >= 24 + 2 bits makes the second rounding the correct single rounding (Boldo and
    Melquiond, "Emulation of FMA and correctly rounded sums: proved algorithms using rounding to odd", 2008). The
    reference uses the same published method (qmv.py:1537-1575 ``_fma32v``)."""
    a, b, c = (np.asarray(v, np.float64) for v in (a, b, c))
    p = a * b
    s = p + c
    bb = s - p
    err = (p - (s - bb)) + (c - bb)
    fix = (err != 0) & ((np.asarray(s).view(np.uint64) & 1) == 0) & np.isfinite(s)
    s = np.where(fix, np.nextafter(s, np.where(err > 0, np.inf, -np.inf)), s)
    return np.asarray(s).astype(F32)


def dequant(q, s16, b16, scale_dtype, group=64):
    """The fp32 weight of every field: w = fma(q, s, b), one rounding (qmv.py:1699-1750's ``w = _fma32v(q, s, b)``).
    q [N, K] fields, s16/b16 [N, K/group] uint16 patterns. Returns fp32 [N, K]."""
    q = np.asarray(q)
    N, K = q.shape
    s = np.repeat(from_16(s16, scale_dtype), group, axis=1)
    b = np.repeat(from_16(b16, scale_dtype), group, axis=1)
    return fma32(q.astype(np.float64), s, b)


def dequant64(q, s16, b16, scale_dtype, group=64):
    """The exact (FP64) value of every weight: q*s + b with no rounding beyond float64 (the FP64 oracle's weights).
    Row blocks run on a thread pool (numpy's array kernels release the GIL)."""
    q = np.asarray(q)
    N, K = q.shape
    s = from_16(s16, scale_dtype).astype(np.float64)
    b = from_16(b16, scale_dtype).astype(np.float64)
    out = np.empty((N, K), np.float64)

    def block(r0, r1):
        w = q[r0:r1].reshape(r1 - r0, K // group, group).astype(np.float64)
        w *= s[r0:r1, :, None]
        w += b[r0:r1, :, None]
        out[r0:r1] = w.reshape(r1 - r0, K)
    parallel_rows(N, block)
    return out


_POOL = None


def parallel_rows(n, fn, min_rows=64):
    """fn(r0, r1) over row blocks of [0, n) on a thread pool of the host's cores (the oracle's elementwise work)."""
    global _POOL
    import os
    from concurrent.futures import ThreadPoolExecutor
    cores = os.cpu_count() or 1
    if _POOL is None:
        _POOL = ThreadPoolExecutor(cores)
    step = max(min_rows, -(-n // (2 * cores)))
    list(_POOL.map(lambda r0: fn(r0, min(n, r0 + step)), range(0, n, step)))


def pack_bytes(N, K, bits, group=64):
    """Algorithmic bytes of one pack: the packed fields plus one 16-bit scale and one 16-bit bias per group."""
    return N * K * bits // 8 + (N * K // group) * 4
