"""Quantized matrix-vector products for decode (the reference's agxforge/kernels/qmv.py), on the B200.

    quantize(W, bits, group, scale_dtype)   MLX affine quantisation on the device (qmv.py:1854-1871), returning the
                                            reference's format: packed uint32 [N, K*bits/32] low field first,
                                            16-bit scales and biases [N, K/64], fields [N, K]
    Pack                                    a pack re-laid out for the B200 GEMV (16x64 tiles)
    Pack.gateup(gate, up)                   gate and up interleaved for the fused SwiGLU (qmv_swiglu_layout 214-219)
    qmv(pack, x, ...)                       y = W x for 1..8 rows of x, with the RMSNorm prologue (with_norm 176-183)
                                            and the epilogues "f32", "add16" / "add32_to16" (with_residual 112-120),
                                            "swiglu" (qmv_swiglu_reference 222-226)

All arrays on the device are torch tensors; numpy inputs are moved to the device. Shapes are checked here and in the
library; violations raise ValueError naming the constraint, as the reference does (qmv.py:74-80).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from agxforge_b200 import _native as N

SCALE_DTYPES = {"fp16": N.SCALE_FP16, "bf16": N.SCALE_BF16}
EPILOGUES = {"f32": N.EPI_F32, "add16": N.EPI_RES1, "add32_to16": N.EPI_RES2, "swiglu": N.EPI_SWIGLU}


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("agxforge_b200 needs a CUDA device (B200); none is visible")
    return torch


def _stream(torch):
    """torch's current stream as a cudaStream_t. torch's default stream has handle 0, which the C ABI reads as "the
    context's own stream"; it is passed as cudaStreamLegacy (1) so our kernels stay ordered with torch's work."""
    h = torch.cuda.current_stream().cuda_stream
    return C.c_void_p(h if h else 1)


def check_shape(N_, K, bits, group=64):
    if bits not in (4, 8):
        raise ValueError("qmv: 4- or 8-bit weights")
    if group != 64:
        raise ValueError("qmv: group 64 only")
    if K % group:
        raise ValueError("qmv: K (%d) must be a multiple of the group (%d)" % (K, group))
    if N_ % 16:
        raise ValueError("qmv: N (%d) must be a multiple of 16 (the tile rows)" % N_)


def quantize(W, bits=4, group=64, scale_dtype="fp16", device=0):
    """Affine quantisation of fp32 weights [N, K] on the device. Returns (packed, scales, biases) as torch tensors
    (uint32 words as int32, 16-bit patterns as int16) in the reference's format; numpy input gives numpy output."""
    torch = _torch()
    as_numpy = isinstance(W, np.ndarray)
    Wt = torch.as_tensor(W, dtype=torch.float32).to("cuda:%d" % device).contiguous()
    Nr, K = Wt.shape
    if bits not in (4, 8) or group != 64 or K % group:
        raise ValueError("quantize: 4 or 8 bits, group 64, K a multiple of 64")
    if scale_dtype not in SCALE_DTYPES:
        raise ValueError("quantize: scale_dtype fp16 or bf16")
    packed = torch.empty((Nr, K * bits // 32), dtype=torch.int32, device=Wt.device)
    s16 = torch.empty((Nr, K // group), dtype=torch.int16, device=Wt.device)
    b16 = torch.empty_like(s16)
    d = N.PackDesc(Nr, K, bits, group, SCALE_DTYPES[scale_dtype])
    N.check(N.lib().agxc_quantize_dev(N.context(device), C.byref(d), N.ptr(Wt), N.ptr(packed), N.ptr(s16),
                                      N.ptr(b16), _stream(torch)), "quantize")
    if as_numpy:
        torch.cuda.synchronize()
        return (packed.cpu().numpy().view(np.uint32), s16.cpu().numpy().view(np.uint16),
                b16.cpu().numpy().view(np.uint16))
    return packed, s16, b16


def _dev(a, torch, device):
    if isinstance(a, np.ndarray):
        a = np.ascontiguousarray(a)
        if a.dtype == np.uint32:
            a = a.view(np.int32)
        elif a.dtype == np.uint16:
            a = a.view(np.int16)
        return torch.from_numpy(a).to("cuda:%d" % device)
    return a.contiguous()


class Pack:
    """A pack on the device in the B200 tile layout (owned by the library; freed with the object)."""

    def __init__(self, packed, scales, biases, N_, K, bits=4, scale_dtype="fp16", device=0, _gateup=None):
        torch = _torch()
        check_shape(N_, K, bits)
        self.N, self.K, self.bits, self.scale_dtype, self.device = N_, K, bits, scale_dtype, device
        self.gateup = _gateup is not None
        d = N.PackDesc(N_ // 2 if self.gateup else N_, K, bits, 64, SCALE_DTYPES[scale_dtype])
        h = C.c_void_p()
        ctx = N.context(device)
        if self.gateup:
            g = [_dev(a, torch, device) for a in (packed, scales, biases)]
            u = [_dev(a, torch, device) for a in _gateup]
            torch.cuda.synchronize()
            N.check(N.lib().agxc_pack_create_gateup(ctx, C.byref(d), *[N.ptr(t) for t in g], *[N.ptr(t) for t in u],
                                                     1, C.byref(h)), "pack_create_gateup")
        else:
            t = [_dev(a, torch, device) for a in (packed, scales, biases)]
            torch.cuda.synchronize()
            N.check(N.lib().agxc_pack_create(ctx, C.byref(d), *[N.ptr(x) for x in t], 1, C.byref(h)), "pack_create")
        self._h = h

    @classmethod
    def gateup(cls, gate, up, F, K, bits=4, scale_dtype="fp16", device=0):
        """gate and up: (packed, scales, biases) each for [F, K]; the pack holds 2F rows (gate rows then up rows)."""
        return cls(*gate, 2 * F, K, bits, scale_dtype, device, _gateup=up)

    @property
    def handle(self):
        return self._h

    @property
    def nbytes(self):
        """Algorithmic bytes: packed fields plus one 16-bit scale and bias per group."""
        return int(N.lib().agxc_pack_bytes(self._h))

    def unpack(self):
        """The fields uint8 [N, K] (assemble._unpack), read back from the device tiles."""
        torch = _torch()
        out = torch.empty((self.N, self.K), dtype=torch.uint8, device="cuda:%d" % self.device)
        N.check(N.lib().agxc_pack_unpack_dev(self._h, N.ptr(out), _stream(torch)), "unpack")
        return out

    def dequant(self):
        """fp32 [N, K] weights w = fma(q, s, b), one rounding (qmv_dq_reference's w)."""
        torch = _torch()
        out = torch.empty((self.N, self.K), dtype=torch.float32, device="cuda:%d" % self.device)
        N.check(N.lib().agxc_pack_dequant_dev(self._h, N.ptr(out), _stream(torch)), "dequant")
        return out

    def __del__(self):
        h = getattr(self, "_h", None)
        lib = getattr(N, "_lib", None) if N is not None else None
        if h and lib is not None:
            lib.agxc_pack_free(h)
        self._h = None


def qmv(pack, x, norm_gain=None, eps=1e-6, epi="f32", res=None, out=None, splits=0, row_tiles=0, chunk_groups=0,
        stages=0):
    """y = W x on the device for x [nb, K] (nb 1..8; fp16 or fp32 torch tensor). Optional RMSNorm of x first
    (norm_gain fp16 [K]). epi: "f32" -> fp32 [nb, N]; "add16" -> fp32 h = y + res (fp16); "add32_to16" -> fp16
    fp16(y + res) (res fp32); "swiglu" -> fp16 [nb, N/2] fp16(silu(gate) up). Returns the output tensor.
    splits / row_tiles / chunk_groups / stages override the launch planner (0 = its choice).
    x is staged as fp16: every GEMV input of the decode graph holds fp16 values."""
    torch = _torch()
    if epi not in EPILOGUES:
        raise ValueError("qmv: epilogue one of %s" % sorted(EPILOGUES))
    if x.dim() == 1:
        x = x[None]
    nb, K = x.shape
    if K != pack.K:
        raise ValueError("qmv: x has %d columns, the pack K is %d" % (K, pack.K))
    if not 1 <= nb <= 8:
        raise ValueError("qmv: 1 to 8 rows of x")
    if x.dtype not in (torch.float16, torch.float32):
        raise ValueError("qmv: x is fp16 or fp32")
    x = x.contiguous()
    nout = pack.N // 2 if epi == "swiglu" else pack.N
    if out is None:
        dt = torch.float32 if epi in ("f32", "add16") else torch.float16
        out = torch.empty((nb, nout), dtype=dt, device=x.device)
    if epi in ("add16", "add32_to16"):
        if res is None:
            raise ValueError("qmv: %s needs res" % epi)
        res = res.contiguous()
    if norm_gain is not None:
        norm_gain = norm_gain.contiguous()
    a = N.QmvArgs(pack.handle, nb, N.ptr(x), int(x.dtype == torch.float32), K, N.ptr(norm_gain), float(eps),
                  EPILOGUES[epi], N.ptr(out), nout, N.ptr(res), pack.N if res is not None else 0, int(splits),
                  int(row_tiles), int(chunk_groups), int(stages))
    N.check(N.lib().agxc_qmv(N.context(pack.device), C.byref(a), _stream(torch)), "qmv")
    return out
