"""Quantized matrix-vector products for decode (the reference's agxforge/kernels/qmv.py), on the B200.

The reference's names, with the same arguments and results:

    quantize(Wf, bits=4, group=64, seed=None, scale_dtype="bf16")
                                    MLX affine quantisation (qmv.py:1854-1871) on the device: (packed uint32
                                    [N, K*bits/32] low field first, scales and biases as 16-bit patterns [N, K/64],
                                    the fields q [N, K]); bf16 scales and biases as the reference emits them,
                                    scale_dtype="fp16" for the BASELINE's synthetic packs
    qmv_layout / with_residual / with_norm / with_batch / qmv_swiglu_layout
                                    the layout records (plain dicts) the reference builds (qmv.py:73-226); here they
                                    carry the shape and the fused prologue / epilogue a call runs
    qmv2_ksplit_reference / qmv2_reference_fast / qmv_dq_reference / qmv_batch_reference / qmv_swiglu_reference
                                    y = W x for a layout and reference-format fields, computed by the B200 GEMV
                                    (qmv.py:1577-1851): the value the reference's CPU functions compute, within the
                                    GEMV tolerance (fp32 sums in another order), returned as numpy like theirs
    residual_reference              the epilogue add: h = fp32(y + x16) or fp16(y + h) (qmv.py:169-173), on the device

The B200 forms underneath:

    Pack                            a pack re-laid out for the B200 GEMV (16x64 tiles)
    Pack.gateup(gate, up)           gate and up interleaved for the fused SwiGLU (qmv_swiglu_layout 214-219)
    qmv(pack, x, ...)               y = W x for 1..8 rows of x, with the RMSNorm prologue (with_norm 176-183) and the
                                    epilogues "f32", "add16" / "add32_to16" (with_residual 112-120), "swiglu"
                                    (qmv_swiglu_reference 222-226)

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
        raise RuntimeError("agxforge needs a CUDA device (B200); none is visible")
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


def quantize(Wf, bits=4, group=64, seed=None, scale_dtype="bf16", device=0):
    """MLX affine quantisation of fp32 weights [N, K] on the device (qmv.py:1854-1871): per group of 64 along K,
    scale = (max - min) / (2^bits - 1) rounded to 16 bits, bias = min rounded to 16 bits, q = clip(rint((w - b) / s)).
    Returns (packed, s16, b16, q): packed uint32 [N, K*bits/32] low field first, the scale and bias 16-bit patterns
    [N, K/64] (bf16 by default, as the reference; fp16 with scale_dtype="fp16") and the fields q [N, K]. numpy input
    gives numpy output (uint32, uint16, uint16, uint32), a torch tensor gives device tensors (int32, int16, int16,
    uint8). `seed` is accepted for the reference's signature and unused there too."""
    torch = _torch()
    as_numpy = isinstance(Wf, np.ndarray)
    Wt = torch.as_tensor(Wf, dtype=torch.float32).to("cuda:%d" % device).contiguous()
    if Wt.dim() != 2:
        raise ValueError("quantize: W is [N, K]")
    Nr, K = Wt.shape
    if bits not in (4, 8):
        raise ValueError("quantize: 4- or 8-bit weights")
    if group != 64:
        raise ValueError("quantize: group 64 only")
    if K % group:
        raise ValueError("quantize: K (%d) must be a multiple of the group (%d)" % (K, group))
    if scale_dtype not in SCALE_DTYPES:
        raise ValueError("quantize: scale_dtype fp16 or bf16")
    packed = torch.empty((Nr, K * bits // 32), dtype=torch.int32, device=Wt.device)
    s16 = torch.empty((Nr, K // group), dtype=torch.int16, device=Wt.device)
    b16 = torch.empty_like(s16)
    d = N.PackDesc(Nr, K, bits, group, SCALE_DTYPES[scale_dtype])
    N.check(N.lib().agxc_quantize_dev(N.context(device), C.byref(d), N.ptr(Wt), N.ptr(packed), N.ptr(s16),
                                      N.ptr(b16), _stream(torch)), "quantize")
    q = fields(packed, bits, K)
    if as_numpy:
        torch.cuda.synchronize()
        return (packed.cpu().numpy().view(np.uint32), s16.cpu().numpy().view(np.uint16),
                b16.cpu().numpy().view(np.uint16), q.cpu().numpy().astype(np.uint32))
    return packed, s16, b16, q


def fields(packed, bits, K):
    """The fields uint8 [N, K] of packed words [N, K*bits/32] (low field first; assemble._unpack 834-840), on the
    device."""
    torch = _torch()
    w = packed.view(torch.int32) if packed.dtype != torch.int32 else packed
    per = 32 // bits
    shifts = torch.arange(per, device=w.device, dtype=torch.int32) * bits
    f = (w.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
    return f.reshape(w.shape[0], K).to(torch.uint8)


def pack_fields(q, bits):
    """Packed words int32 [N, K*bits/32] of fields [N, K] (the inverse of fields), on the device."""
    torch = _torch()
    q = torch.as_tensor(np.asarray(q) if isinstance(q, np.ndarray) else q).to("cuda").to(torch.int64)
    Nr, K = q.shape
    per = 32 // bits
    shifts = torch.arange(per, device=q.device, dtype=torch.int64) * bits
    w = ((q.reshape(Nr, K // per, per) & ((1 << bits) - 1)) << shifts).sum(-1)
    return w.to(torch.uint32).view(torch.int32) if hasattr(torch, "uint32") else \
        ((w + 2 ** 31) % 2 ** 32 - 2 ** 31).to(torch.int32)


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


# ------------------------------------------------------------------------------------------------------------------
# The reference's layout records and per-kernel functions (qmv.py:73-226, 1506-1851), run on the B200.

def qmv_layout(N, K, bits=4, group=64, rows=4, hoist=False, premask=False, fma=False, nocarrier=False):
    """The layout record of one GEMV (qmv.py:73-109). `rows`, `hoist`, `premask`, `fma` and `nocarrier` choose among
    the reference's G17 code forms and are kept in the record; the B200 kernel plans its own tiling."""
    if bits not in (4, 8):
        raise ValueError("qmv: 4- or 8-bit weights")
    if group != 64 or K % group:
        raise ValueError("qmv: K must be a multiple of the group (64)")
    if N % 16:
        raise ValueError("qmv: N must be a multiple of 16 (the tile rows)")
    if N % rows:
        raise ValueError("qmv: N must be a multiple of rows")
    return dict(op="qmv", Nout=N, Kq=K, bits=bits, group=group, rows=rows, groups=N // rows, per_word=32 // bits,
                hoist=hoist, premask=premask, fma=fma, nocarrier=nocarrier)


def with_residual(lay, res):
    """Fold a residual add into the epilogue (qmv.py:112-120): "add16" h = fp32(W x + x16), "add32_to16"
    x = fp16(W x + h)."""
    if res not in ("add16", "add32_to16"):
        raise ValueError(res)
    return dict(lay, res=res)


def with_norm(lay, norm):
    """Fold an RMSNorm of x into the load (qmv.py:176-183); norm is "half" or "float", the row's storage."""
    if norm not in ("half", "float"):
        raise ValueError("with_norm: half or float")
    return dict(lay, norm=norm, eps=lay.get("eps", 1e-5))


def with_batch(lay, nb):
    """nb activation vectors against the same weights (qmv.py:186-203); the B200 GEMV takes up to 8."""
    if nb < 2:
        raise ValueError("with_batch: two or more vectors")
    if nb > 8:
        raise ValueError("with_batch: at most 8 vectors on the GEMV path (32 or more run the batched GEMM)")
    return dict(lay, batch=nb)


def qmv_swiglu_layout(F, K, bits=4, rows=4, nocarrier=True):
    """gate and up fused with the SwiGLU (qmv.py:214-219): one GEMV of 2F rows, gate rows then up rows."""
    lay = qmv_layout(2 * F, K, bits=bits, rows=rows, nocarrier=nocarrier)
    return dict(lay, swiglu=True, ffn=F, groups=F // rows)


def _ref_pack(lay, q, s16, b16, device=0):
    """A device Pack of reference-format fields q [N, K] and 16-bit scale / bias patterns [N, K/64] for a layout."""
    torch = _torch()
    bits, Nn, K = lay["bits"], lay["Nout"], lay["Kq"]
    sdt = lay.get("scale_dtype", "bf16")
    qt = torch.as_tensor(np.ascontiguousarray(q, dtype=np.int64) if isinstance(q, np.ndarray) else q)
    if tuple(qt.shape) != (Nn, K):
        raise ValueError("qmv: q is [N, K] = [%d, %d]" % (Nn, K))
    packed = pack_fields(qt, bits)
    s = _dev(np.ascontiguousarray(s16, dtype=np.uint16) if isinstance(s16, np.ndarray) else s16, torch, device)
    b = _dev(np.ascontiguousarray(b16, dtype=np.uint16) if isinstance(b16, np.ndarray) else b16, torch, device)
    if lay.get("swiglu"):
        F = lay["ffn"]
        return Pack.gateup((packed[:F], s[:F], b[:F]), (packed[F:], s[F:], b[F:]), F, K, bits, sdt, device)
    return Pack(packed, s, b, Nn, K, bits, sdt, device)


def _as_rows(x, K, device=0):
    torch = _torch()
    xt = torch.as_tensor(np.asarray(x, np.float32) if not hasattr(x, "device") else x).to("cuda:%d" % device)
    xt = xt.to(torch.float32).reshape(-1, K)
    return xt


def _run(lay, x, q, s16, b16, epi="f32", res=None, norm_gain=None):
    torch = _torch()
    pack = _ref_pack(lay, q, s16, b16)
    xt = _as_rows(x, lay["Kq"])
    out = qmv(pack, xt, norm_gain=norm_gain, eps=lay.get("eps", 1e-5), epi=epi, res=res)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def qmv2_ksplit_reference(lay, x, q, s16, b16):
    """y fp32 [N] = W x for reference-format fields (qmv.py:1838-1851), by the B200 GEMV. The scale and bias patterns
    are bf16 unless lay["scale_dtype"] says fp16."""
    return _run(lay, x, q, s16, b16)[0]


qmv2_reference_fast = qmv2_ksplit_reference     # qmv.py:1577-1649: the same value in the reference's other order
qmv_dq_reference = qmv2_ksplit_reference        # qmv.py:1699-1750: dequantise-once order


def qmv_batch_reference(lay, xs, q, s16, b16):
    """[nb, N]: every vector's y (qmv.py:206-211), one batched B200 GEMV launch for up to 8 vectors."""
    single = dict(lay)
    single.pop("batch", None)
    return _run(single, np.asarray(xs, np.float32), q, s16, b16)


def qmv_swiglu_reference(lay, x, q, s16, b16):
    """act fp16 [F] = fp16(silu(gate) up) over the 2F-row fused pack (qmv.py:222-226), by the B200 GEMV's SwiGLU
    epilogue."""
    if not lay.get("swiglu"):
        raise ValueError("qmv_swiglu_reference: a qmv_swiglu_layout")
    return _run(lay, x, q, s16, b16, epi="swiglu")[0].astype(np.float16)


def residual_reference(lay, y, x16=None, h32=None):
    """The epilogue's add on an fp32 GEMV output y (qmv.py:169-173): "add16" h = fp32(y + x16); "add32_to16"
    out = fp16(y + h). Computed on the device."""
    torch = _torch()
    yt = torch.as_tensor(np.asarray(y, np.float32)).cuda()
    if lay.get("res") == "add16":
        r = yt + torch.as_tensor(np.asarray(x16, np.float16)).cuda().to(torch.float32)
        return r.cpu().numpy().astype(np.float32)
    if lay.get("res") == "add32_to16":
        r = (yt + torch.as_tensor(np.asarray(h32, np.float32)).cuda()).to(torch.float16)
        return r.cpu().numpy()
    raise ValueError("residual_reference: a with_residual layout")
