"""ctypes binding of libagxcuda.so (include/agxc.h). The only way the package reaches the GPU.

There is no CPU fallback: if the library is missing, ``lib()`` raises FileNotFoundError (the reference raises the same
when its Metal executor is missing, agxforge/inference/execute.py:40-41); a failing call raises ValueError (bad
argument, the reference's convention qmv.py:74-80), TimeoutError (a bounded device wait gave up) or RuntimeError
carrying the library's message (execute.py:47-48's stderr tail).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libagxcuda.so")

OK, EINVAL, ECUDA, ENCCL, ETIMEOUT, ECORRUPT, ENOMEM, EUNSUPPORTED = 0, -1, -2, -3, -4, -5, -6, -7
SCALE_FP16, SCALE_BF16 = 0, 1
TOKEN_UNSET = 0xFFFFFFFF
EPI_F32, EPI_RES1, EPI_RES2, EPI_SWIGLU = 0, 1, 2, 3
ROLE_QKV, ROLE_WO, ROLE_GATE, ROLE_UP, ROLE_DOWN, ROLE_HEAD = range(6)
VEC_ATTN_GAIN, VEC_FFN_GAIN, VEC_QKV_BIAS, VEC_FINAL_GAIN, VEC_EMBED, VEC_Q_NORM, VEC_K_NORM = range(7)
OPT_PDL = 0
OPT_TRACE = 1
OPT_FUSED = 2
OPT_BULK = 3
OPT_WAIT_MS = 4
OPT_TP_FUSED = 5
OPT_QK_NORM = 6
OPT_DEVICE_WAIT_US = 7


class PackDesc(C.Structure):
    _fields_ = [("n", C.c_int32), ("k", C.c_int32), ("bits", C.c_int32), ("group", C.c_int32),
                ("scale_dtype", C.c_int32)]


class QmvArgs(C.Structure):
    _fields_ = [("pack", C.c_void_p), ("nb", C.c_int32), ("x_dev", C.c_void_p), ("x_f32", C.c_int32),
                ("x_ld", C.c_int32), ("norm_gain_dev", C.c_void_p), ("eps", C.c_float), ("epi", C.c_int32),
                ("out_dev", C.c_void_p), ("out_ld", C.c_int32), ("res_dev", C.c_void_p), ("res_ld", C.c_int32),
                ("splits", C.c_int32), ("row_tiles", C.c_int32), ("chunk_groups", C.c_int32),
                ("stages", C.c_int32)]


class ModelDesc(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("ffn", C.c_int32), ("vocab", C.c_int32), ("bits", C.c_int32),
                ("group", C.c_int32), ("scale_dtype", C.c_int32), ("cap", C.c_int32), ("batch", C.c_int32),
                ("qkv_bias", C.c_int32), ("eps", C.c_float), ("rope_theta", C.c_float),
                ("keep_logits", C.c_int32), ("tp_world", C.c_int32), ("tp_rank", C.c_int32),
                ("tp_id", C.c_uint8 * 128)]


class EncoderDesc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("layers", C.c_int32), ("heads", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("max_position", C.c_int32), ("type_vocab", C.c_int32), ("eps", C.c_float),
                ("max_batch", C.c_int32), ("max_seq", C.c_int32)]


class Timing(C.Structure):
    _fields_ = [("gpu_ms", C.c_float), ("host_ms", C.c_float), ("launches_per_step", C.c_int32)]


_P = C.c_void_p
_I = C.c_int
SIGNATURES = {
    "agxc_last_error": (C.c_char_p, []),
    "agxc_version": (_I, []),
    "agxc_init": (_I, [_I, C.POINTER(_P)]),
    "agxc_ctx_free": (None, [_P]),
    "agxc_ctx_sync": (_I, [_P]),
    "agxc_ctx_stream": (_I, [_P, C.POINTER(C.c_void_p)]),
    "agxc_ctx_error_word": (_I, [_P, C.POINTER(C.c_uint32)]),
    "agxc_quantize_dev": (_I, [_P, C.POINTER(PackDesc), _P, _P, _P, _P, _P]),
    "agxc_pack_create": (_I, [_P, C.POINTER(PackDesc), _P, _P, _P, _I, C.POINTER(_P)]),
    "agxc_pack_create_gateup": (_I, [_P, C.POINTER(PackDesc), _P, _P, _P, _P, _P, _P, _I, C.POINTER(_P)]),
    "agxc_pack_free": (None, [_P]),
    "agxc_pack_bytes": (C.c_int64, [_P]),
    "agxc_pack_unpack_dev": (_I, [_P, _P, _P]),
    "agxc_pack_dequant_dev": (_I, [_P, _P, _P]),
    "agxc_qmv": (_I, [_P, C.POINTER(QmvArgs), _P]),
    "agxc_qmv_noalloc": (_I, [_P, C.POINTER(QmvArgs), _P]),
    "agxc_qmm": (_I, [_P, _P, _P, _I, _P, _I, _I, _P]),
    "agxc_rmsnorm_dev": (_I, [_P, _P, _I, _I, _I, _P, C.c_float, _P, _P]),
    "agxc_attention_dev": (_I, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P]),
    "agxc_rope_append_dev": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, C.c_float, _P, _P, _P, _P]),
    "agxc_argmax_dev": (_I, [_P, _P, _I, _P, _P]),
    "agxc_tp_reduce_dev": (_I, [_P, _P, _I, _I, _P, _P, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _P]),
    "agxc_model_create": (_I, [_P, C.POINTER(ModelDesc), C.POINTER(_P)]),
    "agxc_tp_unique_id": (_I, [_P]),
    "agxc_model_prefill": (_I, [_P, _I, _P, _I, C.POINTER(Timing)]),
    "agxc_model_verify": (_I, [_P, _I, _P, _I, _P, C.POINTER(C.c_int32), _P]),
    "agxc_hgemm_dev": (_I, [_P, _P, _P, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P, C.c_float, _P]),
    "agxc_encoder_create": (_I, [_P, C.POINTER(EncoderDesc), C.POINTER(_P)]),
    "agxc_encoder_free": (None, [_P]),
    "agxc_encoder_set_param": (_I, [_P, _I, _I, _P, C.c_size_t, _I]),
    "agxc_encoder_forward": (_I, [_P, _P, _P, _P, _I, _I, _P, _I, C.POINTER(Timing)]),
    "agxc_encoder_profile": (_I, [_P, _I, _I, _I, _P, _P]),
    "agxc_encoder_replay": (_I, [_P, _I, _I, C.POINTER(Timing)]),
    "agxc_model_vocab_slice": (_I, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "agxc_model_free": (None, [_P]),
    "agxc_model_set_pack": (_I, [_P, _I, _I, _P, _P, _P, _I]),
    "agxc_model_set_vector": (_I, [_P, _I, _I, _P, C.c_size_t, _I]),
    "agxc_model_weight_bytes": (C.c_int64, [_P]),
    "agxc_model_start": (_I, [_P, _I, _P, _I]),
    "agxc_model_force": (_I, [_P, _I, _I, _P, _I]),
    "agxc_model_fill_history": (_I, [_P, _I, _I, C.c_uint64]),
    "agxc_decode": (_I, [_P, _I, _P, _P, _P, _I, C.POINTER(Timing)]),
    "agxc_model_state": (_I, [_P, _I, _P, _P]),
    "agxc_model_read_kv": (_I, [_P, _I, _I, _I, _P, _P]),
    "agxc_model_state_bytes": (C.c_int64, [_P, _I]),
    "agxc_model_state_save": (_I, [_P, _I, _P, C.c_size_t, C.POINTER(C.c_size_t)]),
    "agxc_model_state_restore": (_I, [_P, _I, _P, C.c_size_t]),
    "agxc_model_logits_dev": (_I, [_P, C.POINTER(_P)]),
    "agxc_model_profile": (_I, [_P, _I, _P, _P]),
    "agxc_model_set_option": (_I, [_P, _I, _I]),
    "agxc_model_plan_info": (_I, [_P, C.c_char_p, C.c_size_t]),
    "agxc_model_trace_read": (_I, [_P, C.POINTER(C.c_uint64), _I, C.POINTER(C.c_int32)]),
    "agxc_model_trace_cta_read": (_I, [_P, C.POINTER(C.c_uint64), C.c_size_t, C.POINTER(C.c_int32),
                                       C.POINTER(C.c_int32)]),
    "agxc_model_kernel_count": (_I, [_P, C.POINTER(C.c_int32)]),
}

_lib = None
_lock = threading.Lock()
_ctx = {}


def lib():
    """The loaded library (built in-tree by ``python -m agxforge_b200.build``)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise FileNotFoundError("%s: build the CUDA library first (python -m agxforge_b200.build)"
                                            % LIB_PATH)
                L = C.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    f = getattr(L, name)
                    f.restype = res
                    f.argtypes = args
                _lib = L
    return _lib


def check(rc, what=""):
    if rc == OK:
        return
    msg = lib().agxc_last_error().decode(errors="replace")
    text = "%s: %s" % (what, msg) if what else msg
    if rc == EINVAL:
        raise ValueError(text)
    if rc == ETIMEOUT:
        raise TimeoutError(text)
    if rc == ENOMEM:
        raise MemoryError(text)
    raise RuntimeError("%s (code %d)" % (text, rc))


def context(device=0):
    """The process's context on ``device`` (one stream per device)."""
    with _lock:
        h = _ctx.get(device)
    if h is None:
        L = lib()
        p = C.c_void_p()
        check(L.agxc_init(device, C.byref(p)), "agxc_init")
        with _lock:
            _ctx[device] = p
        h = p
    return h


def ctx_stream(device=0):
    """The context's own stream on ``device`` as a torch.cuda.ExternalStream (the stream the model and encoder calls
    enqueue on)."""
    import torch
    h = C.c_void_p()
    check(lib().agxc_ctx_stream(context(device), C.byref(h)), "ctx_stream")
    return torch.cuda.ExternalStream(h.value, device=device)


def ptr(t):
    """Device pointer of a torch tensor (or None)."""
    return None if t is None else C.c_void_p(t.data_ptr())
