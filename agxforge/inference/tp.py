"""Tensor parallelism of the decode step over the GPUs of one node (the reference runs one device and has no
counterpart; this follows the partitioning its decoder layer admits).

Rank r of t holds: query heads [r H/t, (r+1) H/t) and KV heads [r KVH/t, (r+1) KVH/t) (their qkv rows, bias entries
and KV cache), the o_proj columns of its query heads, gate and up rows [r F/t, (r+1) F/t) and the down columns of the
same range, and a slice of the vocabulary head in 128-row tiles (`vocab_slice`). RMSNorm gains, the embedding table
and the residual stream are replicated. Per layer the o_proj and down partial sums are all-reduced (fp32 sum) before
their residual; the head's per-rank first maxima are all-gathered before the token choice. Group-64 quantisation runs
along K, so row slices and 64-aligned column slices of a reference-format pack (packed uint32 [N, K bits/32], 16-bit
scale and bias [N, K/64]) are exactly the packs of the sliced matrices.

    vocab_slice(vocab, world, rank)      (first token id, count) of the rank's head rows
    shard_pack(role, pack, shape, bits, world, rank)   the rank's reference-format pack of one projection
    shard_bias(bias, shape, world, rank)               the rank's qkv bias entries
    exchange_id(world, rank)             rank 0's communicator id, the same 128 bytes on every rank
"""
from __future__ import annotations

import numpy as np


def vocab_slice(vocab, world, rank):
    """The rank's head rows [first, first + count): whole 128-row tiles, split as evenly as the tiles allow (the
    library's own rule)."""
    if world <= 1:
        return 0, vocab
    if vocab % 128:
        raise ValueError("vocab_slice: vocab must be a multiple of 128 under tensor parallelism")
    tiles = vocab // 128
    t0 = tiles * rank // world
    t1 = tiles * (rank + 1) // world
    return 128 * t0, 128 * (t1 - t0)


def check(shape, world, batch):
    """ValueError unless the shape splits over `world` ranks (the library's checks, before any device work)."""
    if world not in (1, 2, 4, 8):
        raise ValueError("tensor parallelism: tp 1, 2, 4 or 8")
    if world == 1:
        return
    if batch < 32:
        raise ValueError("tensor parallelism: batch >= 32 (the tensor-core GEMM step)")
    if shape.HEADS % world or shape.KV_HEADS % world:
        raise ValueError("tensor parallelism: heads and KV heads divisible by tp")
    if shape.FFN % (64 * world):
        raise ValueError("tensor parallelism: ffn divisible by 64 x tp")
    if shape.VOCAB % 128 or shape.VOCAB // 128 < world:
        raise ValueError("tensor parallelism: vocab a multiple of 128 with at least one 128-row tile per rank")


def _cat(parts):
    if isinstance(parts[0], np.ndarray):
        return np.ascontiguousarray(np.concatenate(parts, axis=0))
    import torch
    return torch.cat(parts, dim=0).contiguous()


def _rows(pack, r0, r1):
    return tuple(a[r0:r1] for a in pack)


def _cols(pack, k0, k1, bits):
    p, s, b = pack
    w = 32 // bits
    sl = (lambda a, i, j: np.ascontiguousarray(a[:, i:j])) if isinstance(p, np.ndarray) else \
        (lambda a, i, j: a[:, i:j].contiguous())
    return sl(p, k0 // w, k1 // w), sl(s, k0 // 64, k1 // 64), sl(b, k0 // 64, k1 // 64)


def _qkv_ranges(shape, world, rank):
    hd = shape.HEAD_DIM
    hq, hk = shape.HEADS // world, shape.KV_HEADS // world
    q = (rank * hq * hd, (rank + 1) * hq * hd)
    k0 = shape.HEADS * hd
    k = (k0 + rank * hk * hd, k0 + (rank + 1) * hk * hd)
    v0 = k0 + shape.KV_HEADS * hd
    v = (v0 + rank * hk * hd, v0 + (rank + 1) * hk * hd)
    return q, k, v


def shard_pack(role, pack, shape, bits, world, rank):
    """The rank's slice of a global reference-format pack (packed, scales, biases) of `role` (qkv, wo, gate, up,
    down, head); torch tensors or numpy arrays, returned the same kind."""
    if world <= 1:
        return pack
    hd = shape.HEAD_DIM
    if role == "qkv":
        parts = [_rows(pack, a, b) for a, b in _qkv_ranges(shape, world, rank)]
        return tuple(_cat([pt[i] for pt in parts]) for i in range(3))
    if role == "wo":
        hq = shape.HEADS // world
        return _cols(pack, rank * hq * hd, (rank + 1) * hq * hd, bits)
    fl = shape.FFN // world
    if role in ("gate", "up"):
        return tuple(a.contiguous() if hasattr(a, "contiguous") else np.ascontiguousarray(a)
                     for a in _rows(pack, rank * fl, (rank + 1) * fl))
    if role == "down":
        return _cols(pack, rank * fl, (rank + 1) * fl, bits)
    if role == "head":
        v0, vn = vocab_slice(shape.VOCAB, world, rank)
        return tuple(a.contiguous() if hasattr(a, "contiguous") else np.ascontiguousarray(a)
                     for a in _rows(pack, v0, v0 + vn))
    raise ValueError("shard_pack: unknown role %r" % (role,))


def shard_bias(bias, shape, world, rank):
    """The rank's entries of the qkv bias (the rows of its heads)."""
    if world <= 1:
        return bias
    return _cat([bias[a:b] for a, b in _qkv_ranges(shape, world, rank)])


def exchange_id(world, rank, make_id=None, group=None):
    """Rank 0 makes the communicator id (`make_id()`, default the library's agxc_tp_unique_id) and every rank
    receives the same 128 bytes over torch.distributed (which must be initialised; any backend)."""
    import torch.distributed as dist
    if make_id is None:
        def make_id():
            import ctypes as C
            from agxforge_b200 import _native as N
            buf = (C.c_uint8 * 128)()
            N.check(N.lib().agxc_tp_unique_id(buf), "tp_unique_id")
            return bytes(buf)
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("exchange_id: expected 128 bytes from rank 0")
    return bytes(uid)
