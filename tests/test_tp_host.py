"""Host side of tensor parallelism, on the CPU: the rank slices of reference-format packs are exactly the packs of
the sliced matrices (rows of the qkv heads, o_proj and down columns, gate/up rows, vocabulary tiles), the vocabulary
split covers the head, and the communicator-id exchange over torch.distributed (gloo, world size 2) gives every rank
rank 0's bytes — or fails within the process group's timeout when a rank never joins (no GPU involved)."""
import datetime
import os
import socket

import numpy as np
import pytest

from agxforge.inference import models
from agxforge.inference import tp as TP
from oracle import pack as OP


def _pack(N, K, bits, seed):
    W = np.random.default_rng(seed).standard_normal((N, K)).astype(np.float32) * 0.02
    packed, s, b, q = OP.quantize(W, bits=bits, scale_dtype="fp16")
    return (packed, s, b), q


def _fields(pack, bits, N, K):
    return OP.unpack(pack[0], bits, N, K), pack[1], pack[2]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("bits", [4, 8])
def test_shards_are_the_sliced_matrices(world, bits):
    S = models.Model("t", 256, 1, 8, 8, 64, 1024, 2048, 1e6, 1e-6)
    hd, H, KVH, F, d, V = S.HEAD_DIM, S.HEADS, S.KV_HEADS, S.FFN, S.D_MODEL, S.VOCAB
    qkv, qq = _pack((H + 2 * KVH) * hd, d, bits, 1)
    wo, qo = _pack(d, H * hd, bits, 2)
    up, qu = _pack(F, d, bits, 3)
    down, qd = _pack(d, F, bits, 4)
    head, qh = _pack(V, d, bits, 5)
    hq, hk, fl = H // world, KVH // world, F // world
    seen_v = []
    for r in range(world):
        # qkv: the rank's q heads, then its k heads, then its v heads
        sh = TP.shard_pack("qkv", qkv, S, bits, world, r)
        rows = np.r_[r * hq * hd:(r + 1) * hq * hd, H * hd + r * hk * hd:H * hd + (r + 1) * hk * hd,
                     (H + KVH) * hd + r * hk * hd:(H + KVH) * hd + (r + 1) * hk * hd]
        q, s, b = _fields(sh, bits, len(rows), d)
        assert np.array_equal(q, qq[rows]) and np.array_equal(s, qkv[1][rows]) and np.array_equal(b, qkv[2][rows])
        # o_proj: the columns of the rank's q heads
        sh = TP.shard_pack("wo", wo, S, bits, world, r)
        c0, c1 = r * hq * hd, (r + 1) * hq * hd
        q, s, b = _fields(sh, bits, d, c1 - c0)
        assert np.array_equal(q, qo[:, c0:c1]) and np.array_equal(s, wo[1][:, c0 // 64:c1 // 64])
        # gate/up rows and down columns of the rank's ffn range
        sh = TP.shard_pack("up", up, S, bits, world, r)
        assert np.array_equal(_fields(sh, bits, fl, d)[0], qu[r * fl:(r + 1) * fl])
        sh = TP.shard_pack("down", down, S, bits, world, r)
        q, s, b = _fields(sh, bits, d, fl)
        assert np.array_equal(q, qd[:, r * fl:(r + 1) * fl]) and np.array_equal(b, down[2][:, r * fl // 64:(r + 1) * fl // 64])
        # head: whole 128-row tiles
        v0, vn = TP.vocab_slice(V, world, r)
        assert v0 % 128 == 0 and vn % 128 == 0 and vn > 0
        sh = TP.shard_pack("head", head, S, bits, world, r)
        assert np.array_equal(_fields(sh, bits, vn, d)[0], qh[v0:v0 + vn])
        seen_v.append((v0, vn))
    # the slices tile the vocabulary in order
    assert seen_v[0][0] == 0 and all(a[0] + a[1] == b[0] for a, b in zip(seen_v, seen_v[1:]))
    assert seen_v[-1][0] + seen_v[-1][1] == V


def test_vocab_slice_of_the_baseline_vocabulary():
    V = models.INTERNLM25_7B.VOCAB  # 92,544 = 723 tiles: uneven over 2, 4, 8 ranks
    for world in (2, 4, 8):
        sl = [TP.vocab_slice(V, world, r) for r in range(world)]
        assert sum(n for _, n in sl) == V
        assert max(n for _, n in sl) - min(n for _, n in sl) <= 128


def test_bias_shard():
    S = models.Model("t", 256, 1, 8, 4, 64, 1024, 2048, 1e6, 1e-6, True)
    bias = np.arange((8 + 2 * 4) * 64, dtype=np.float32)
    parts = [TP.shard_bias(bias, S, 2, r) for r in range(2)]
    assert np.array_equal(parts[0][:4 * 64], bias[:256]) and np.array_equal(parts[1][:4 * 64], bias[256:512])
    assert np.array_equal(parts[0][256:384], bias[512:640]) and np.array_equal(parts[1][384:], bias[896:])


def test_check_rejects_unsplittable_shapes():
    S = models.INTERNLM25_7B
    TP.check(S, 8, 64)
    with pytest.raises(ValueError):
        TP.check(S, 3, 64)
    with pytest.raises(ValueError):
        TP.check(S, 2, 8)            # the GEMV step (batch <= 8) is single-device
    with pytest.raises(ValueError):
        TP.check(models.Model("t", 256, 1, 6, 6, 64, 1024, 2048, 1e6, 1e-6), 4, 32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_dir):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    path = os.path.join(out_dir, "rank%d" % rank)
    try:
        if mode == "absent" and rank == 1:
            os._exit(0)  # this rank leaves before the exchange: rank 0 must not wait for it for good
        uid = TP.exchange_id(world, rank, make_id=lambda: bytes(range(128)))
        with open(path, "wb") as f:
            f.write(uid)
    except Exception as e:  # noqa: BLE001 - the error is the result
        with open(path + ".err", "w") as f:
            f.write(type(e).__name__ + ": " + str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _spawn(mode, tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, mode, str(tmp_path)), nprocs=2, join=True, start_method="spawn")


def test_exchange_id_two_ranks(tmp_path):
    _spawn("ok", tmp_path)
    for r in range(2):
        assert (tmp_path / ("rank%d" % r)).read_bytes() == bytes(range(128))


def test_exchange_id_fails_when_a_rank_never_joins(tmp_path):
    _spawn("absent", tmp_path)
    assert not (tmp_path / "rank0").exists()
    assert (tmp_path / "rank0.err").exists()
