"""The MiniLM sentence encoder on the B200.

* the tensor-core GEMM (agxc_hgemm_dev) against torch fp32 matmuls of the same fp16 operands, every epilogue;
* the reference's golden vectors (tools/g17inferencereference.py graph_reference, 32-token sequences with 32, 20 and 7
  valid tokens, MiniLM-L6 with seeded parameters): |got - half_transport_fp64| <= 2e-4 (1 + |ref|) and cosine >= 0.999
  against original_fp64 — the reference's own contract (g17inferencereference.py:155);
* the BASELINE workload (32 sequences x 128 tokens, valid lengths 16..128) against the FP64 oracle under the same
  bound;
* the device-pointer path equals the host path; inputs outside their domain are refused."""
import os

import numpy as np
import pytest

from oracle import encoder as E

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "minilm_ref.npz")


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


@pytest.fixture(scope="module")
def enc(torch):
    from agxforge.inference.encoder import Encoder
    e = Encoder(E.MINILM_L6, max_batch=32, max_seq=128).load(E.make_params(1))
    yield e
    e.close()


@pytest.mark.parametrize("M,N,K,epi", [(m, n, k, e) for (m, n, k) in [(128, 64, 64), (256, 1152, 384),
                                                                      (4096, 384, 1536), (384, 1536, 384)]
                                         for e in (0, 1, 2)] + [(256, 384, 384, 3), (4096, 384, 1536, 3),
                                                                (128, 128, 64, 3), (256, 256, 256, 3)])
def test_hgemm_against_torch(torch, M, N, K, epi):
    import ctypes as C
    from agxforge_b200 import _native as N_
    from agxforge.kernels import qmv as Q
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi)
    A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).half()
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    bias = (torch.randn(N, device="cuda", generator=g) * 0.1).half()
    res = torch.randn(M, N, device="cuda", generator=g)
    out32 = torch.full((M, N), float("nan"), device="cuda")
    out16 = torch.full((M, N), float("nan"), device="cuda").half()
    ref = A.float() @ W.float().T + bias.float()
    g1 = (1 + 0.1 * torch.randn(N, device="cuda", generator=g)).half()
    b1 = (0.1 * torch.randn(N, device="cuda", generator=g)).half()
    if epi == 3:
        out32 = res.clone()  # in place over the residual, as the encoder runs it
    N_.check(N_.lib().agxc_hgemm_dev(N_.context(0), C.c_void_p(A.data_ptr()), C.c_void_p(W.data_ptr()), M, N, K,
                                     C.c_void_p(bias.data_ptr()), epi, C.c_void_p(out32.data_ptr()),
                                     C.c_void_p(out16.data_ptr()),
                                     C.c_void_p(out32.data_ptr() if epi == 3 else res.data_ptr()),
                                     C.c_void_p(g1.data_ptr()), C.c_void_p(b1.data_ptr()), C.c_float(1e-12),
                                     Q._stream(torch)),  # torch's stream: ordered after the operands' writes
             "hgemm")
    torch.cuda.synchronize()
    # fp32 accumulation of exact fp16 products: only the summation order differs from the reference matmul
    tol = 1e-5 * (A.float().abs() @ W.float().abs().T).max().item() + 1e-6
    if epi == 0:
        assert (out32 - ref).abs().max().item() <= tol
    elif epi == 1:
        want = torch.nn.functional.gelu(ref, approximate="none")
        err = (out16.float() - want).abs()
        assert (err <= tol + 2 ** -10 * want.abs() + 1e-7).all(), err.max().item()
    elif epi == 2:
        assert (out32 - (ref + res)).abs().max().item() <= tol + 1e-6
    else:
        x = ref + res
        c = x - x.mean(-1, keepdim=True)
        want = c / torch.sqrt((c * c).mean(-1, keepdim=True) + 1e-12) * g1.float() + b1.float()
        scale = 1.0 / torch.sqrt((c * c).mean(-1, keepdim=True))
        assert ((out32 - want).abs() <= 4 * (tol + 1e-6) * scale * g1.float().abs() + 1e-5).all()
        assert ((out16.float() - want).abs() <= 4 * (tol + 1e-6) * scale * g1.float().abs() + 2 ** -10 *
                want.abs() + 1e-5).all()


def test_reference_golden_vectors(enc):
    gold = np.load(GOLD)
    ids = np.stack([gold["case%d_token_ids" % c] for c in range(3)])
    mask = np.stack([gold["case%d_mask" % c] for c in range(3)])
    got = enc.forward(dict(token_ids=ids, attention_mask=mask))
    for c in range(3):
        half = gold["case%d_half_transport_fp64_embedding" % c]
        orig = gold["case%d_original_fp64_embedding" % c]
        assert E.within_bound(got[c], half).all(), np.abs(got[c] - half).max()
        assert E.cosine(got[c], orig) >= 0.999


def _workload(seed=1, B=32, S=128, V=30522):
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, V, (B, S)).astype(np.int32)
    lens = rng.integers(16, S + 1, B)
    mask = (np.arange(S)[None, :] < lens[:, None]).astype(np.int32)
    return ids, mask


def test_baseline_workload_against_oracle(enc):
    ids, mask = _workload()
    got, t = enc.forward(dict(token_ids=ids, attention_mask=mask), timing=True)
    params = E.make_params(1)
    half = E.forward(params, ids, mask, policy="half")
    orig = E.forward(params, ids, mask, policy="fp64")
    assert E.within_bound(got, half).all(), np.abs(got - half).max()
    for b in range(32):
        assert E.cosine(got[b], orig[b]) >= 0.999
    assert t["launches"] == 1 + 7 * 6 + 1  # embedding, per layer qkv / attention / o / LN / up / down / LN, pooling


def test_token_types_and_shorter_batches(enc):
    ids, mask = _workload(seed=3, B=5, S=40)
    types = (np.arange(40)[None, :] >= 20).astype(np.int32).repeat(5, 0)
    got = enc.forward(dict(token_ids=ids, attention_mask=mask, token_type_ids=types))
    ref = E.forward(E.make_params(1), ids, mask, token_type_ids=types, policy="half")
    assert E.within_bound(got, ref).all()


def test_device_path_equals_host_path(torch, enc):
    ids, mask = _workload(seed=4, B=8, S=64)
    host = enc.forward(dict(token_ids=ids, attention_mask=mask))
    dev = enc.forward_device(torch.from_numpy(ids).cuda(), torch.from_numpy(mask).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


def test_refusals(enc):
    ids, mask = _workload(seed=5, B=2, S=32)
    bad = mask.copy()
    bad[1] = 0
    with pytest.raises(ValueError):
        enc.forward(dict(token_ids=ids, attention_mask=bad))          # a sequence without a valid token
    with pytest.raises(ValueError):
        enc.forward(dict(token_ids=ids, attention_mask=mask * 2))     # mask values 0/1
    with pytest.raises(ValueError):
        enc.forward(dict(token_ids=ids + 30522, attention_mask=mask))  # ids outside the vocabulary
    with pytest.raises(ValueError):
        enc.forward(dict(token_ids=ids, attention_mask=mask, position_ids=np.arange(32)[::-1]))
    with pytest.raises(ValueError):
        enc.forward(dict(token_ids=np.zeros((33, 8), np.int32), attention_mask=np.ones((33, 8), np.int32)))


def test_long_sequences_fp32_attention_path(torch):
    """Sequences longer than 128 tokens take the fp32 CUDA-core attention (the tensor-core kernel holds a whole
    score row of at most 128 keys in registers); both paths meet the same bound."""
    from agxforge.inference.encoder import Encoder
    cfg = dict(E.MINILM_L6, num_hidden_layers=2)
    e = Encoder(cfg, max_batch=4, max_seq=200).load(E.make_params(7, cfg))
    ids, mask = _workload(seed=8, B=4, S=200)
    for S in (200, 128, 50):
        got = e.forward(dict(token_ids=ids[:, :S], attention_mask=mask[:, :S]))
        ref = E.forward(E.make_params(7, cfg), ids[:, :S], mask[:, :S], policy="half", config=cfg)
        assert E.within_bound(got, ref).all(), (S, np.abs(got - ref).max())
    e.close()


def test_large_batch_fused_layernorm_epilogue(torch):
    """Enough token rows for one full wave of 128-row tiles: o_proj and FFN down carry the LayerNorm in their
    epilogue (5 launches a layer instead of 7), within the same bound."""
    from agxforge.inference.encoder import Encoder
    cfg = dict(E.MINILM_L6, num_hidden_layers=2)
    B, S = 152, 128                                   # 19,456 rows = 152 tiles >= 148 SMs
    e = Encoder(cfg, max_batch=B, max_seq=S).load(E.make_params(9, cfg))
    ids, mask = _workload(seed=10, B=B, S=S)
    got, t = e.forward(dict(token_ids=ids, attention_mask=mask), timing=True)
    assert t["launches"] == 1 + 5 * 2 + 1
    ref = E.forward(E.make_params(9, cfg), ids, mask, policy="half", config=cfg)
    assert E.within_bound(got, ref).all(), np.abs(got - ref).max()
    e.close()
