"""The encoder oracle (oracle/encoder.py) pinned against the reference's own complete-encoder reference (golden
vectors of tools/g17inferencereference.py ``graph_reference``, both FP64 policies, made by
tests/golden/make_minilm_golden.py) and against transformers' BertModel in float64 as an independent framework
control; the batched form [B, S] equals the per-sequence form."""
import os

import numpy as np
import pytest

from oracle import encoder as E

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "minilm_ref.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


@pytest.fixture(scope="module")
def params():
    return E.make_params(1)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_oracle_matches_reference_graph_policies(gold, params, case):
    ids = gold["case%d_token_ids" % case][None]
    mask = gold["case%d_mask" % case][None]
    for policy, name in (("fp64", "original_fp64"), ("half", "half_transport_fp64")):
        got = E.forward(params, ids, mask, policy=policy)[0]
        ref = gold["case%d_%s_embedding" % (case, name)]
        assert np.abs(got - ref).max() < 1e-12, (policy, np.abs(got - ref).max())


def test_oracle_last_hidden_rows(gold, params):
    _, x = E.forward(params, gold["case0_token_ids"][None], gold["case0_mask"][None], keep=True)
    assert np.abs(x[0] - gold["case0_original_fp64_last_hidden"]).max() < 1e-10


def test_policies_differ_but_agree_in_cosine(gold, params):
    a = gold["case1_original_fp64_embedding"]
    b = gold["case1_half_transport_fp64_embedding"]
    assert np.abs(a - b).max() > 0           # the half transport does round
    assert E.cosine(a, b) > 0.9999


def test_batched_form_equals_per_sequence(gold, params):
    ids = np.stack([gold["case%d_token_ids" % c] for c in range(3)])
    mask = np.stack([gold["case%d_mask" % c] for c in range(3)])
    emb = E.forward(params, ids, mask, policy="half")
    for c in range(3):
        assert np.abs(emb[c] - gold["case%d_half_transport_fp64_embedding" % c]).max() < 1e-12


def test_framework_control_transformers_bert():
    """transformers' BertModel (float64, eager attention, padding mask) on a 2-layer MiniLM-width model: its last
    hidden rows equal the oracle's."""
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    cfg = dict(num_hidden_layers=2, vocab_size=1000, max_position_embeddings=64)
    p = E.make_params(5, cfg)
    c = dict(E.MINILM_L6, **cfg)
    bc = tr.BertConfig(hidden_size=c["hidden_size"], num_attention_heads=c["num_attention_heads"],
                       intermediate_size=c["intermediate_size"], num_hidden_layers=2, vocab_size=1000,
                       max_position_embeddings=64, type_vocab_size=2, layer_norm_eps=1e-12, hidden_act="gelu",
                       attn_implementation="eager")
    model = tr.BertModel(bc, add_pooling_layer=False).double().eval()
    sd = {k: torch.from_numpy(np.asarray(v, np.float64)) for k, v in p.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("position_ids" in m for m in missing)
    rng = np.random.default_rng(6)
    ids = rng.integers(0, 1000, (3, 24))
    mask = np.ones((3, 24), np.int64)
    mask[1, 17:] = 0
    mask[2, 5:] = 0
    with torch.inference_mode():
        ref = model(input_ids=torch.from_numpy(ids), attention_mask=torch.from_numpy(mask),
                    token_type_ids=torch.zeros_like(torch.from_numpy(ids))).last_hidden_state.numpy()
    _, x = E.forward(p, ids, mask, config=cfg, keep=True)
    assert np.abs(x - ref).max() < 1e-10
