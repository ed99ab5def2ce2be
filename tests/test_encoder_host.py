"""Host side of the encoder, on the CPU: the config admission follows the reference's refusals
(agxforge/g17/inferencegraph.py:116-157) plus this encoder's shape limits, and the MiniLM-L6 config is admitted."""
import pytest

from agxforge.inference import encoder as ENC


def test_minilm_config_admitted():
    W, L, H, F, V, P, T, eps = ENC.check_config(dict(ENC.MINILM_L6))
    assert (W, L, H, F, V, P, T) == (384, 6, 12, 1536, 30522, 512, 2) and eps == 1e-12


@pytest.mark.parametrize("change", [
    dict(model_type="qwen2"),                     # another architecture
    dict(architectures=["BertForMaskedLM"]),
    dict(hidden_act="relu"),                      # activation outside the architecture
    dict(position_embedding_type="relative_key"),
    dict(is_decoder=True),
    dict(layer_norm_eps=0),                       # a positive epsilon is required
    dict(hidden_size=0),
    dict(num_attention_heads=5),                  # head width not integral
    dict(hidden_size=384, num_attention_heads=4),  # head width 96: not 32 or 64
    dict(intermediate_size=1500),                 # ffn not a multiple of 64
])
def test_config_refusals(change):
    with pytest.raises(ValueError, match="refused"):
        ENC.check_config(dict(ENC.MINILM_L6, **change))


def test_config_must_be_a_mapping():
    with pytest.raises(ValueError, match="refused"):
        ENC.check_config([("model_type", "bert")])
