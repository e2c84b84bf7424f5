"""LlamaConfig.fromJson's strict subset (models/src/main/scala/scalatorch/models/LlamaConfig.scala:44-112),
checked on the host: every unsupported option or malformed field raises IllegalArgumentException
before any device work (the cases of LlamaSuite.scala:11-21, plus the token-id and head rules)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "scala-torch_b200"))

from scalatorch.ffm import IllegalArgumentException  # noqa: E402
from scalatorch.models import LlamaConfig, llama_weight_shapes  # noqa: E402

BASE = ('{"model_type":"llama","vocab_size":8,"hidden_size":4,"intermediate_size":8,"num_hidden_layers":1,'
        '"num_attention_heads":2,"num_key_value_heads":1,"max_position_embeddings":16,"bos_token_id":1,'
        '"eos_token_id":2} ')


def with_field(extra: str) -> str:
    return BASE.strip()[:-1] + "," + extra + "}"


def test_supported_config_parses():
    c = LlamaConfig.from_json(BASE)
    assert (c.head_dim, c.num_key_value_heads, c.max_positions) == (2, 1, 16)
    assert c.eos_token_ids == (2,) and c.bos_token_id == 1 and not c.tie_word_embeddings
    assert LlamaConfig.from_json(with_field('"head_dim":2')).head_dim == 2  # the implied width is accepted
    assert LlamaConfig.from_json(BASE.replace('"eos_token_id":2', '"eos_token_id":[2,3]')).eos_token_ids == (2, 3)
    assert LlamaConfig.from_json(BASE.replace('"eos_token_id":2', '"eos_token_id":null')).eos_token_ids == ()


@pytest.mark.parametrize("extra", ['"rope_scaling":{}', '"attention_bias":true', '"hidden_act":"relu"',
                                   '"sliding_window":4', '"head_dim":4', '"partial_rotary_factor":0.5',
                                   '"mlp_bias":true', '"pretraining_tp":2', '"attention_dropout":0.1'])
def test_unsupported_options_reject(extra):
    with pytest.raises(IllegalArgumentException):
        LlamaConfig.from_json(with_field(extra))


@pytest.mark.parametrize("text", [
    BASE.replace('"hidden_size":4', '"hidden_size":4.0'),                      # fractional integer
    BASE.replace('"hidden_size":4', '"hidden_size":4,"hidden_size":4'),        # duplicate key
    BASE.replace('"num_attention_heads":2', '"num_attention_heads":3'),        # heads do not divide hidden
    BASE.replace('"num_key_value_heads":1', '"num_key_value_heads":3'),        # KV heads do not divide heads
    BASE.replace('"model_type":"llama"', '"model_type":"mistral"'),
    BASE.replace('"eos_token_id":2', '"eos_token_id":8'),                      # outside the vocabulary
    BASE.replace('"vocab_size":8', '"vocab_size":-8'),
    BASE.replace('"num_hidden_layers":1', '"num_hidden_layers":true'),         # boolean is not an integer
    "[1, 2]",
    "{",
    BASE.replace('"eos_token_id":2', '"eos_token_id":[2,"3"]'),               # EOS ids must be integers
    BASE.replace('"eos_token_id":2', '"eos_token_id":[2,true]'),
    BASE.replace('"bos_token_id":1', '"bos_token_id":"1"'),
    with_field('"tie_word_embeddings":"true"'),                              # booleans are JSON booleans
    with_field('"rms_norm_eps":NaN'),                                        # non-finite constants
    with_field('"rope_theta":Infinity'),
    with_field('"initializer_range":-0.5'),
    BASE.replace('"vocab_size":8,', ''),                                     # required field missing
])
def test_malformed_configs_reject(text):
    with pytest.raises(IllegalArgumentException):
        LlamaConfig.from_json(text)


def test_weight_shapes_follow_the_config():
    """LlamaModel.shapes (LlamaModel.scala:115-128): (out, in) per projection, KV width = kv heads x
    head width, norms [hidden]."""
    c = LlamaConfig.from_json(BASE)
    shapes = llama_weight_shapes(c)
    assert shapes["model.embed_tokens.weight"] == (8, 4) and shapes["lm_head.weight"] == (8, 4)
    assert shapes["model.layers.0.self_attn.k_proj.weight"] == (2, 4)
    assert shapes["model.layers.0.mlp.down_proj.weight"] == (4, 8)
    assert shapes["model.layers.0.input_layernorm.weight"] == (4,)
    assert len(shapes) == 3 + 9 * c.num_layers


def test_configs_over_one_mib_reject():
    with pytest.raises(IllegalArgumentException):
        LlamaConfig.from_json(with_field('"pad":"' + "x" * 1048576 + '"'))


def test_random_field_values_fail_only_as_invalid_arguments():
    """Any JSON value in any recognised field either parses into a valid LlamaConfig or raises
    IllegalArgumentException, never another exception type."""
    import json

    from hypothesis import given, settings
    from hypothesis import strategies as st

    keys = ["vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "max_position_embeddings", "rms_norm_eps", "rope_theta", "tie_word_embeddings",
            "bos_token_id", "eos_token_id", "initializer_range", "head_dim", "hidden_act", "attention_dropout",
            "pretraining_tp", "rope_scaling", "model_type"]
    scalars = st.one_of(st.none(), st.booleans(), st.integers(-3, 40), st.floats(allow_nan=False, width=32),
                        st.sampled_from(["llama", "silu", "relu", ""]))
    values = st.one_of(scalars, st.lists(scalars, max_size=3), st.dictionaries(st.sampled_from(["a"]), scalars))
    base = json.loads(BASE)

    @settings(max_examples=500, deadline=None)
    @given(st.dictionaries(st.sampled_from(keys), values, max_size=4))
    def check(changes):
        doc = dict(base, **changes)
        try:
            c = LlamaConfig.from_json(json.dumps(doc))
        except IllegalArgumentException:
            return
        assert c.hidden_size % c.num_attention_heads == 0 and c.head_dim % 2 == 0

    check()
