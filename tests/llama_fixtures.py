"""Oracle-side copies of the device Llama's synthetic weights (same generator, same streams)."""
import numpy as np

import oracle
from scalatorch.models import (LlamaConfig, W_DOWN, W_EMBED, W_GATE, W_K, W_LM_HEAD, W_O, W_Q, W_UP, W_V,
                               weight_stream)

TINY = dict(vocab_size=1000, hidden_size=64, intermediate_size=128, num_layers=2, num_attention_heads=4,
            num_key_value_heads=2, max_positions=64, tie_word_embeddings=False, eos_token_ids=())
SMOL = dict(vocab_size=49152, hidden_size=576, intermediate_size=1536, num_layers=30, num_attention_heads=9,
            num_key_value_heads=3, max_positions=2048, tie_word_embeddings=True, rope_theta=10000.0,
            rms_norm_eps=1e-6, eos_token_ids=())


def bf16_matrix(seed, which, layer, rows, cols, std):
    return oracle.normal_bf16(rows * cols, seed, weight_stream(which, layer), std).reshape(rows, cols)


def named_bf16_weights(config: LlamaConfig, seed: int):
    """name -> BF16 bits, exactly what stb_llama_init_random generates."""
    c, std = config, config.initializer_range
    H, I, V, kvd = c.hidden_size, c.intermediate_size, c.vocab_size, c.num_key_value_heads * c.head_dim
    out = {"model.embed_tokens.weight": bf16_matrix(seed, W_EMBED, 0, V, H, std),
           "model.norm.weight": oracle.round_bf16(np.ones(H, np.float32))}
    if not c.tie_word_embeddings:
        out["lm_head.weight"] = bf16_matrix(seed, W_LM_HEAD, 0, V, H, std)
    for l in range(c.num_layers):
        p = f"model.layers.{l}"
        out[f"{p}.input_layernorm.weight"] = oracle.round_bf16(np.ones(H, np.float32))
        out[f"{p}.post_attention_layernorm.weight"] = oracle.round_bf16(np.ones(H, np.float32))
        for name, which, rows, cols in (("self_attn.q_proj", W_Q, H, H), ("self_attn.k_proj", W_K, kvd, H),
                                        ("self_attn.v_proj", W_V, kvd, H), ("self_attn.o_proj", W_O, H, H),
                                        ("mlp.gate_proj", W_GATE, I, H), ("mlp.up_proj", W_UP, I, H),
                                        ("mlp.down_proj", W_DOWN, H, I)):
            out[f"{p}.{name}.weight"] = bf16_matrix(seed, which, l, rows, cols, std)
    return out


def oracle_model(config: LlamaConfig, seed: int, threads: int = 0, replace: dict | None = None) -> oracle.OracleLlama:
    """The reference CPU path's view of the same model: weights widened to Float32 (SafeTensors.readFloat).
    replace: name -> BF16 bits of tensors uploaded over the generated ones (BackendLlama.set_weight)."""
    named = named_bf16_weights(config, seed)
    named.update(replace or {})
    wide = {k: oracle.widen(v, oracle.BF16) for k, v in named.items()}
    embed = wide["model.embed_tokens.weight"]
    head = embed if config.tie_word_embeddings else wide["lm_head.weight"]
    layers = []
    for l in range(config.num_layers):
        p = f"model.layers.{l}"
        layers.append({"in_norm": wide[f"{p}.input_layernorm.weight"], "post_norm": wide[f"{p}.post_attention_layernorm.weight"],
                       "q": wide[f"{p}.self_attn.q_proj.weight"], "k": wide[f"{p}.self_attn.k_proj.weight"],
                       "v": wide[f"{p}.self_attn.v_proj.weight"], "o": wide[f"{p}.self_attn.o_proj.weight"],
                       "gate": wide[f"{p}.mlp.gate_proj.weight"], "up": wide[f"{p}.mlp.up_proj.weight"],
                       "down": wide[f"{p}.mlp.down_proj.weight"]})
    return oracle.OracleLlama(_OracleCfg(config), oracle.LlamaWeights(embed, wide["model.norm.weight"], head, layers),
                              threads)


class _OracleCfg:
    def __init__(self, c: LlamaConfig):
        self.vocab_size, self.hidden_size, self.intermediate_size = c.vocab_size, c.hidden_size, c.intermediate_size
        self.num_layers, self.num_attention_heads = c.num_layers, c.num_attention_heads
        self.num_key_value_heads, self.max_positions = c.num_key_value_heads, c.max_positions
        self.tie_word_embeddings, self.rms_norm_eps, self.rope_theta = c.tie_word_embeddings, c.rms_norm_eps, c.rope_theta
