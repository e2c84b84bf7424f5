"""The reference's per-op Llama on the CPU backend, composed from the oracle's restated ops.

TEST INFRASTRUCTURE ONLY: the checker for PerOpLlama (scalatorch.models).  It runs
BackendLlama.run (models/src/main/scala/scalatorch/models/BackendLlama.scala:41-111) with
CpuFloatBackend's operations (cpu/src/main/scala/scalatorch/cpu/CpuFloatBackend.scala): numscala
matmul (oracle.linear / oracle.matmul_tr), Float32 add / multiply / scale (numpy float32, one IEEE
rounding each), SiLU / RMSNorm / RoPE / attention in double (the oracle's C restatements), reshape
and transpose as exact copies.
"""
import numpy as np

import oracle

LAYER = (("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"), ("v", "self_attn.v_proj"), ("o", "self_attn.o_proj"),
         ("gate", "mlp.gate_proj"), ("up", "mlp.up_proj"), ("down", "mlp.down_proj"))


class CpuPerOpLlama:
    """weights: name -> BF16 bits (uint16); lora: projection name -> (A, B, alpha)."""

    def __init__(self, config, weights: dict, lora: dict | None = None):
        self.c = config
        self.w = weights
        self.lora = lora or {}
        self.embed = oracle.widen(weights["model.embed_tokens.weight"], oracle.BF16)

    def _linear(self, x, name):
        w = self.w[name + ".weight"]
        base = oracle.linear(x, w, oracle.BF16)
        if name not in self.lora:
            return base
        a, b, alpha = self.lora[name]
        low = oracle.matmul_tr(x, a)
        delta = oracle.matmul_tr(low, b)
        scaled = delta * np.float32(alpha / a.shape[0])
        return (base + scaled).astype(np.float32)

    def _norm(self, x, name):
        w = oracle.widen(self.w[name], oracle.BF16)
        return oracle.rmsnorm(x, w, self.c.rms_norm_eps)

    def forward(self, tokens, position, caches):
        c = self.c
        ids = np.asarray(tokens, np.int64)
        b, t = ids.shape
        hd = c.head_dim
        hidden = self.embed[ids]  # (b, t, H)
        for i in range(c.num_layers):
            p = f"model.layers.{i}"
            x = self._norm(hidden, f"{p}.input_layernorm.weight")
            flat = x.reshape(b * t, c.hidden_size)

            def heads(name, count):
                return np.ascontiguousarray(self._linear(flat, f"{p}.{name}").reshape(b, t, count, hd).transpose(0, 2, 1, 3))

            q = oracle.rope(heads("self_attn.q_proj", c.num_attention_heads), position, c.rope_theta)
            k = oracle.rope(heads("self_attn.k_proj", c.num_key_value_heads), position, c.rope_theta)
            v = heads("self_attn.v_proj", c.num_key_value_heads)
            kc, vc = caches[i]
            kc[:, :, position:position + t] = k
            vc[:, :, position:position + t] = v
            att = oracle.causal_attention(q, kc, vc, start=position, key_stride=kc.shape[2], keys=position + t)
            matrix = np.ascontiguousarray(att.transpose(0, 2, 1, 3)).reshape(b * t, c.hidden_size)
            attended = self._linear(matrix, f"{p}.self_attn.o_proj").reshape(b, t, c.hidden_size)
            hidden = (hidden + attended).astype(np.float32)
            post = self._norm(hidden, f"{p}.post_attention_layernorm.weight").reshape(b * t, c.hidden_size)
            gate = self._linear(post, f"{p}.mlp.gate_proj")
            act = oracle.silu(gate)
            up = self._linear(post, f"{p}.mlp.up_proj")
            down = self._linear((act * up).astype(np.float32), f"{p}.mlp.down_proj").reshape(b, t, c.hidden_size)
            hidden = (hidden + down).astype(np.float32)
        normalized = self._norm(hidden, "model.norm.weight").reshape(b * t, c.hidden_size)
        head = self.w["model.embed_tokens.weight"] if c.tie_word_embeddings else self.w["lm_head.weight"]
        return oracle.linear(normalized, head, oracle.BF16).reshape(b, t, c.vocab_size)

    def new_cache(self, batch, capacity):
        c = self.c
        shape = (batch, c.num_key_value_heads, capacity, c.head_dim)
        return [(np.zeros(shape, np.float32), np.zeros(shape, np.float32)) for _ in range(c.num_layers)]

    def generate(self, prompt, max_new):
        ids = list(prompt)
        caches = self.new_cache(1, len(ids) + max_new)
        pos, chunk = 0, list(ids)
        for _ in range(max_new):
            logits = self.forward([chunk], pos, caches)
            pos += len(chunk)
            nxt = oracle.argmax(logits[0, -1])
            ids.append(nxt)
            chunk = [nxt]
        return ids
