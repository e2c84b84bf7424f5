"""Llama runtime mirror: LlamaConfig, BackendLlama and BackendLlamaCache over libstb200.so.

Names, argument meaning and error behaviour follow the reference
(models/src/main/scala/scalatorch/models/{LlamaConfig,BackendLlama,BackendLlamaCache}.scala):
invalid requests raise IllegalArgumentException before any native call; the cache position
advances only after a whole chunk succeeded; generation is greedy (temperature 0) with the
reference's lowest-id tie rule and EOS stop.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass

import numpy as np

from .ffm import (B200Session, IllegalArgumentException, IllegalStateException, STB_BF16, STB_F16, STB_F32,
                  call, library, require)

# stb_llama_weight
W_EMBED, W_FINAL_NORM, W_LM_HEAD, W_IN_NORM, W_POST_NORM = 0, 1, 2, 3, 4
W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = 5, 6, 7, 8, 9, 10, 11
LAYER_WEIGHTS = {
    "input_layernorm": W_IN_NORM, "post_attention_layernorm": W_POST_NORM,
    "self_attn.q_proj": W_Q, "self_attn.k_proj": W_K, "self_attn.v_proj": W_V, "self_attn.o_proj": W_O,
    "mlp.gate_proj": W_GATE, "mlp.up_proj": W_UP, "mlp.down_proj": W_DOWN,
}
GLOBAL_WEIGHTS = {"model.embed_tokens.weight": W_EMBED, "model.norm.weight": W_FINAL_NORM, "lm_head.weight": W_LM_HEAD}


def weight_stream(which: int, layer: int = 0) -> int:
    """Generator stream of a named tensor in stb_llama_init_random."""
    return 4096 + which if which in (W_EMBED, W_FINAL_NORM, W_LM_HEAD) else layer * 16 + which


@dataclass
class LlamaConfig:
    """LlamaConfig (LlamaConfig.scala:12-23) with the same validation."""
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_positions: int = 2048
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    tie_word_embeddings: bool = False
    bos_token_id: int | None = 1
    eos_token_ids: tuple = (2,)
    initializer_range: float = 0.02

    def __post_init__(self):
        require(self.vocab_size > 0 and self.hidden_size > 0 and self.intermediate_size > 0 and self.num_layers > 0
                and self.max_positions > 0, "invalid Llama dimensions")
        require(self.num_attention_heads > 0 and self.num_key_value_heads > 0
                and self.hidden_size % self.num_attention_heads == 0
                and self.num_attention_heads % self.num_key_value_heads == 0, "invalid Llama head dimensions")
        require(self.head_dim % 2 == 0, "Llama rotary head width must be even")
        require(np.isfinite(self.rms_norm_eps) and self.rms_norm_eps > 0 and np.isfinite(self.rope_theta)
                and self.rope_theta > 0, "invalid Llama norm/rotary configuration")
        require(np.isfinite(self.initializer_range) and self.initializer_range >= 0,
                "invalid Llama initializer range")
        require(all(0 <= i < self.vocab_size for i in ([self.bos_token_id] if self.bos_token_id is not None else [])
                    + list(self.eos_token_ids)), "special token ID out of vocabulary")

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @staticmethod
    def from_json(text: str) -> "LlamaConfig":
        """LlamaConfig.fromJson (LlamaConfig.scala:44-112): strict llama/SiLU subset with typed fields
        (integers in [0, 2^31), finite numbers, JSON booleans, EOS as null / id / array of at most
        1024 ids), duplicate keys, non-finite constants and configs over 1 MiB rejected."""
        require(isinstance(text, str) and len(text) <= 1048576, "Llama config exceeds size limit")
        try:
            f = json.loads(text, object_pairs_hook=_no_duplicates, parse_constant=_no_constant)
        except ValueError as e:
            raise IllegalArgumentException(f"invalid Llama config JSON: {e}") from e
        require(isinstance(f, dict), "Llama config must be an object")
        missing = object()

        def integer(key, default=missing):
            v = f.get(key, missing)
            if v is missing and default is not missing:
                return default
            require(type(v) is int and 0 <= v <= 0x7FFFFFFF, f"expected nonnegative integer config: {key}")
            return v

        def number(key, default):
            v = f.get(key, default)
            require(type(v) in (int, float), f"expected numeric config: {key}")
            require(np.isfinite(v), f"nonfinite config: {key}")
            return float(v)

        def boolean(key, default):
            v = f.get(key, default)
            require(type(v) is bool, f"expected boolean config: {key}")
            return v

        require(f.get("model_type") == "llama", "only model_type=llama is supported")
        require(f.get("hidden_act", "silu") == "silu", "only SiLU Llama MLP is supported")
        for key in ("rope_scaling", "rope_parameters", "sliding_window"):
            require(f.get(key) is None, f"unsupported Llama option: {key}")
        require(not boolean("attention_bias", False) and not boolean("mlp_bias", False),
                "Llama projection biases unsupported")
        require(number("attention_dropout", 0.0) == 0 and integer("pretraining_tp", 1) == 1,
                "unsupported Llama dropout/tensor parallel setting")
        require(number("partial_rotary_factor", 1.0) == 1.0, "partial rotary dimensions unsupported")
        heads = integer("num_attention_heads")
        bos = f.get("bos_token_id", 1)
        require(bos is None or type(bos) is int, "invalid BOS ID")
        eos = f.get("eos_token_id", 2)
        if eos is None:
            eos = ()
        elif type(eos) is int:
            eos = (eos,)
        else:
            require(isinstance(eos, list) and len(eos) <= 1024 and all(type(i) is int for i in eos), "invalid EOS IDs")
            eos = tuple(eos)
        c = LlamaConfig(integer("vocab_size"), integer("hidden_size"), integer("intermediate_size"),
                        integer("num_hidden_layers"), heads, integer("num_key_value_heads", heads),
                        integer("max_position_embeddings", 2048), number("rms_norm_eps", 1e-6),
                        number("rope_theta", 10000.0), boolean("tie_word_embeddings", False), bos, eos,
                        number("initializer_range", 0.02))
        require(integer("head_dim", c.head_dim) == c.head_dim, "custom Llama head_dim unsupported")
        return c


def _no_constant(name):
    raise ValueError(f"non-numeric JSON constant {name}")


def _no_duplicates(pairs):
    keys = [k for k, _ in pairs]
    if len(keys) != len(set(keys)):
        raise ValueError("duplicate key")
    return dict(pairs)


class _Config(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int), ("hidden_size", ctypes.c_int), ("intermediate_size", ctypes.c_int),
                ("num_layers", ctypes.c_int), ("num_attention_heads", ctypes.c_int),
                ("num_key_value_heads", ctypes.c_int), ("max_positions", ctypes.c_int),
                ("tie_word_embeddings", ctypes.c_int), ("rms_norm_eps", ctypes.c_double),
                ("rope_theta", ctypes.c_double), ("weight_dtype", ctypes.c_int), ("tp_rank", ctypes.c_int),
                ("tp_size", ctypes.c_int), ("tc_prefill_rows", ctypes.c_int)]


def _declare_llama():
    L = library()
    P, I, U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
    sig = {
        "stb_llama_create": [P, P, ctypes.POINTER(P)],
        "stb_llama_destroy": [P],
        "stb_llama_weight_bytes": [P, ctypes.POINTER(U64)],
        "stb_llama_set_weight": [P, I, I, P, U64, I],
        "stb_llama_init_random": [P, U64, ctypes.c_double],
        "stb_llama_cache_create": [P, I, I, ctypes.POINTER(P)],
        "stb_llama_cache_destroy": [P],
        "stb_llama_cache_position": [P, ctypes.POINTER(I)],
        "stb_llama_cache_reset": [P],
        "stb_llama_decode": [P, P, I, I, P, P],
        "stb_llama_generate": [P, P, I, I, I, P, I, P, P, P],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args


class BackendLlama:
    """Prepared, thread-confined inference over resident half weights (BackendLlama.scala:27-174)."""

    def __init__(self, session: B200Session, config: LlamaConfig, weight_dtype: int = STB_BF16,
                 tp_rank: int = 0, tp_size: int = 1, tc_prefill_rows: int = 0):
        """tc_prefill_rows: chunks with at least this many token rows use the tensor-core prefill
        (activations rounded to the weight type); 0 = library default (256), < 0 = never."""
        _declare_llama()
        require(weight_dtype in (STB_BF16, STB_F16), "Llama weights must be BF16 or F16")
        self.session = session
        self.config = config
        self.weight_dtype = weight_dtype
        c = _Config(config.vocab_size, config.hidden_size, config.intermediate_size, config.num_layers,
                    config.num_attention_heads, config.num_key_value_heads, config.max_positions,
                    int(config.tie_word_embeddings), config.rms_norm_eps, config.rope_theta, weight_dtype,
                    tp_rank, tp_size, tc_prefill_rows)
        h = ctypes.c_void_p()
        call("stb_llama_create", session.handle, ctypes.byref(c), ctypes.byref(h))
        self.handle = h
        self._closed = False
        self._caches = []

    # -- preparation
    @classmethod
    def prepare_random(cls, session, config, seed: int, weight_dtype: int = STB_BF16, tp_rank=0, tp_size=1,
                       tc_prefill_rows: int = 0):
        """LlamaModel.init + BackendLlama.prepare in one step: N(0, initializer_range) matrices generated
        on the device by the counter-based generator, norms = 1."""
        m = cls(session, config, weight_dtype, tp_rank, tp_size, tc_prefill_rows)
        try:
            call("stb_llama_init_random", m.handle, seed, config.initializer_range)
        except Exception:
            m.close()
            raise
        return m

    def set_weight(self, name: str, payload: np.ndarray, dtype: int) -> None:
        """Upload one named tensor's raw payload (full tensor; this rank keeps its shard)."""
        which, layer = _parse_name(name)
        raw = np.ascontiguousarray(payload)
        call("stb_llama_set_weight", self.handle, which, layer, raw.ctypes.data, raw.nbytes, dtype)

    @property
    def weight_bytes(self) -> int:
        v = ctypes.c_uint64()
        call("stb_llama_weight_bytes", self.handle, ctypes.byref(v))
        return v.value

    def close(self) -> None:
        if not self._closed:
            for c in list(self._caches):
                c.close()
            self._closed = True
            call("stb_llama_destroy", self.handle)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self):
        if self._closed:
            raise IllegalStateException("BackendLlama", 6, "prepared Llama is closed")

    # -- inference
    def new_cache(self, batch_size: int = 1, capacity: int | None = None) -> "BackendLlamaCache":
        self._check()
        cap = self.config.max_positions if capacity is None else capacity
        require(batch_size > 0 and 0 < cap <= self.config.max_positions, "invalid model cache dimensions/budget")
        c = BackendLlamaCache(self, batch_size, cap)
        self._caches.append(c)
        return c

    def generate_ids(self, prompt, max_new_tokens: int, eos_token_ids=None, timings: list | None = None):
        """Greedy BackendLlama.generateIds (BackendLlama.scala:126-141).  prompt: 1-D ids, or 2-D
        (batch, tokens) for a batch of equal-length prompts; returns list(s) of ids."""
        self._check()
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int64))
        single = p.ndim == 1
        if single:
            p = p[None, :]
        require(p.ndim == 2 and p.shape[1] > 0 and max_new_tokens >= 0
                and p.shape[1] + max_new_tokens <= self.config.max_positions, "invalid generation length")
        require(bool(np.all((p >= 0) & (p < self.config.vocab_size))), "generation token outside vocabulary")
        eos = np.ascontiguousarray(np.asarray(self.config.eos_token_ids if eos_token_ids is None else eos_token_ids,
                                              np.int64).reshape(-1))
        b, t = p.shape
        out = np.empty((b, t + max_new_tokens), np.int64)
        gen = np.zeros(b, np.int32)
        tm = np.zeros(2, np.float32)
        call("stb_llama_generate", self.handle, p.ctypes.data, b, t, max_new_tokens,
             eos.ctypes.data if eos.size else None, int(eos.size), out.ctypes.data, gen.ctypes.data, tm.ctypes.data)
        if timings is not None:
            timings[:] = [float(tm[0]), float(tm[1])]
        rows = [out[i, :t + gen[i]].tolist() for i in range(b)]
        return rows[0] if single else rows


class BackendLlamaCache:
    """Resident KV cache (BackendLlamaCache.scala:8-49)."""

    def __init__(self, model: BackendLlama, batch_size: int, capacity: int):
        self.model = model
        self.batch_size = batch_size
        self.capacity = capacity
        h = ctypes.c_void_p()
        call("stb_llama_cache_create", model.handle, batch_size, capacity, ctypes.byref(h))
        self.handle = h
        self._closed = False

    @property
    def position(self) -> int:
        self._check()
        v = ctypes.c_int()
        call("stb_llama_cache_position", self.handle, ctypes.byref(v))
        return v.value

    def _check(self):
        if self._closed:
            raise IllegalStateException("BackendLlamaCache", 6, "model cache is closed")

    def decode(self, tokens, want_logits: bool = True):
        """tokens (batch, count) -> logits (batch, count, vocab) as float32, and the greedy next ids."""
        self._check()
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64))
        require(t.ndim == 2 and t.shape[0] == self.batch_size and t.shape[1] > 0,
                "cache tokens must match batch with positive chunk length")
        require(self.position + t.shape[1] <= self.capacity, "model cache capacity exceeded")
        require(bool(np.all((t >= 0) & (t < self.model.config.vocab_size))), "embedding token ID out of bounds")
        logits = np.empty((t.shape[0], t.shape[1], self.model.config.vocab_size), np.float32) if want_logits else None
        nxt = np.empty(t.shape[0], np.int64)
        call("stb_llama_decode", self.handle, t.ctypes.data, t.shape[0], t.shape[1],
             logits.ctypes.data if logits is not None else None, nxt.ctypes.data)
        return logits, nxt.tolist()

    def reset(self) -> None:
        self._check()
        call("stb_llama_cache_reset", self.handle)

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            if self in self.model._caches:
                self.model._caches.remove(self)
            call("stb_llama_cache_destroy", self.handle)


@dataclass(frozen=True)
class ShardPlan:
    """What one rank of a tensor-parallel group holds (stb_llama_shard_plan)."""
    heads: tuple
    kv_heads: tuple
    intermediate: tuple
    vocab: tuple
    o_cols: tuple
    down_cols: tuple
    weight_bytes: int


def shard_plan(config: LlamaConfig, rank: int, tp: int, weight_dtype: int = STB_BF16) -> ShardPlan:
    """Host-only Megatron split of `config` for `rank` of `tp` (no device is touched)."""
    L = library()
    L.stb_llama_shard_plan.restype = ctypes.c_int
    L.stb_llama_shard_plan.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    c = _Config(config.vocab_size, config.hidden_size, config.intermediate_size, config.num_layers,
                config.num_attention_heads, config.num_key_value_heads, config.max_positions,
                int(config.tie_word_embeddings), config.rms_norm_eps, config.rope_theta, weight_dtype, rank, tp)
    out = (ctypes.c_int64 * 14)()
    call("stb_llama_shard_plan", ctypes.byref(c), rank, tp, out)
    v = list(out)
    return ShardPlan((v[0], v[1]), (v[2], v[3]), (v[4], v[5]), (v[6], v[7]), (v[8], v[9]), (v[10], v[11]), v[12])


def _parse_name(name: str):
    if name in GLOBAL_WEIGHTS:
        return GLOBAL_WEIGHTS[name], 0
    parts = name.split(".")
    require(len(parts) >= 5 and parts[0] == "model" and parts[1] == "layers" and parts[-1] == "weight",
            f"Llama weight names mismatch: {name}")
    layer = int(parts[2])
    key = ".".join(parts[3:-1])
    require(key in LAYER_WEIGHTS, f"Llama weight names mismatch: {name}")
    return LAYER_WEIGHTS[key], layer


def llama_weight_shapes(config: LlamaConfig) -> dict:
    """Every tensor name of a Llama checkpoint with its (out, in) shape (LlamaModel.shapes,
    LlamaModel.scala:115-128); lm_head.weight is optional when the embeddings are tied."""
    H, I, V = config.hidden_size, config.intermediate_size, config.vocab_size
    kvw = config.num_key_value_heads * config.head_dim
    out = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,), "lm_head.weight": (V, H)}
    for i in range(config.num_layers):
        p = f"model.layers.{i}"
        out.update({f"{p}.input_layernorm.weight": (H,), f"{p}.post_attention_layernorm.weight": (H,),
                    f"{p}.self_attn.q_proj.weight": (H, H), f"{p}.self_attn.k_proj.weight": (kvw, H),
                    f"{p}.self_attn.v_proj.weight": (kvw, H), f"{p}.self_attn.o_proj.weight": (H, H),
                    f"{p}.mlp.gate_proj.weight": (I, H), f"{p}.mlp.up_proj.weight": (I, H),
                    f"{p}.mlp.down_proj.weight": (H, I)})
    return out


def check_llama_archive(config: LlamaConfig, archive) -> tuple:
    """LlamaModel.load's checks (LlamaModel.scala:158-173) before any device work: the archive holds
    exactly the expected names (lm_head optional when tied), each with its shape and an F32 / F16 /
    BF16 dtype, and a head stored beside tied embeddings equals them bit for bit (after widening).
    The device keeps matrices in their on-disk half type, so the matrices must also share one of
    BF16 / F16.  Returns (weight dtype STB_BF16 / STB_F16, whether a tied head is stored)."""
    expected = llama_weight_shapes(config)
    optional = {"lm_head.weight"} if config.tie_word_embeddings else set()
    names = set(archive.tensors)
    require(set(expected) - optional <= names <= set(expected), "Llama weight names mismatch")
    for name in sorted(names):
        info = archive.tensors[name]
        require(tuple(info.shape) == expected[name] and info.dtype in ("F32", "F16", "BF16"),
                f"Llama weight metadata mismatch: {name}")
    uploaded = names - optional  # a head stored beside tied embeddings is checked, not uploaded
    dtypes = {archive.tensors[n].dtype for n in uploaded if len(expected[n]) == 2}
    require(len(dtypes) == 1 and next(iter(dtypes)) in ("BF16", "F16"),
            "Llama matrices must share one BF16/F16 dtype (they stay half precision on the device)")
    tied_head = config.tie_word_embeddings and "lm_head.weight" in names
    if tied_head:
        head, emb = archive.tensors["lm_head.weight"], archive.tensors["model.embed_tokens.weight"]
        require(np.array_equal(_float_bits(archive.read_raw("lm_head.weight"), head.dtype),
                               _float_bits(archive.read_raw("model.embed_tokens.weight"), emb.dtype)),
                "conflicting tied lm_head weight")
    return (STB_BF16 if next(iter(dtypes)) == "BF16" else STB_F16), tied_head


def _float_bits(raw: np.ndarray, dtype: str) -> np.ndarray:
    """Float32 bit patterns of a raw payload, widened as SafeTensors.readFloat does."""
    if dtype == "BF16":
        return raw.astype(np.uint32) << 16
    if dtype == "F16":
        return raw.view(np.float16).astype(np.float32).view(np.uint32)
    return raw.view(np.uint32)


def load_safetensors(session: B200Session, directory: str, weight_dtype: int | None = None,
                     tp_rank: int = 0, tp_size: int = 1, read_limits=None, shard_limits=None) -> BackendLlama:
    """LlamaModel.load + BackendLlama.prepare with raw half uploads (no F32 widening on the host).
    The checkpoint directory holds config.json and model.safetensors or model.safetensors.index.json
    (SafeTensorSet.open).  read_limits.max_tensor_bytes bounds each raw payload read on the host
    (default 1 GiB, as ReadLimits; a 70B-shaped lm_head needs it raised)."""
    import os

    from .io import ReadLimits, SafeTensorSet, ShardLimits
    with open(os.path.join(directory, "config.json")) as f:
        config = LlamaConfig.from_json(f.read())
    with SafeTensorSet.open(directory, read_limits or ReadLimits(), shard_limits or ShardLimits()) as archive:
        wdt, tied_head = check_llama_archive(config, archive)
        m = BackendLlama(session, config, weight_dtype or wdt, tp_rank, tp_size)
        try:
            for name in archive.names():
                if tied_head and name == "lm_head.weight":
                    continue
                info = archive.info(name)
                dtype = {"F32": STB_F32, "BF16": STB_BF16, "F16": STB_F16}[info.dtype]
                m.set_weight(name, archive.read_raw(name), dtype)
        except BaseException:
            m.close()
            raise
    return m


class _Scope:
    """BackendScope (BackendLlama.scala:9-24): owns handles, releases them in reverse order, and hands
    one result to the caller with take()."""

    def __init__(self, backend: B200Session):
        self.backend, self.owned = backend, []

    def keep(self, t):
        self.owned.append(t)
        return t

    def take(self, t):
        for i in range(len(self.owned) - 1, -1, -1):
            if self.owned[i] is t:
                del self.owned[i]
                return t
        raise IllegalArgumentException("backend handle is not owned by this scope")

    def release(self, t):
        self.backend.release(self.take(t))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        failure = None
        for t in reversed(self.owned):
            try:
                self.backend.release(t)
            except Exception as e:  # first failure wins, as the reference's scope
                failure = failure or e
        self.owned.clear()
        if failure is not None and exc[0] is None:
            raise failure


class PerOpLlama:
    """BackendLlama's per-op path (models/src/main/scala/scalatorch/models/BackendLlama.scala:27-111) on
    the B200 FloatBackend: every operation of LlamaBlock is one device op of B200Session
    (embedding, rmsNorm, matmul against the resident (out,in) half weights, reshape / transpose views,
    rope, causalAttention or the attention cache, silu, multiply, add), in the reference's order and
    with its releases.  It is the path for models the fused runtime does not take -- Linear layers
    with low-rank adapters, applied as BackendLlama.linear does (base + ((x A^T) B^T) * (alpha / r),
    BackendLlama.scala:41-49) -- and the drop-in form of BackendLlama.prepare(model, backend).

    weights: safetensors name -> raw payload (half bits as uint16, or float32), dtype per tensor.
    lora: projection name (e.g. "model.layers.0.self_attn.q_proj") -> (A [rank, in] f32, B [out, rank]
    f32, alpha)."""

    def __init__(self, session: B200Session, config: LlamaConfig, weights: dict, dtypes: dict, lora: dict | None = None):
        self.session, self.config = session, config
        c = config
        self._owned = []
        try:
            def up_half(name):
                bits = np.ascontiguousarray(weights[name])
                if dtypes[name] == STB_F32:
                    return self._keep(session.upload_weight_f32(bits.view(np.float32)))
                return self._keep(session.upload_weight(bits, dtypes[name]))

            def up_norm(name):
                return self._keep(session.upload(_widen(weights[name], dtypes[name])))

            emb = np.ascontiguousarray(weights["model.embed_tokens.weight"])
            et = dtypes["model.embed_tokens.weight"]
            self.embed = self._keep(session.upload(emb.view(np.float32)) if et == STB_F32
                                    else session.upload_half(emb, et))
            self.final_norm = up_norm("model.norm.weight")
            if c.tie_word_embeddings:  # the table's (vocab, hidden) bytes are the head's (out, in) layout
                self.lm_head = self._keep(session.reshape(self.embed, (c.hidden_size, c.vocab_size)))
                self.lm_head.transposed_weight = True
            else:
                self.lm_head = up_half("lm_head.weight")
            self.layers = []
            for i in range(c.num_layers):
                p = f"model.layers.{i}"
                layer = {"in_norm": up_norm(f"{p}.input_layernorm.weight"),
                         "post_norm": up_norm(f"{p}.post_attention_layernorm.weight")}
                for key, name in (("q", "self_attn.q_proj"), ("k", "self_attn.k_proj"), ("v", "self_attn.v_proj"),
                                  ("o", "self_attn.o_proj"), ("gate", "mlp.gate_proj"), ("up", "mlp.up_proj"),
                                  ("down", "mlp.down_proj")):
                    w = up_half(f"{p}.{name}.weight")
                    adapter = None
                    if lora and f"{p}.{name}" in lora:
                        a, b, alpha = lora[f"{p}.{name}"]
                        require(a.ndim == 2 and b.ndim == 2 and a.shape[1] == w.shape[0] and b.shape[0] == w.shape[1]
                                and a.shape[0] == b.shape[1] and a.shape[0] > 0, "Linear adapter shape mismatch")
                        scale = float(np.float32(alpha / a.shape[0])) if np.isfinite(alpha) and alpha > 0 else np.nan
                        require(np.isfinite(scale) and scale > 0, "invalid adapter scale")
                        # (A, B) uploaded as (out,in) Float32 matrices used transposed, as prepare does
                        adapter = (self._keep(session.upload_weight_f32(a)), self._keep(session.upload_weight_f32(b)),
                                   scale)
                    layer[key] = (w, adapter)
                self.layers.append(layer)
        except BaseException:
            self.close()
            raise

    def _keep(self, t):
        self._owned.append(t)
        return t

    def close(self) -> None:
        for t in reversed(self._owned):
            self.session.release(t)
        self._owned = []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- BackendLlama.scala:41-111, op for op
    def _linear(self, x, layer):
        """BackendLlama.linear (BackendLlama.scala:41-49)."""
        be = self.session
        w, adapter = layer
        if adapter is None:
            return be.matmul(x, w)
        a, b, scale = adapter
        with _Scope(be) as scope:
            base = scope.keep(be.matmul(x, w))
            low = scope.keep(be.matmul(x, a))
            delta = scope.keep(be.matmul(low, b))
            scaled = scope.keep(be.scale(delta, scale))
            return scope.take(scope.keep(be.add(base, scaled)))

    def _attention(self, x, layer, b, t, position, cache):
        be, c = self.session, self.config
        hd = c.head_dim
        with _Scope(be) as scope:
            keep = scope.keep
            flat = keep(be.reshape(x, (b * t, c.hidden_size)))

            def heads(proj, count):
                projected = keep(self._linear(flat, layer[proj]))
                split = keep(be.reshape(projected, (b, t, count, hd)))
                return keep(be.transpose(split, 1, 2))

            q = keep(be.rope(heads("q", c.num_attention_heads), position, c.rope_theta))
            k = keep(be.rope(heads("k", c.num_key_value_heads), position, c.rope_theta))
            v = heads("v", c.num_key_value_heads)
            attended = keep(cache.attend(q, k, v, position) if cache is not None else be.causal_attention(q, k, v))
            joined = keep(be.transpose(attended, 1, 2))
            matrix = keep(be.reshape(joined, (b * t, c.hidden_size)))
            projected = keep(self._linear(matrix, layer["o"]))
            return scope.take(keep(be.reshape(projected, (b, t, c.hidden_size))))

    def _mlp(self, x, layer, b, t):
        be, c = self.session, self.config
        with _Scope(be) as scope:
            keep = scope.keep
            flat = keep(be.reshape(x, (b * t, c.hidden_size)))
            gate = keep(self._linear(flat, layer["gate"]))
            activated = keep(be.silu(gate))
            up = keep(self._linear(flat, layer["up"]))
            product = keep(be.multiply(activated, up))
            down = keep(self._linear(product, layer["down"]))
            return scope.take(keep(be.reshape(down, (b, t, c.hidden_size))))

    def _block(self, x, layer, b, t, position, cache):
        be, eps = self.session, self.config.rms_norm_eps
        with _Scope(be) as scope:
            keep = scope.keep
            normalized = keep(be.rms_norm(x, layer["in_norm"], eps))
            attended = keep(self._attention(normalized, layer, b, t, position, cache))
            hidden = keep(be.add(x, attended))
            post = keep(be.rms_norm(hidden, layer["post_norm"], eps))
            feed = keep(self._mlp(post, layer, b, t))
            return scope.take(keep(be.add(hidden, feed)))

    def forward(self, tokens, position: int = 0, caches=None):
        """BackendLlama.run (BackendLlama.scala:86-101): logits (batch, tokens, vocab) as a device tensor
        owned by the caller."""
        be, c = self.session, self.config
        ids = np.asarray(tokens, np.int64)
        require(ids.ndim == 2, "Llama tokens must have shape (batch,tokens)")
        b, t = ids.shape
        require(position >= 0 and position + t <= c.max_positions, "Llama context limit exceeded")
        require(b * t * c.vocab_size <= 16777216 and b * t * c.vocab_size <= 0x7FFFFFFF,
                "Llama logits allocation limit exceeded")
        with _Scope(be) as scope:
            hidden = scope.keep(be.embedding(self.embed, ids))
            for i, layer in enumerate(self.layers):
                nxt = scope.keep(self._block(hidden, layer, b, t, position, caches[i] if caches else None))
                scope.release(hidden)
                hidden = nxt
            normalized = scope.keep(be.rms_norm(hidden, self.final_norm, c.rms_norm_eps))
            flat = scope.keep(be.reshape(normalized, (b * t, c.hidden_size)))
            logits = scope.keep(self._linear(flat, (self.lm_head, None)))
            return scope.take(scope.keep(be.reshape(logits, (b, t, c.vocab_size))))

    def logits(self, tokens) -> np.ndarray:
        out = self.forward(tokens)
        try:
            return self.session.download(out)
        finally:
            self.session.release(out)

    def new_cache(self, batch_size: int = 1, capacity: int | None = None) -> "PerOpCache":
        return PerOpCache(self, batch_size, self.config.max_positions if capacity is None else capacity)

    def generate_ids(self, prompt, max_new_tokens: int) -> list:
        """Greedy BackendLlama.generateIds with the cache (BackendLlama.scala:126-141; TokenSampler's
        strict '>' keeps the lowest id among equal logits)."""
        c = self.config
        ids = [int(v) for v in prompt]
        require(len(ids) > 0 and max_new_tokens >= 0 and len(ids) + max_new_tokens <= c.max_positions,
                "invalid generation length")
        require(all(0 <= i < c.vocab_size for i in ids), "generation token outside vocabulary")
        if max_new_tokens == 0:
            return ids
        cache = self.new_cache(1, len(ids) + max_new_tokens)
        try:
            chunk = list(ids)
            for _ in range(max_new_tokens):
                logits = cache.decode([chunk])
                row = logits[0, -1]
                nxt = int(np.argmax(row))  # first maximum = lowest id
                ids.append(nxt)
                chunk = [nxt]
                if nxt in c.eos_token_ids:
                    break
        finally:
            cache.close()
        return ids


class PerOpCache:
    """BackendLlamaCache over per-layer device attention caches (BackendLlamaCache.scala:8-49): the
    position advances only after a whole chunk succeeded."""

    def __init__(self, model: PerOpLlama, batch_size: int, capacity: int):
        c = model.config
        require(batch_size > 0 and 0 < capacity <= c.max_positions, "invalid model cache dimensions/budget")
        self.model, self.batch_size, self.capacity, self.position = model, batch_size, capacity, 0
        self.layers = []
        try:
            for _ in range(c.num_layers):
                self.layers.append(model.session.attention_cache(batch_size, c.num_key_value_heads, capacity,
                                                                 c.head_dim, c.head_dim, 1 << 40))
        except BaseException:
            self.close()
            raise

    def decode(self, tokens) -> np.ndarray:
        ids = np.asarray(tokens, np.int64)
        require(ids.ndim == 2 and ids.shape[0] == self.batch_size and ids.shape[1] > 0,
                "cache tokens must match batch with positive chunk length")
        end = self.position + ids.shape[1]
        require(end <= self.capacity, "model cache capacity exceeded")
        c = self.model.config
        require(self.batch_size * c.num_attention_heads * ids.shape[1] * end <= 16777216,
                "cached score workspace limit exceeded")
        out = self.model.forward(ids, self.position, self.layers)
        try:
            logits = self.model.session.download(out)
        finally:
            self.model.session.release(out)
        self.position = end
        return logits

    def close(self) -> None:
        for layer in self.layers:
            layer.close()
        self.layers = []


def _widen(raw, dtype: int) -> np.ndarray:
    """SafeTensors.readFloat's exact widening of a raw payload (SafeTensors.scala:63-77)."""
    raw = np.ascontiguousarray(raw)
    if dtype == STB_F32:
        return raw.view(np.float32)
    return _float_bits(raw.view(np.uint16), "BF16" if dtype == STB_BF16 else "F16").view(np.float32)
