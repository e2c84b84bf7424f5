"""ctypes view of the CPU oracle (oracle/stb_oracle.c).

TEST INFRASTRUCTURE ONLY.  This module is the checker for the parity tests, the smoke check
and the timed CPU baseline of bench.py.  The product (libstb200.so and the scalatorch Python
mirror) never imports it; a product path that reached it would void the parity claims.

Each wrapper restates one piece of scala-torch's CPU Float32 arithmetic; the reference file:line
is in stb_oracle.h beside the C declaration.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, BF16, F16 = 0, 1, 2
ORDER_NUMSCALA, ORDER_SEQUENTIAL = 0, 1

_lib = None


def build() -> str:
    """Compile stb_oracle.c into oracle/liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "stb_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_p = ctypes.c_void_p
_i = ctypes.c_int
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t
_d = ctypes.c_double


def _declare(L):
    sig = {
        "oracle_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "oracle_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "oracle_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
        "oracle_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
        "oracle_widen": (None, [_p, _i, _p, _sz]),
        "oracle_round_bf16": (None, [_p, _p, _sz]),
        "oracle_round_f16": (None, [_p, _p, _sz]),
        "oracle_matmul_tr": (None, [_p, _p, _p, _i, _i, _i, _i]),
        "oracle_matmul_seq": (None, [_p, _p, _p, _i, _i, _i]),
        "oracle_linear": (None, [_p, _p, _i, _p, _p, _i, _i, _i, _i, _i]),
        "oracle_linear_adapted": (None, [_p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _i, _i, _i]),
        "oracle_rmsnorm": (None, [_p, _p, _p, _i, _i, _d]),
        "oracle_silu": (ctypes.c_float, [ctypes.c_float]),
        "oracle_rope": (None, [_p, _p, _i, _i, _i, _i, _i, _d]),
        "oracle_causal_attention": (None, [_p, _p, _p, _p] + [_i] * 9),
        "oracle_argmax": (ctypes.c_int64, [_p, ctypes.c_int64]),
        "oracle_rng_u64": (_u64, [_u64, _u64, _u64]),
        "oracle_rng_normal": (_d, [_u64, _u64, _u64]),
        "oracle_fill_normal_bf16": (None, [_p, _sz, _u64, _u64, _d, _i]),
        "oracle_fill_normal_f32": (None, [_p, _sz, _u64, _u64, _d, _i]),
        "oracle_log": (_d, [_d]),
        "oracle_cache_create": (_p, [_p, _i, _i]),
        "oracle_cache_destroy": (None, [_p]),
        "oracle_cache_position": (_i, [_p]),
        "oracle_llama_decode": (_i, [_p, _p, _p, _p, _i, _i, _p, _i]),
        "oracle_llama_generate": (_i, [_p, _p, _p, _i, _i, _p, _i, _p, _i]),
        "oracle_max_threads": (_i, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def max_threads() -> int:
    return lib().oracle_max_threads()


# ---------------------------------------------------------------- conversions

def widen(bits: np.ndarray, dtype: int) -> np.ndarray:
    """SafeTensors.readFloat widening (SafeTensors.scala:63-77)."""
    src = np.ascontiguousarray(bits)
    out = np.empty(src.size, np.float32)
    lib().oracle_widen(_ptr(src), dtype, _ptr(out), src.size)
    return out.reshape(src.shape)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """SafeTensorsWriter.bfloat RNE (SafeTensorsWriter.scala:58-61)."""
    src = np.ascontiguousarray(x, np.float32)
    out = np.empty(src.size, np.uint16)
    lib().oracle_round_bf16(_ptr(src), _ptr(out), src.size)
    return out.reshape(src.shape)


def round_f16(x: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(x, np.float32)
    out = np.empty(src.size, np.uint16)
    lib().oracle_round_f16(_ptr(src), _ptr(out), src.size)
    return out.reshape(src.shape)


# ---------------------------------------------------------------- GEMM / Linear

def matmul_tr(x: np.ndarray, w: np.ndarray, threads: int = 0) -> np.ndarray:
    """x[M,K] . W[N,K]^T in numscala's transposed-right order (NumscalaBackend.scala:8-30)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    lib().oracle_matmul_tr(_ptr(x), _ptr(w), _ptr(y), M, N, K, threads or max_threads())
    return y


def matmul_seq(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Ops.matmul (Ops.scala:61-81): a[M,K] . b[K,N], sequential accumulator."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    M, K = a.shape
    N = b.shape[1]
    c = np.empty((M, N), np.float32)
    lib().oracle_matmul_seq(_ptr(a), _ptr(b), _ptr(c), M, N, K)
    return c


def linear(x: np.ndarray, w_bits: np.ndarray, w_dtype: int, bias: np.ndarray | None = None,
           order: int = ORDER_NUMSCALA, threads: int = 0) -> np.ndarray:
    """nn.Linear.apply with a widened half/F32 (out,in) weight (Linear.scala:11-17)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w_bits)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().oracle_linear(_ptr(x), _ptr(w), w_dtype, _ptr(b), _ptr(y), M, N, K, order,
                        threads or max_threads())
    return y


def adapter_scale(alpha: float, rank: int) -> np.float32:
    """LowRankAdapter.scale (LowRankAdapter.scala:24-27): (alpha / rank) rounded to Float32."""
    value = np.float32(alpha / rank)
    if not (np.isfinite(alpha) and alpha > 0 and np.isfinite(value) and value > 0):
        raise ValueError("invalid adapter scale")
    return value


def linear_adapted(x: np.ndarray, w_bits: np.ndarray, w_dtype: int, bias: np.ndarray | None = None,
                   lora=None, scoped=(), threads: int = 0) -> np.ndarray:
    """nn.Linear.apply with its low-rank adapter and LinearAdapterScope entries (Linear.scala:11-17).
    lora = (A[rank,K], B[N,rank], alpha) or None; scoped = [((A, B, alpha), multiplier), ...]."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w_bits)
    M, K = x.shape
    N = w.shape[0]
    terms = ([(lora, 0, 1.0)] if lora is not None else []) + [(a, 1, m) for a, m in scoped]
    keep, a_ptrs, b_ptrs, ranks, scales, flags, mults = [], [], [], [], [], [], []
    for (A, B, alpha), flag, mult in terms:
        A = np.ascontiguousarray(A, np.float32)
        B = np.ascontiguousarray(B, np.float32)
        keep += [A, B]
        a_ptrs.append(A.ctypes.data)
        b_ptrs.append(B.ctypes.data)
        ranks.append(A.shape[0])
        scales.append(adapter_scale(alpha, A.shape[0]))
        flags.append(flag)
        mults.append(mult)
    n = len(terms)
    pa = (ctypes.c_void_p * max(n, 1))(*a_ptrs)
    pb = (ctypes.c_void_p * max(n, 1))(*b_ptrs)
    pr = np.array(ranks or [0], np.int32)
    ps = np.array(scales or [0], np.float32)
    pf = np.array(flags or [0], np.int32)
    pm = np.array(mults or [0], np.float32)
    y = np.empty((M, N), np.float32)
    bb = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().oracle_linear_adapted(_ptr(x), _ptr(w), w_dtype, _ptr(bb), ctypes.cast(pa, ctypes.c_void_p),
                                ctypes.cast(pb, ctypes.c_void_p), _ptr(pr), _ptr(ps), _ptr(pf), _ptr(pm), n,
                                _ptr(y), M, N, K, threads or max_threads())
    return y


# ---------------------------------------------------------------- decode-step ops

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    width = w.size
    y = np.empty_like(x)
    lib().oracle_rmsnorm(_ptr(x), _ptr(w), _ptr(y), x.size // width, width, eps)
    return y


def silu(x: np.ndarray) -> np.ndarray:
    f = lib().oracle_silu
    return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.float32).reshape(np.shape(x))


def rope(x: np.ndarray, start: int = 0, theta: float = 10000.0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    b, h, t, d = x.shape
    y = np.empty_like(x)
    lib().oracle_rope(_ptr(x), _ptr(y), b, h, t, d, start, theta)
    return y


def causal_attention(q, k, v, start: int = 0, key_stride: int | None = None, keys: int | None = None):
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    b, h, t, d = q.shape
    kvh, s = k.shape[1], k.shape[2]
    dv = v.shape[3]
    out = np.empty((b, h, t, dv), np.float32)
    lib().oracle_causal_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, h, t, d, kvh,
                                  keys if keys is not None else s,
                                  key_stride if key_stride is not None else s, dv, start)
    return out


def argmax(logits: np.ndarray) -> int:
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().oracle_argmax(_ptr(x), x.size))


# ---------------------------------------------------------------- synthetic weights

def rng_u64(seed: int, stream: int, index: int) -> int:
    return int(lib().oracle_rng_u64(seed, stream, index))


def rng_normal(seed: int, stream: int, index: int) -> float:
    return float(lib().oracle_rng_normal(seed, stream, index))


def normal_bf16(count: int, seed: int, stream: int, std: float, threads: int = 0) -> np.ndarray:
    out = np.empty(count, np.uint16)
    lib().oracle_fill_normal_bf16(_ptr(out), count, seed, stream, std, threads or max_threads())
    return out


def normal_f32(count: int, seed: int, stream: int, std: float, threads: int = 0) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().oracle_fill_normal_f32(_ptr(out), count, seed, stream, std, threads or max_threads())
    return out


# ---------------------------------------------------------------- Llama

class _Config(ctypes.Structure):
    _fields_ = [("vocab", _i), ("hidden", _i), ("intermediate", _i), ("layers", _i), ("heads", _i),
                ("kv_heads", _i), ("max_positions", _i), ("tie_embeddings", _i),
                ("rms_eps", _d), ("rope_theta", _d)]


class _Weights(ctypes.Structure):
    _fields_ = [("embed", _p), ("final_norm", _p), ("lm_head", _p)] + [
        (n, ctypes.POINTER(_p)) for n in
        ("in_norm", "post_norm", "q", "k", "v", "o", "gate", "up", "down")]


LAYER_FIELDS = ("in_norm", "post_norm", "q", "k", "v", "o", "gate", "up", "down")


@dataclass
class LlamaWeights:
    """F32 weights (the reference's widened in-memory form) for the oracle model."""
    embed: np.ndarray
    final_norm: np.ndarray
    lm_head: np.ndarray
    layers: list  # list of dict field -> np.ndarray


class OracleLlama:
    """LlamaModel + LlamaCache on the CPU (LlamaModel.scala:17-90, LlamaCache.scala:26-78)."""

    def __init__(self, config, weights: LlamaWeights, threads: int = 0):
        self.config = config
        self.weights = weights
        self.threads = threads or max_threads()
        c = _Config(config.vocab_size, config.hidden_size, config.intermediate_size,
                    config.num_layers, config.num_attention_heads, config.num_key_value_heads,
                    config.max_positions, int(config.tie_word_embeddings), config.rms_norm_eps,
                    config.rope_theta)
        self._c = c
        w = _Weights()
        w.embed = weights.embed.ctypes.data
        w.final_norm = weights.final_norm.ctypes.data
        w.lm_head = weights.lm_head.ctypes.data
        self._arrays = {}
        for f in LAYER_FIELDS:
            arr = (_p * config.num_layers)(*[lw[f].ctypes.data for lw in weights.layers])
            self._arrays[f] = arr
            setattr(w, f, ctypes.cast(arr, ctypes.POINTER(_p)))
        self._w = w

    def new_cache(self, batch: int, capacity: int):
        return lib().oracle_cache_create(ctypes.byref(self._c), batch, capacity)

    def free_cache(self, cache):
        lib().oracle_cache_destroy(cache)

    def decode(self, cache, tokens: np.ndarray) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, np.int64)
        b, t = tokens.shape
        logits = np.empty((b, t, self.config.vocab_size), np.float32)
        rc = lib().oracle_llama_decode(ctypes.byref(self._c), ctypes.byref(self._w), cache,
                                       _ptr(tokens), b, t, _ptr(logits), self.threads)
        if rc != 0:
            raise ValueError(f"oracle decode failed ({rc})")
        return logits

    def generate(self, prompt, max_new: int, eos=()) -> list:
        prompt = np.ascontiguousarray(prompt, np.int64)
        out = np.empty(prompt.size + max_new, np.int64)
        e = np.ascontiguousarray(list(eos) or [0], np.int64)
        n = lib().oracle_llama_generate(ctypes.byref(self._c), ctypes.byref(self._w), _ptr(prompt),
                                        prompt.size, max_new, _ptr(e), len(eos), _ptr(out),
                                        self.threads)
        if n < 0:
            raise ValueError("oracle generate failed")
        return out[:n].tolist()
