"""The FloatBackend operator set on the device (stb_op_*, B200Session) against the CPU oracle, and the
per-op BackendLlama path (PerOpLlama) layer by layer as BackendLlama.run drives it.

Tolerances: Float32 add / multiply / scale / transpose / embedding / expandScalar / cache append are
bit-exact (one IEEE operation, or a copy); SiLU, RMSNorm, RoPE, sum and attention compute in double as
the reference does and may differ from the oracle in the last double bits only, so their Float32
results are within 2 ulp (4e-7 relative + 1e-30); Llama logits 1e-5 * (1 + |e|)
(models/src/test/scala/scalatorch/models/BackendLlamaSuite.scala:18) and greedy ids identical.
"""
import numpy as np
import pytest

import oracle
from llama_fixtures import SMOL, TINY, named_bf16_weights, oracle_model
from per_op_oracle import CpuPerOpLlama
from scalatorch import ffm
from scalatorch.models import BackendLlama, LlamaConfig, PerOpLlama

pytestmark = pytest.mark.gpu


def ulp_close(got, want, rel=4e-7):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    err = np.abs(got - want)
    assert np.all(err <= rel * np.abs(want) + 1e-30), f"max err {err.max()}"


def bits_equal(got, want):
    """Bit for bit, except that NaNs compare as a class: the JVM does not distinguish NaN payloads
    (Float.floatToIntBits), and the GPU's NaN sign and payload differ from the host's."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), "NaN positions differ"
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_elementwise_ops_are_bit_exact(session):
    rng = np.random.default_rng(1)
    for n in (1, 3, 4, 1001, 1 << 16):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        if n > 4:
            a[:4] = [np.inf, -np.inf, np.nan, 0.0]
            b[:4] = [np.inf, np.inf, 1.0, -0.0]
        da, db = session.upload(a), session.upload(b)
        for fn, want in ((session.add, a + b), (session.multiply, a * b)):
            y = fn(da, db)
            bits_equal(session.download(y), want)
            session.release(y)
        for s in (0.5, -3.0, np.inf, 0.0):
            y = session.scale(da, s)
            with np.errstate(invalid="ignore"):
                bits_equal(session.download(y), a * np.float32(s))
            session.release(y)
        session.release(da)
        session.release(db)


def test_add_rejects_unequal_shapes(session):
    a, b = session.upload(np.zeros((2, 3), np.float32)), session.upload(np.zeros((3, 2), np.float32))
    with pytest.raises(ffm.IllegalArgumentException):
        session.add(a, b)
    session.release(a)
    session.release(b)


def test_silu_rmsnorm_rope_match_the_oracle(session):
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((3, 4, 5, 64)) * 4).astype(np.float32)
    x.flat[:3] = [np.inf, -np.inf, 0.0]
    dx = session.upload(x)
    y = session.silu(dx)
    got, want = session.download(y), oracle.silu(x)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    fin = np.isfinite(want)
    ulp_close(got[fin], want[fin])
    session.release(y)
    xf = x.copy()
    xf.flat[:3] = 1.0
    dxf = session.upload(xf)
    w = (rng.standard_normal(64) + 1).astype(np.float32)
    dw = session.upload(w)
    y = session.rms_norm(dxf, dw, 1e-5)
    ulp_close(session.download(y), oracle.rmsnorm(xf, w, 1e-5))
    session.release(y)
    for start, theta in ((0, 10000.0), (17, 500000.0)):
        y = session.rope(dxf, start, theta)
        ulp_close(session.download(y), oracle.rope(xf, start, theta))
        session.release(y)
    odd = session.reshape(dxf, (3, 4, 64, 5))
    with pytest.raises(ffm.IllegalArgumentException):
        session.rope(odd)  # odd width
    for t in (dx, dxf, dw, odd):
        session.release(t)


def test_sum_expand_fill(session):
    rng = np.random.default_rng(3)
    for n in (1, 7, 4096, 300001):
        x = rng.standard_normal(n).astype(np.float32)
        dx = session.upload(x)
        s = session.sum(dx)
        assert s.shape == ()
        want = np.float32(np.sum(x.astype(np.float64)))
        ulp_close(session.download(s), np.array(want))
        e = session.expand_scalar(s, (2, 3))
        bits_equal(session.download(e), np.full((2, 3), session.download(s)))
        for t in (dx, s, e):
            session.release(t)
    ints = session.upload(np.arange(1, 101, dtype=np.float32))
    s = session.sum(ints)
    assert float(session.download(s)) == 5050.0
    f = session.fill((4, 5), -2.5)
    bits_equal(session.download(f), np.full((4, 5), -2.5, np.float32))
    for t in (ints, s, f):
        session.release(t)
    vec = session.fill((2,), 1.0)
    with pytest.raises(ffm.IllegalArgumentException):
        session.expand_scalar(vec, (3,))
    session.release(vec)


def test_reshape_views_share_the_allocation(session):
    base = session.allocated_bytes
    x = session.upload(np.arange(24, dtype=np.float32).reshape(2, 3, 4))
    v = session.reshape(x, (6, 4))
    session.release(x)
    assert session.allocated_bytes > base  # the view keeps the allocation
    bits_equal(session.download(v), np.arange(24, dtype=np.float32).reshape(6, 4))
    session.release(v)
    session.release(v)  # idempotent
    assert session.allocated_bytes == base
    four = session.fill((4,), 0.0)
    with pytest.raises(ffm.IllegalArgumentException):
        session.reshape(four, (5,))
    session.release(four)


def test_transpose_and_embedding_are_copies(session):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 3, 4, 5)).astype(np.float32)
    dx = session.upload(x)
    for d0, d1 in ((1, 2), (0, 3), (2, 2), (3, 1)):
        y = session.transpose(dx, d0, d1)
        bits_equal(session.download(y), np.swapaxes(x, d0, d1))
        session.release(y)
    session.release(dx)
    table = oracle.normal_bf16(100 * 48, 5, 5, 1.0).reshape(100, 48)
    ids = np.array([[3, 99, 0], [3, 7, 50]], np.int64)
    for dt, t in ((ffm.STB_BF16, session.upload_half(table, ffm.STB_BF16)),
                  (ffm.STB_F32, session.upload(oracle.widen(table, oracle.BF16)))):
        y = session.embedding(t, ids)
        assert y.shape == (2, 3, 48)
        bits_equal(session.download(y), oracle.widen(table, oracle.BF16)[ids])
        session.release(y)
        with pytest.raises(ffm.IllegalArgumentException):
            session.embedding(t, np.array([100]))
        session.release(t)


@pytest.mark.parametrize("b,h,kv,t,d,dv,start", [(1, 4, 2, 5, 16, 16, 0), (2, 8, 2, 3, 64, 32, 0),
                                                  (2, 6, 3, 7, 32, 32, 0), (1, 2, 1, 1, 128, 128, 0),
                                                  (1, 4, 2, 4, 16, 16, 2)])
def test_causal_attention_matches_the_oracle(session, b, h, kv, t, d, dv, start):
    rng = np.random.default_rng(b * 100 + h)
    q = rng.standard_normal((b, h, t, d)).astype(np.float32)
    k = rng.standard_normal((b, kv, t, d)).astype(np.float32)
    v = rng.standard_normal((b, kv, t, dv)).astype(np.float32)
    dq, dk, dv_ = session.upload(q), session.upload(k), session.upload(v)
    y = session.causal_attention(dq, dk, dv_, start)
    ulp_close(session.download(y), oracle.causal_attention(q, k, v, start), rel=2e-6)
    for x in (dq, dk, dv_, y):
        session.release(x)


def test_attention_cache_appends_and_attends(session):
    """AttentionCache.attend over a capacity-strided cache: prompt chunk then single tokens, against the
    oracle's capacity-strided attention; a gap or an overflow is rejected before any device work."""
    rng = np.random.default_rng(6)
    b, h, kv, d, cap = 2, 4, 2, 32, 16
    cache = session.attention_cache(b, kv, cap, d, d)
    kc = np.zeros((b, kv, cap, d), np.float32)
    vc = np.zeros((b, kv, cap, d), np.float32)
    pos = 0
    for t in (5, 1, 1, 3):
        q = rng.standard_normal((b, h, t, d)).astype(np.float32)
        k = rng.standard_normal((b, kv, t, d)).astype(np.float32)
        v = rng.standard_normal((b, kv, t, d)).astype(np.float32)
        kc[:, :, pos:pos + t], vc[:, :, pos:pos + t] = k, v
        dq, dk, dv = session.upload(q), session.upload(k), session.upload(v)
        y = cache.attend(dq, dk, dv, pos)
        want = oracle.causal_attention(q, kc, vc, start=pos, key_stride=cap, keys=pos + t)
        ulp_close(session.download(y), want, rel=2e-6)
        for x in (dq, dk, dv, y):
            session.release(x)
        pos += t
    one = [session.upload(rng.standard_normal((b, n, 1, d)).astype(np.float32)) for n in (h, kv, kv)]
    with pytest.raises(ffm.IllegalArgumentException):
        cache.attend(*one, pos + 1)  # gap
    cache.close()
    for x in one:
        session.release(x)


def _lora(config, seed):
    rng = np.random.default_rng(seed)
    H, I = config.hidden_size, config.intermediate_size
    kvw = config.num_key_value_heads * config.head_dim

    def pair(out, inp, rank):
        return ((rng.uniform(-1, 1, (rank, inp)) / np.sqrt(inp)).astype(np.float32),
                (rng.standard_normal((out, rank)) * 0.05).astype(np.float32), 8.0)

    return {"model.layers.0.self_attn.q_proj": pair(H, H, 4), "model.layers.0.self_attn.v_proj": pair(kvw, H, 2),
            "model.layers.0.mlp.down_proj": pair(H, I, 8), "model.layers.1.mlp.gate_proj": pair(I, H, 4)}


@pytest.mark.parametrize("with_lora", [False, True])
def test_per_op_llama_matches_the_reference_per_op_path(session, with_lora):
    """PerOpLlama through the C ABI, op for op as BackendLlama.run, against the reference's per-op path on
    the CPU backend: logits of a 2-row prompt chunk and two single-token steps within 1e-5 (1 + |e|),
    greedy ids identical; with adapters on four projections (BackendLlama.linear's LoRA order)."""
    cfg = LlamaConfig(**TINY)
    w = named_bf16_weights(cfg, 11)
    lora = _lora(cfg, 12) if with_lora else None
    cpu = CpuPerOpLlama(cfg, w, lora)
    dtypes = {k: ffm.STB_BF16 for k in w}
    with PerOpLlama(session, cfg, w, dtypes, lora) as m:
        cache = m.new_cache(2, 12)
        caches = cpu.new_cache(2, 12)
        prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, (2, 5))
        got = cache.decode(prompt)
        want = cpu.forward(prompt, 0, caches)
        np.testing.assert_array_less(np.abs(got - want), 1e-5 * (1 + np.abs(want)) + 1e-30)
        for step, tok in enumerate(([[5], [9]], [[600], [2]])):
            got = cache.decode(tok)
            want = cpu.forward(np.array(tok), 5 + step, caches)
            np.testing.assert_array_less(np.abs(got - want), 1e-5 * (1 + np.abs(want)) + 1e-30)
        assert cache.position == 7
        cache.close()
        prompt1 = [1, 17, 400, 999, 3]
        assert m.generate_ids(prompt1, 12) == cpu.generate(prompt1, 12)
        if not with_lora:  # the fused runtime takes the same model: same ids
            with BackendLlama.prepare_random(session, cfg, seed=11) as fused:
                assert fused.generate_ids(prompt1, 12) == m.generate_ids(prompt1, 12)
    assert session.allocated_bytes >= 0


def test_per_op_llama_smollm2_shape_with_tied_head(session):
    """The SmolLM2 shape (tied embeddings: the head is a view of the table) on the per-op path: greedy
    ids identical to the oracle's Llama decode on a short prompt."""
    cfg = LlamaConfig(**SMOL)
    w = named_bf16_weights(cfg, 2024)
    ref = oracle_model(cfg, seed=2024)
    prompt = [5, 9, 700, 12, 44, 3000]
    with PerOpLlama(session, cfg, w, {k: ffm.STB_BF16 for k in w}) as m:
        assert m.generate_ids(prompt, 5) == ref.generate(prompt, 5)
