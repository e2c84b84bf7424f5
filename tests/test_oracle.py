"""The CPU oracle against scala-torch's own known answers (tests/golden/reference_vectors.json).

Pins the restatement before any device result is compared with it.
"""
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.json")))["cases"]


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32).tolist()


def check_bits(actual, expected):
    for a, e in zip(bits(actual), expected):
        if e == "nan":
            assert (a & 0x7F800000) == 0x7F800000 and (a & 0x7FFFFF) != 0
        else:
            assert a == e


def test_bf16_widening_table():
    g = GOLDEN["bf16_decode"]
    check_bits(oracle.widen(np.array(g["bits"], np.uint16), oracle.BF16), g["expected_f32_bits"])


def test_f16_widening_table():
    g = GOLDEN["f16_decode"]
    check_bits(oracle.widen(np.array(g["bits"], np.uint16), oracle.F16), g["expected_f32_bits"])


def test_chunked_decode_crosses_64k_boundaries():
    g = GOLDEN["chunked_decode"]
    n = g["count"]
    for words, expected, dt in ((g["f16_words"], g["f16_expected"], oracle.F16),
                                (g["bf16_words"], g["bf16_expected"], oracle.BF16)):
        src = np.array([words[i % len(words)] for i in range(n)], np.uint16)
        out = oracle.widen(src, dt)
        want = np.array([expected[i % len(expected)] for i in range(n)], np.float32)
        assert np.array_equal(out, want)


def test_bf16_rne_matches_writer_rule():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38, 1e-40, -1e-42], np.float32)])
    u = x.view(np.uint32).astype(np.uint64)
    want = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # SafeTensorsWriter.scala:58-61
    assert np.array_equal(oracle.round_bf16(x), want)
    nan = np.array([0x7FC00001, 0x7F800001, 0xFF812345], np.uint32).view(np.float32)
    assert oracle.round_bf16(nan).tolist() == [((int(b) >> 16) | 0x40) & 0xFFFF for b in nan.view(np.uint32)]


def test_f16_rounding_agrees_with_numpy():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(50000).astype(np.float32) * 1000,
                        rng.standard_normal(5000).astype(np.float32) * 1e-6,
                        np.array([65504, 65519.99, 65520, 1e-8, 2.0 ** -25, 2.0 ** -24], np.float32)])
    with np.errstate(over="ignore"):  # 65520 and the large normals round to infinity on purpose
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.round_f16(x), want)


def test_upstream_safetensors_linear_is_24_52():
    g = GOLDEN["upstream_safetensors"]
    w = np.array(g["weight"], np.float32).reshape(g["weight_shape"])
    x = np.array([g["input"]], np.float32)
    for order in (oracle.ORDER_NUMSCALA, oracle.ORDER_SEQUENTIAL):
        y = oracle.linear(x, w, oracle.F32, np.array(g["bias"], np.float32), order=order)
        assert y.ravel().tolist() == g["expected"]
    # the fixture's half payloads decode to the documented values
    assert oracle.widen(np.array(g["half_bits"], np.uint16), oracle.F16).tolist() == [1.0, -2.0, 2.0 ** -24, 65504.0]
    b = oracle.widen(np.array(g["bfloat_bits"], np.uint16), oracle.BF16)
    assert b[:3].tolist() == [1.0, -2.0, 2.0 ** -133] and math.isnan(b[3])


@pytest.mark.parametrize("case", ["gemm_small", "gemm_2x2"])
def test_gemm_known_answers(case):
    g = GOLDEN[case]
    a = np.array(g["a"], np.float32)
    b = np.array(g["b"], np.float32)
    assert oracle.matmul_seq(a, b).tolist() == g["expected"]
    assert oracle.matmul_tr(a, np.ascontiguousarray(b.T)).tolist() == g["expected"]


def test_gemm_probe_patterns_exact():
    for c in GOLDEN["gemm_probe_patterns"]["cases"]:
        m, n, k = c["m"], c["n"], c["k"]
        a = np.array([(i % 11 - 5) / 8 for i in range(m * k)], np.float32).reshape(m, k)
        b = np.array([(i % 7 - 3) / 4 for i in range(k * n)], np.float32).reshape(k, n)
        assert oracle.matmul_seq(a, b).ravel().tolist() == c["expected"]
        assert oracle.matmul_tr(a, np.ascontiguousarray(b.T)).ravel().tolist() == c["expected"]


def test_gemm_empty_inner_and_nan_times_zero():
    g = GOLDEN["gemm_empty_inner"]
    y = oracle.linear(np.zeros((g["M"], 0), np.float32), np.zeros((g["N"], 0), np.float32), oracle.F32)
    assert y.ravel().tolist() == g["expected"]
    y = oracle.linear(np.zeros((1, 1), np.float32), np.full((1, 1), np.nan, np.float32), oracle.F32)
    assert np.isnan(y[0, 0])


def test_numscala_order_is_four_partial_sums():
    # A case that separates the two orders: large cancellation in lane 0.
    x = np.array([[1e8, 1.0, 1.0, 1.0, -1e8, 1.0]], np.float32)
    w = np.ones((1, 6), np.float32)
    # numscala: s0 = 1e8 + -1e8 = 0 (k=0,4), s1 = 1 + 1 (k=1 and tail k=5 -> s0!), exactly:
    #   k=0..3 -> s0=1e8 s1=1 s2=1 s3=1 ; tail k=4 -> s0=0, k=5 -> s0=1 ; (1+1)+(1+1) = 4
    assert oracle.matmul_tr(x, w).item() == 4.0
    # sequential: ((1e8+1+1+1) - 1e8) + 1 = 0 + 1 with float rounding of 1e8+1 -> 1e8
    assert oracle.matmul_seq(x, np.ascontiguousarray(w.T)).item() == 1.0


def test_orders_agree_within_tolerance_on_random_data():
    rng = np.random.default_rng(2)
    for k in list(range(1, 8)) + [576, 577, 578, 579]:
        x = (rng.standard_normal((3, k)) * 3).astype(np.float32)
        w = (rng.standard_normal((5, k)) * 3).astype(np.float32)
        a = oracle.matmul_tr(x, w)
        b = oracle.matmul_seq(x, np.ascontiguousarray(w.T))
        ref = x.astype(np.float64) @ w.astype(np.float64).T
        # Higham's bound for recursive Float32 summation: |err| <= gamma_K * sum |x_k w_k|.
        bound = (k * 2.0 ** -24) / (1 - k * 2.0 ** -24) * (np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T)
        assert np.all(np.abs(a - ref) <= bound)
        assert np.all(np.abs(b - ref) <= bound)


def test_rmsnorm_silu_embedding_known_answers():
    g = GOLDEN["rmsnorm"]
    y = oracle.rmsnorm(np.array(g["x"], np.float32), np.array(g["w"], np.float32), g["eps"])
    assert bits(y.ravel()) == g["expected_f32_bits"]
    g = GOLDEN["silu"]
    s = oracle.silu(np.array(g["x"] + [-np.inf, np.inf, np.nan], np.float32))
    assert abs(s[0] - g["expected"][0]) < g["tol"] and abs(s[1] - g["expected"][1]) < g["tol"]
    assert bits(s[2:3]) == [g["neg_inf_bits"]] and s[3] == np.inf and np.isnan(s[4])


def test_rope_and_attention_known_answers():
    g = GOLDEN["rope"]
    y = oracle.rope(np.array(g["x"], np.float32).reshape(1, 1, 1, 4), g["start"], g["theta"]).ravel()
    assert abs(y[0] - g["expected"][0]) < g["tol"] and abs(y[1] - g["expected"][1]) < g["tol"]
    g = GOLDEN["attention"]
    q = np.zeros(g["q_shape"], np.float32)
    k = np.zeros(g["k_shape"], np.float32)
    v = np.array(g["v"], np.float32).reshape(g["v_shape"])
    assert oracle.causal_attention(q, k, v, 0).ravel().tolist() == g["expected_start0"]
    assert oracle.causal_attention(q, k, v, 1).ravel().tolist() == g["expected_start1"]


def test_greedy_lowest_index_wins_ties():
    g = GOLDEN["greedy_ties"]
    assert oracle.argmax(np.array(g["logits"], np.float32)) == g["expected"]
    assert oracle.argmax(np.array([-0.0, 0.0], np.float32)) == 0


def test_rng_is_normal_and_counter_addressed():
    z = np.array([oracle.rng_normal(7, 3, i) for i in range(200000)])
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    assert abs(np.mean(np.abs(z) < 1) - 0.6827) < 0.005
    # counter-based: any slice regenerates independently
    a = oracle.normal_bf16(1000, 5, 9, 0.02)
    assert np.array_equal(a[500:], np.array([oracle.round_bf16(np.array([np.float32(0.02 * oracle.rng_normal(5, 9, i))]))[0]
                                             for i in range(500, 1000)], np.uint16))
    assert not np.array_equal(oracle.normal_bf16(64, 5, 9, 0.02), oracle.normal_bf16(64, 5, 10, 0.02))


def test_log_restatement_is_accurate():
    for x in [1e-300, 1e-20, 0.001, 0.25, 0.5, 0.70710678, 0.75, 0.999999, 1.0 - 2.0 ** -52]:
        assert abs(oracle.lib().oracle_log(x) - math.log(x)) <= 4e-16 * max(1.0, abs(math.log(x)))


def test_linear_adapters_known_answer():
    """Linear.apply with its adapter, two LinearAdapterScope entries and a bias (Linear.scala:11-17),
    small integers so every step is exact: base [1,2]; own adapter adds ((x.A^T).B^T)*1 = [3,6];
    scoped (scale 2, multiplier 0.5) adds [1,1]; scoped (scale 1, multiplier -1) adds [-2,-2]."""
    x = np.array([[1.0, 2.0]], np.float32)
    w = oracle.round_bf16(np.eye(2, dtype=np.float32))
    own = (np.array([[1.0, 1.0]]), np.array([[1.0], [2.0]]), 1.0)
    half = (np.array([[1.0, 0.0]]), np.array([[1.0], [1.0]]), 2.0)
    neg = (np.array([[0.0, 1.0]]), np.array([[1.0], [1.0]]), 1.0)
    y = oracle.linear_adapted(x, w, oracle.BF16, np.array([0.5, -1.0], np.float32), lora=own,
                              scoped=[(half, 0.5), (neg, -1.0)])
    assert y.tolist() == [[1 + 3 + 1 - 2 + 0.5, 2 + 6 + 1 - 2 - 1.0]]


def test_linear_adapter_with_zero_up_factor_is_the_base_product():
    """LowRankAdapter.init zero-fills B (LowRankAdapter.scala:37): the adapted Linear equals the
    plain Linear bit for bit."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 40)).astype(np.float32)
    w = oracle.round_bf16(rng.standard_normal((7, 40)).astype(np.float32))
    b = rng.standard_normal(7).astype(np.float32)
    own = (rng.standard_normal((4, 40)).astype(np.float32), np.zeros((7, 4), np.float32), 8.0)
    assert np.array_equal(oracle.linear_adapted(x, w, oracle.BF16, b, lora=own), oracle.linear(x, w, oracle.BF16, b))
    assert oracle.adapter_scale(8.0, 4) == np.float32(2.0)
    with pytest.raises(ValueError):
        oracle.adapter_scale(0.0, 4)
