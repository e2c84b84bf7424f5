"""Parity of the device Linear (stb_linear, decode GEMV family) with the CPU oracle.

Tolerance: |y - ref| <= 1e-5 * (1 + |ref|) for BF16/F16-weight GEMV with
Float32 activations and FP32 accumulation; the reference's own form |a-e| <= tol*(1+|e|)
(models/src/test/scala/scalatorch/models/BackendLlamaSuite.scala:18).
"""
import json
import os

import numpy as np
import pytest

import oracle
from scalatorch import ffm

pytestmark = pytest.mark.gpu
GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.json")))["cases"]
TOL = 1e-5


def close(y, ref, tol=TOL):
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    lim = tol * (1 + np.abs(ref.astype(np.float64)))
    assert np.all(err <= lim), f"max err {err.max()} (worst ratio {np.max(err / lim)})"


def run_linear(session, x, w_bits, dtype, bias=None):
    xd = session.upload(x)
    wd = session.upload_weight(w_bits, dtype) if dtype != ffm.STB_F32 else None
    if wd is None:
        wd = session.upload(w_bits)
        wd.shape = (w_bits.shape[1], w_bits.shape[0])
        wd.transposed_weight = True
    bd = session.upload(bias) if bias is not None else None
    y = session.linear(xd, wd, bd)
    out = session.download(y)
    for t in (xd, wd, y) + ((bd,) if bd is not None else ()):
        session.release(t)
    return out


def test_config1_single_linear(session):
    """The single-Linear configuration: x F32 [16,576] ~N(0,1); W BF16 [1536,576] N(0,0.02) RNE; no bias."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal((16, 576)).astype(np.float32)
    w = oracle.normal_bf16(1536 * 576, seed=1, stream=1, std=0.02).reshape(1536, 576)
    y = run_linear(session, x, w, ffm.STB_BF16)
    close(y, oracle.linear(x, w, oracle.BF16))
    close(y, oracle.linear(x, w, oracle.BF16, order=oracle.ORDER_SEQUENTIAL))


@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 6, 7, 8, 576, 577, 578, 579])
@pytest.mark.parametrize("dtype", [ffm.STB_BF16, ffm.STB_F16])
def test_complete_groups_and_tails(session, k, dtype):
    """CudaOpsSuite.scala:34-47 widths (K in 1..7, 576..579), here within tolerance."""
    rng = np.random.default_rng(k)
    x = (rng.standard_normal((3, k)) * 3).astype(np.float32)
    wf = (rng.standard_normal((5, k)) * 3).astype(np.float32)
    w = oracle.round_bf16(wf) if dtype == ffm.STB_BF16 else oracle.round_f16(wf)
    y = run_linear(session, x, w, dtype)
    ref = oracle.linear(x, w, oracle.BF16 if dtype == ffm.STB_BF16 else oracle.F16)
    wide = oracle.widen(w, oracle.BF16 if dtype == ffm.STB_BF16 else oracle.F16).astype(np.float64)
    bound = 2 * k * 2.0 ** -24 * (np.abs(x).astype(np.float64) @ np.abs(wide).T) + 1e-30
    assert np.all(np.abs(y - ref) <= 2 * bound)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 16, 31, 32, 33, 64])
def test_decode_batches(session, m):
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, 1024)).astype(np.float32)
    w = oracle.normal_bf16(3000 * 1024, seed=m, stream=2, std=0.02).reshape(3000, 1024)
    close(run_linear(session, x, w, ffm.STB_BF16), oracle.linear(x, w, oracle.BF16))


SKINNY_SHAPES = [(2, 1000, 1000), (9, 128, 64), (16, 1000, 4104), (17, 300, 2048), (40, 1536, 576), (64, 2500, 1000),
                 (100, 576, 576), (300, 1536, 576)]
SKINNY_MIN_WORK = 1 << 24  # products up to this many multiply-adds take the GEMV


@pytest.mark.parametrize("m,n,k", SKINNY_SHAPES)
def test_skinny_tensor_core_form(session, m, n, k):
    """Two or more rows with BF16 weights and more than 2^24 multiply-adds run on the tensor cores
    (per 64-row block: prologue, stream-K GEMM, fixup), activations split into three BF16 terms:
    still within the FP32 GEMV tolerance; smaller products take the one-launch GEMV.
    Ragged N (tile tails), K tails below one 64-wide block, bias; repeated calls are identical.
    Magnitudes as the single-Linear configuration (x ~ N(0,1), W ~ N(0, 0.02)): the bound is relative
    to |y| ~ 1.  test_skinny_form_on_small_products runs the small shapes on the tensor cores too."""
    rng = np.random.default_rng(m * 7 + n)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = oracle.normal_bf16(n * k, seed=m, stream=9, std=0.02).reshape(n, k)
    b = rng.standard_normal(n).astype(np.float32)
    xd, wd, bd = session.upload(x), session.upload_weight(w, ffm.STB_BF16), session.upload(b)
    l0 = session.launches
    y1 = session.linear(xd, wd, bd)
    assert session.launches - l0 == (3 * ((m + 63) // 64) if m * n * k > SKINNY_MIN_WORK else 1)
    y2 = session.linear(xd, wd, bd)
    a1, a2 = session.download(y1), session.download(y2)
    for t in (xd, wd, bd, y1, y2):
        session.release(t)
    assert np.array_equal(a1.view(np.uint32), a2.view(np.uint32))
    close(a1, oracle.linear(x, w, oracle.BF16, b))


def test_skinny_form_on_small_products():
    """The skinny tensor-core form forced onto the products the library routes to the GEMV
    (STB_SKINNY_MIN_WORK=0, read once per process: a child process) keeps its tolerance and launch
    count on every shape of test_skinny_tensor_core_form."""
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    paths = [here, os.path.dirname(here), os.path.join(os.path.dirname(here), "scala-torch_b200")]
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = {paths!r}\n"
        "import oracle\n"
        "from scalatorch import ffm\n"
        "from test_linear_gpu import SKINNY_SHAPES, close\n"
        "s = ffm.B200Session(0, 8 << 30)\n"
        "for m, n, k in SKINNY_SHAPES:\n"
        "    rng = np.random.default_rng(m * 7 + n)\n"
        "    x = rng.standard_normal((m, k)).astype(np.float32)\n"
        "    w = oracle.normal_bf16(n * k, seed=m, stream=9, std=0.02).reshape(n, k)\n"
        "    b = rng.standard_normal(n).astype(np.float32)\n"
        "    xd, wd, bd = s.upload(x), s.upload_weight(w, ffm.STB_BF16), s.upload(b)\n"
        "    l0 = s.launches\n"
        "    y = s.linear(xd, wd, bd)\n"
        "    assert s.launches - l0 == 3 * ((m + 63) // 64), (m, n, k)\n"
        "    close(s.download(y), oracle.linear(x, w, oracle.BF16, b))\n"
        "    for t in (xd, wd, bd, y):\n"
        "        s.release(t)\n"
        "s.close()\n"
        "print('ok')\n")
    env = dict(os.environ, STB_SKINNY_MIN_WORK="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]


FLT_MAX = float(np.finfo(np.float32).max)
SPECIALS = ("inf", "-inf", "nan", "max", "-max", "subnormal")
NONFINITE_MS = (1, 2, 17, 64)


def nonfinite_case(m, rotation, n=256, k=576):
    """x ~ N(0,1) [m,k] with one IEEE special per row (row r gets SPECIALS[(r + rotation) % 6] at column
    (7 r + 3) % k; "subnormal" makes the whole row subnormal), W ~ N(0,0.02) BF16 [n,k] with row 5 all
    zeros (0 x Inf = NaN, as the reference's CPU product gives).  One special per row keeps every
    finite sum far from overflow, so the reduction order cannot decide a row's class."""
    rng = np.random.default_rng(1000 * m + rotation)
    x = rng.standard_normal((m, k)).astype(np.float32)
    for r in range(m):
        kind, col = SPECIALS[(r + rotation) % len(SPECIALS)], (7 * r + 3) % k
        if kind == "subnormal":
            x[r] = (rng.standard_normal(k) * 1e-39).astype(np.float32)
        else:
            x[r, col] = {"inf": np.inf, "-inf": -np.inf, "nan": np.nan, "max": FLT_MAX, "-max": -FLT_MAX}[kind]
    w = oracle.normal_bf16(n * k, seed=m, stream=40 + rotation, std=0.02).reshape(n, k)
    w[5] = 0
    return x, w


def same_class(y, ref, tol=TOL):
    """IEEE class element for element (NaN where NaN, the same signed infinities), finite values
    within tol * (1 + |e|)."""
    assert np.array_equal(np.isnan(y), np.isnan(ref)), "NaN positions differ"
    assert np.array_equal(np.isposinf(y), np.isposinf(ref)) and np.array_equal(np.isneginf(y), np.isneginf(ref)), \
        "infinities differ"
    fin = np.isfinite(ref)
    close(y[fin], ref[fin], tol)


def test_nonfinite_activations_on_the_gemv(session):
    """The reference's CPU Linear keeps IEEE semantics (cpu/src/test/scala/scalatorch/cpu/BackendSuite.scala:22-43):
    +-Inf, NaN, +-FLT_MAX and subnormal activations on the products the library runs as the vector GEMV
    (every M below the skinny form's work threshold, these included)."""
    for m in NONFINITE_MS:
        for rot in range(len(SPECIALS)):
            x, w = nonfinite_case(m, rot)
            same_class(run_linear(session, x, w, ffm.STB_BF16), oracle.linear(x, w, oracle.BF16))


def test_nonfinite_activations_on_the_skinny_form():
    """The same IEEE cases on the tensor-core skinny form (STB_SKINNY_MIN_WORK=0 routes every M there, one
    row included; read once per process, so a child process): the three-term BF16 split keeps Inf / NaN
    in its first term and truncates a finite value above BF16's largest, so no Inf - Inf appears."""
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    paths = [here, os.path.dirname(here), os.path.join(os.path.dirname(here), "scala-torch_b200")]
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = {paths!r}\n"
        "import oracle\n"
        "from scalatorch import ffm\n"
        "from test_linear_gpu import NONFINITE_MS, SPECIALS, nonfinite_case, same_class\n"
        "s = ffm.B200Session(0, 8 << 30)\n"
        "for m in NONFINITE_MS:\n"
        "    for rot in range(len(SPECIALS)):\n"
        "        x, w = nonfinite_case(m, rot)\n"
        "        xd, wd = s.upload(x), s.upload_weight(w, ffm.STB_BF16)\n"
        "        l0 = s.launches\n"
        "        y = s.linear(xd, wd)\n"
        "        assert s.launches - l0 == 3, (m, s.launches - l0)\n"
        "        same_class(s.download(y), oracle.linear(x, w, oracle.BF16))\n"
        "        for t in (xd, wd, y):\n"
        "            s.release(t)\n"
        "s.close()\n"
        "print('ok')\n")
    env = dict(os.environ, STB_SKINNY_MIN_WORK="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]


def test_f16_weights_and_bias(session):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 4096)).astype(np.float32)
    w = oracle.round_f16(rng.standard_normal((1024, 4096)).astype(np.float32) * 0.02)
    b = rng.standard_normal(1024).astype(np.float32)
    close(run_linear(session, x, w, ffm.STB_F16, b), oracle.linear(x, w, oracle.F16, b))


def test_known_answers_through_the_device(session):
    g = GOLDEN["upstream_safetensors"]  # SafeWeightsSuite.scala:10-24 -> [24, 52]
    w = np.array(g["weight"], np.float32).reshape(g["weight_shape"])
    y = run_linear(session, np.array([g["input"]], np.float32), w, ffm.STB_F32, np.array(g["bias"], np.float32))
    assert y.ravel().tolist() == g["expected"]
    g = GOLDEN["gemm_small"]  # BackendSuite.scala:22-43 -> [58,64,139,154], exact in BF16
    w = oracle.round_bf16(np.ascontiguousarray(np.array(g["b"], np.float32).T))
    y = run_linear(session, np.array(g["a"], np.float32), w, ffm.STB_BF16)
    assert y.tolist() == g["expected"]
    for c in GOLDEN["gemm_probe_patterns"]["cases"]:  # CudaProbeSuite.scala:17-28, exact
        m, n, k = c["m"], c["n"], c["k"]
        a = np.array([(i % 11 - 5) / 8 for i in range(m * k)], np.float32).reshape(m, k)
        b = np.array([(i % 7 - 3) / 4 for i in range(k * n)], np.float32).reshape(k, n)
        y = run_linear(session, a, oracle.round_bf16(np.ascontiguousarray(b.T)), ffm.STB_BF16)
        assert y.ravel().tolist() == c["expected"]


def test_nan_times_zero_propagates(session):
    y = run_linear(session, np.zeros((1, 8), np.float32), oracle.round_bf16(np.full((1, 8), np.nan, np.float32)),
                   ffm.STB_BF16)
    assert np.isnan(y[0, 0])


def test_empty_shapes(session):
    y = run_linear(session, np.zeros((2, 0), np.float32), np.zeros((3, 0), np.uint16), ffm.STB_BF16)
    assert y.tolist() == [[0.0] * 3] * 2


def test_llama8b_projection_shapes_against_fp32(session):
    """Llama-3-8B projection shapes at M = 1, 4, 16, 32 against a float64 product of the same widened
    weights (an fp32 cuBLAS reference carries its own rounding at the 1e-5 level)."""
    import torch
    shapes = {"q": (4096, 4096), "k": (1024, 4096), "gate": (14336, 4096), "down": (4096, 14336),
              "lm_head": (128256, 4096)}
    for stream, (name, (n, k)) in enumerate(shapes.items()):
        w = torch.empty(n * k, dtype=torch.bfloat16, device="cuda")
        wt = ffm.DeviceTensor(session, w.data_ptr(), (k, n), ffm.STB_BF16, w.numel() * 2,
                              transposed_weight=True, owner=False)
        session.fill_normal(wt, seed=11, stream=stream, std=0.02)
        session.sync()
        wf = w.view(n, k).double()
        for m in (1, 4, 16, 32):
            x = torch.randn(m, k, device="cuda", generator=torch.Generator("cuda").manual_seed(m))
            torch.cuda.synchronize()
            xt = ffm.DeviceTensor(session, x.data_ptr(), (m, k), ffm.STB_F32, x.numel() * 4, owner=False)
            y = session.linear(xt, wt)
            got = session.download(y)
            session.release(y)
            ref = (x.double() @ wf.T).cpu().numpy()
            close(got, ref)
        del w, wf
        torch.cuda.empty_cache()


def test_device_generator_matches_oracle_bits(session):
    for dtype, odt in ((ffm.STB_BF16, "bf16"), (ffm.STB_F32, "f32")):
        t = session.allocate((100003,), dtype)
        session.fill_normal(t, seed=123, stream=77, std=0.02)
        raw = session.download_raw(t)
        session.release(t)
        if odt == "bf16":
            assert np.array_equal(raw.view(np.uint16), oracle.normal_bf16(100003, 123, 77, 0.02))
        else:
            assert np.array_equal(raw.view(np.float32), oracle.normal_f32(100003, 123, 77, 0.02))


def test_budget_rejects_before_allocation():
    with ffm.B200Session(0, 1 << 20) as s:
        with pytest.raises(ffm.IllegalStateException):
            s.allocate((1 << 20,), ffm.STB_F32)
        assert s.allocated_bytes == 0


def _adapter(session, rng, n, k, rank, alpha, zero_b=False):
    a = (rng.uniform(-1, 1, (rank, k)) / np.sqrt(k)).astype(np.float32)
    b = np.zeros((n, rank), np.float32) if zero_b else (rng.standard_normal((n, rank)) * 0.1).astype(np.float32)
    dev = ffm.LowRankAdapter(session.upload(a), session.upload(b), alpha)
    return (a, b, alpha), dev


@pytest.mark.parametrize("m", [1, 3, 16, 40])
def test_linear_with_adapters_matches_oracle(session, m):
    """nn.Linear.apply with its own LoRA adapter, two LinearAdapterScope entries (one with a negative
    multiplier) and a bias (Linear.scala:11-17), in the reference's operation order; the base
    product takes the GEMV below the skinny form's work threshold (M = 1, 3, 16 here) or the skinny
    tensor-core form (M = 40)."""
    rng = np.random.default_rng(m)
    n, k = 1536, 576
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = oracle.normal_bf16(n * k, seed=m, stream=5, std=0.02).reshape(n, k)
    b = rng.standard_normal(n).astype(np.float32)
    own, own_d = _adapter(session, rng, n, k, 8, 16.0)
    s1, s1_d = _adapter(session, rng, n, k, 4, 4.0)
    s2, s2_d = _adapter(session, rng, n, k, 16, 8.0)
    xd, wd, bd = session.upload(x), session.upload_weight(w, ffm.STB_BF16), session.upload(b)
    y = session.linear(xd, wd, bd, lora=own_d, scoped=[(s1_d, 0.75), (s2_d, -1.5)])
    got = session.download(y)
    close(got, oracle.linear_adapted(x, w, oracle.BF16, b, lora=own, scoped=[(s1, 0.75), (s2, -1.5)]))
    for t in (xd, wd, bd, y, own_d.a, own_d.b, s1_d.a, s1_d.b, s2_d.a, s2_d.b):
        session.release(t)


def test_fresh_adapter_leaves_the_linear_unchanged(session):
    """LowRankAdapter.init zero-fills B (LowRankAdapter.scala:37): the adapted device Linear equals
    the plain device Linear bit for bit."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal((5, 576)).astype(np.float32)
    w = oracle.normal_bf16(1536 * 576, seed=9, stream=6, std=0.02).reshape(1536, 576)
    b = rng.standard_normal(1536).astype(np.float32)
    _, own_d = _adapter(session, rng, 1536, 576, 8, 16.0, zero_b=True)
    xd, wd, bd = session.upload(x), session.upload_weight(w, ffm.STB_BF16), session.upload(b)
    plain, adapted = session.linear(xd, wd, bd), session.linear(xd, wd, bd, lora=own_d)
    assert np.array_equal(session.download(plain).view(np.uint32), session.download(adapted).view(np.uint32))
    with pytest.raises(ffm.IllegalArgumentException):
        bad = ffm.LowRankAdapter(own_d.a, session.upload(np.zeros((10, 8), np.float32)), 16.0)
        session.linear(xd, wd, bd, lora=bad)
    with pytest.raises(ffm.IllegalArgumentException):
        ffm.LowRankAdapter(own_d.a, own_d.b, 0.0)
