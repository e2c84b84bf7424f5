"""The tcgen05 prefill Linear (stb_linear_prefill) against the CPU oracle.

Tolerance source: the activations are rounded to the weight's 16-bit type
for the tensor cores.  Checked two ways:
* against the oracle on the *rounded* activations (exact products, only the accumulation order
  differs): |y - e| <= 1e-4 * (1 + |e|) elementwise;
* against the oracle on the Float32 activations (the reference's own arithmetic): normwise
  relative error ||y - e|| / ||e|| <= 2e-3.
"""
import numpy as np
import pytest

import oracle
from scalatorch import ffm

pytestmark = pytest.mark.gpu


def run_prefill(session, x, w_bits, dtype, bias=None):
    xd = session.upload(x)
    wd = session.upload_weight(w_bits, dtype)
    bd = session.upload(bias) if bias is not None else None
    y = session.linear(xd, wd, bd, prefill=True)
    out = session.download(y)
    for t in (xd, wd, y) + ((bd,) if bd is not None else ()):
        session.release(t)
    return out


def check(y, x, w_bits, odt, bias=None):
    xr = oracle.widen(oracle.round_bf16(x) if odt == oracle.BF16 else oracle.round_f16(x), odt)
    e = oracle.linear(xr, w_bits, odt, bias)
    err = np.abs(y.astype(np.float64) - e)
    assert np.all(err <= 1e-4 * (1 + np.abs(e))), f"max err {err.max()}"
    full = oracle.linear(x, w_bits, odt, bias)
    rel = np.linalg.norm(y.astype(np.float64) - full) / np.linalg.norm(full)
    assert rel <= 2e-3, rel


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 576), (300, 1000, 200), (1, 8, 8), (129, 257, 136)])
def test_prefill_shapes_bf16(session, m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = oracle.normal_bf16(n * k, seed=m, stream=n, std=0.02).reshape(n, k)
    check(run_prefill(session, x, w, ffm.STB_BF16), x, w, oracle.BF16)


def test_prefill_f16_weights_and_bias(session):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((384, 512)).astype(np.float32)
    w = oracle.round_f16(rng.standard_normal((768, 512)).astype(np.float32) * 0.02)
    b = rng.standard_normal(768).astype(np.float32)
    check(run_prefill(session, x, w, ffm.STB_F16, b), x, w, oracle.F16, b)


def test_prefill_rejects_bad_k(session):
    x = session.upload(np.zeros((4, 12), np.float32))
    w = session.upload_weight(np.zeros((8, 12), np.uint16), ffm.STB_BF16)
    with pytest.raises(ffm.IllegalArgumentException):
        session.linear(x, w, prefill=True)
    session.release(x)
    session.release(w)


def test_llama8b_prefill_shapes_sampled_rows(session):
    """Llama-3-8B prefill shapes at M = 2048 against a float64 product on sampled output rows."""
    import torch
    shapes = {"q": (4096, 4096), "k": (1024, 4096), "gate": (14336, 4096), "down": (4096, 14336),
              "lm_head": (128256, 4096)}
    M = 2048
    for stream, (name, (n, k)) in enumerate(shapes.items()):
        w = torch.empty(n * k, dtype=torch.bfloat16, device="cuda")
        wt = ffm.DeviceTensor(session, w.data_ptr(), (k, n), ffm.STB_BF16, w.numel() * 2,
                              transposed_weight=True, owner=False)
        session.fill_normal(wt, seed=21, stream=stream, std=0.02)
        x = torch.randn(M, k, device="cuda", generator=torch.Generator("cuda").manual_seed(stream))
        torch.cuda.synchronize()
        session.sync()
        xt = ffm.DeviceTensor(session, x.data_ptr(), (M, k), ffm.STB_F32, x.numel() * 4, owner=False)
        y = session.linear(xt, wt, prefill=True)
        got = session.download(y)
        session.release(y)
        rows = torch.tensor([0, 1, 127, 128, 1000, 2047], device="cuda")
        xr = x[rows].to(torch.bfloat16).double()
        ref = (xr @ w.view(n, k).double().T).cpu().numpy()
        sub = got[rows.cpu().numpy()]
        err = np.abs(sub - ref)
        assert np.all(err <= 1e-4 * (1 + np.abs(ref))), (name, err.max())
        full = (x[rows].double() @ w.view(n, k).double().T).cpu().numpy()
        assert np.linalg.norm(sub - full) / np.linalg.norm(full) <= 2e-3, name
        del w, x
        torch.cuda.empty_cache()


def test_single_cta_kernel_matches_oracle():
    """The single-CTA GEMM (STB_GEMM_PAIR=0: tcgen05.mma.cta_group::1, 128 x 256 tiles; the default is
    the CTA-pair kernel) on the shapes above, in a child process because the switch is read once per
    process."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    paths = [here, os.path.dirname(here), os.path.join(os.path.dirname(here), "scala-torch_b200")]
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = {paths!r}\n"
        "import oracle\n"
        "from scalatorch import ffm\n"
        "from test_prefill_gpu import check, run_prefill\n"
        "s = ffm.B200Session(0, 8 << 30)\n"
        "for m, n, k in [(128, 256, 64), (256, 512, 576), (300, 1000, 200), (1, 8, 8), (129, 257, 136),\n"
        "                (1000, 3000, 1024)]:\n"
        "    rng = np.random.default_rng(m * 7 + n + k)\n"
        "    x = rng.standard_normal((m, k)).astype(np.float32)\n"
        "    w = oracle.normal_bf16(n * k, seed=m, stream=n, std=0.02).reshape(n, k)\n"
        "    b = rng.standard_normal(n).astype(np.float32)\n"
        "    check(run_prefill(s, x, w, ffm.STB_BF16, b), x, w, oracle.BF16, b)\n"
        "s.close()\n"
        "print('ok')\n")
    env = dict(os.environ, STB_GEMM_PAIR="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-2000:] + r.stderr[-4000:]
