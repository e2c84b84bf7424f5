"""stb_linear_prefill_static: the prefill Linear for callers that may not allocate device memory.

Such callers (a host framework that owns every device allocation through its own allocator or
budget, a serving loop that forbids allocation after warm-up) get the same tensor-core product with
its scratch in a fixed 16 MiB array compiled into the library.  This file is collected last so a
run that stops at the first failure has already run every other test; it also passes alone in a
fresh process.
"""
import ctypes

import numpy as np
import pytest

import oracle
from scalatorch import ffm

pytestmark = pytest.mark.gpu
TOL = 1e-4  # the elementwise tolerance of the prefill tests (activations rounded to BF16)


def _static(stream, x, w, dtype, bias, y, m, n, k):
    lib = ffm.library()
    code = lib.stb_linear_prefill_static(ctypes.c_void_p(stream), x, w, dtype, bias, y, m, n, k)
    if code != 0:
        raise ffm.IllegalStateException("stb_linear_prefill_static", code, lib.stb_last_error().decode())


def test_static_scratch_matches_the_allocating_entry_point_twice():
    with ffm.B200Session(0, 1 << 30) as s:
        rng = np.random.default_rng(31)
        shapes = [(256, 512, 576), (300, 1000, 200)]
        for m, n, k in shapes:
            x = s.upload(rng.standard_normal((m, k)).astype(np.float32))
            w = s.upload_weight(oracle.normal_bf16(n * k, seed=m, stream=k, std=0.02).reshape(n, k), ffm.STB_BF16)
            ref = s.linear(x, w, prefill=True)
            want = s.download(ref)
            got = []
            for _ in range(2):  # two calls in a row share (and reuse) the static array
                y = s.allocate((m, n))
                _static(s.stream, x.address, w.address, ffm.STB_BF16, 0, y.address, m, n, k)
                got.append(s.download(y))
                s.release(y)
            for g in got:
                err = np.abs(g.astype(np.float64) - want)
                assert np.all(err <= TOL * (1 + np.abs(want))), err.max()
            for t in (x, w, ref):
                s.release(t)


def test_static_scratch_rejects_requests_beyond_its_limit():
    with ffm.B200Session(0, 1 << 30) as s:
        lib = ffm.library()
        # 4096 x 4096 activations = 16,777,216 > 8,388,608: rejected before any device work
        code = lib.stb_linear_prefill_static(ctypes.c_void_p(s.stream), 16, 16, ffm.STB_BF16, 0, 16, 4096, 8, 4096)
        assert code == 1
        assert "static scratch limit" in lib.stb_last_error().decode()
