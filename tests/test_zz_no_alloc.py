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
TOL = 2e-3  # the prefill tolerance against the oracle: normwise per row (activations rounded to half)
LIMIT = 8 << 20  # M * K activations the array holds


def _static(stream, x, w, dtype, bias, y, m, n, k):
    lib = ffm.library()
    code = lib.stb_linear_prefill_static(ctypes.c_void_p(stream), x, w, dtype, bias, y, m, n, k)
    if code != 0:
        raise ffm.IllegalStateException("stb_linear_prefill_static", code, lib.stb_last_error().decode())


def _weight(n, k, dtype, seed):
    wf = oracle.normal_f32(n * k, seed, 7, 0.02).reshape(n, k)
    return oracle.round_bf16(wf) if dtype == ffm.STB_BF16 else oracle.round_f16(wf)


def _rowwise(got, want):
    err = np.linalg.norm(got.astype(np.float64) - want, axis=1)
    assert np.all(err <= TOL * np.linalg.norm(want, axis=1)), err.max()


# (M, N, K, weight type): ragged M and N, both half types, and M * K exactly at the limit
CASES = [(256, 512, 576, ffm.STB_BF16), (300, 1000, 200, ffm.STB_BF16), (256, 384, 512, ffm.STB_F16),
         (2048, 256, LIMIT // 2048, ffm.STB_BF16)]


def test_static_scratch_matches_the_allocating_entry_point_twice():
    """Two calls in a row on each case give the allocating entry point's output bit for bit (same
    rounding, same kernels) and the oracle's within the prefill tolerance; after a warm-up call of
    each weight type, the device's free memory does not change over the later calls."""
    import torch
    with ffm.B200Session(0, 1 << 30) as s:
        rng = np.random.default_rng(31)
        data = []
        for m, n, k, dt in CASES:
            x = rng.standard_normal((m, k)).astype(np.float32)
            w = _weight(n, k, dt, m)
            xd, wd = s.upload(x), s.upload_weight(w, dt)
            ref = s.linear(xd, wd, prefill=True)
            data.append((x, w, xd, wd, s.download(ref), s.allocate((m, n))))
            s.release(ref)
        s.sync()
        # warm-up: the first call per weight type loads the module and looks up the array's address
        for i in (0, 2):
            m, n, k, dt = CASES[i]
            _static(s.stream, data[i][2].address, data[i][3].address, dt, 0, data[i][5].address, m, n, k)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info(0)[0]
        for (m, n, k, dt), (x, w, xd, wd, want, y) in zip(CASES, data):
            odt = oracle.BF16 if dt == ffm.STB_BF16 else oracle.F16
            xr = oracle.widen(oracle.round_bf16(x) if dt == ffm.STB_BF16 else oracle.round_f16(x), odt)
            expect = oracle.linear(xr, w, odt).astype(np.float64)
            for _ in range(2):  # two calls in a row share (and reuse) the static array
                s.sync()
                _static(s.stream, xd.address, wd.address, dt, 0, y.address, m, n, k)
                got = s.download(y)
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (m, n, k)
                _rowwise(got, expect)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info(0)[0] == free0, "the allocation-free entry point changed free device memory"
        for *_, xd, wd, _, y in data:
            for t in (xd, wd, y):
                s.release(t)


def test_static_scratch_rejects_requests_beyond_its_limit():
    with ffm.B200Session(0, 1 << 30) as s:
        lib = ffm.library()
        # 4096 x 4096 activations = 16,777,216 > 8,388,608: rejected before any device work
        code = lib.stb_linear_prefill_static(ctypes.c_void_p(s.stream), 16, 16, ffm.STB_BF16, 0, 16, 4096, 8, 4096)
        assert code == 1
        assert "static scratch limit" in lib.stb_last_error().decode()
        # one row past the limit: (LIMIT / 8 + 1) x 8 activations
        code = lib.stb_linear_prefill_static(ctypes.c_void_p(s.stream), 16, 16, ffm.STB_BF16, 0, 16, LIMIT // 8 + 1, 8, 8)
        assert code == 1
        assert "static scratch limit" in lib.stb_last_error().decode()
