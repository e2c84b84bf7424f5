"""Failure detection without a GPU fault: a device-side wait that nothing satisfies expires within
its limit, records its code in the session's error word, and the context stays usable."""
import ctypes

import numpy as np
import pytest

import oracle
from scalatorch import ffm

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives():
    with ffm.B200Session(0, 1 << 28) as s:
        lib = ffm.library()
        lib.stb_check_bounded_wait.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        code = ctypes.c_int(-1)
        ffm.call("stb_check_bounded_wait", s.handle, 50_000_000, ctypes.byref(code))  # 50 ms
        assert code.value == 99
        s.sync()  # the error word was cleared: no stale failure is reported
        x = np.ones((1, 16), np.float32)
        w = oracle.round_bf16(np.full((4, 16), 0.5, np.float32))
        xd, wd = s.upload(x), s.upload_weight(w, ffm.STB_BF16)
        y = s.download(s.linear(xd, wd))
        assert y.tolist() == [[8.0] * 4]
        with pytest.raises(ffm.IllegalArgumentException):
            ffm.call("stb_check_bounded_wait", s.handle, 0, ctypes.byref(code))
