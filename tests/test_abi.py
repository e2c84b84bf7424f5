"""The C-ABI library loads here (no GPU) and exports every entry point include/stb200.h declares;
host-side validation rejects bad requests before any native call."""
import os
import re

import pytest

from scalatorch import ffm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "stb200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(stb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("stb_session_create", "stb_upload", "stb_linear", "stb_linear_prefill", "stb_download",
                     "stb_llama_create", "stb_llama_generate", "stb_allreduce_sum_f32", "stb_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ffm.library()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert missing == []
    assert lib.stb_version() >= 100


def test_invalid_requests_rejected_before_native_calls():
    with pytest.raises(ffm.IllegalArgumentException):
        ffm.B200Session(-1, 1 << 20)
    with pytest.raises(ffm.IllegalArgumentException):
        ffm.require(False, "x")


def test_error_text_of_a_failed_call_is_reported():
    # stb_session_stream on a null session fails natively with STATE; no device is touched.
    with pytest.raises(ffm.IllegalStateException) as e:
        ffm.call("stb_sync", None)
    assert "session is null" in str(e.value)
