"""Test setup: import paths for the oracle (checker) and the scalatorch mirror, the gpu marker."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "scala-torch_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs on the GPU box with -m gpu)")


_gpu = None


def gpu_available() -> bool:
    global _gpu
    if _gpu is None:
        try:
            import torch
            _gpu = bool(torch.cuda.is_available())
        except Exception:
            _gpu = False
    return _gpu


def pytest_collection_modifyitems(config, items):
    for item in items:
        if "gpu" in item.keywords and not gpu_available():
            item.add_marker(pytest.mark.skip(reason="no GPU visible in this process"))


@pytest.fixture(scope="session")
def session():
    from scalatorch.ffm import B200Session
    s = B200Session(0, 100 << 30)
    yield s
    s.close()
