import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs at least two CUDA devices")


@pytest.fixture(autouse=True)
def _device_env(request, monkeypatch):
    """CPU tests run on CPU/gloo; GPU tests pick cuda and the default backend."""
    if request.node.get_closest_marker("gpu") is None:
        monkeypatch.setenv("MINISPEED_DEVICE", "cpu")
        monkeypatch.setenv("MINISPEED_BACKEND", "gloo")
    else:
        import torch

        if not torch.cuda.is_available():
            pytest.skip("CUDA device required")
        monkeypatch.setenv("MINISPEED_DEVICE", "cuda:0")
        monkeypatch.delenv("MINISPEED_BACKEND", raising=False)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
