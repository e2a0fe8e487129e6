"""pytest configuration: the `gpu` marker and import paths (repo root for rabbit_b200/oracle)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and librmoe.so")


@pytest.fixture(scope="session")
def cuda_ctx():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import rabbit_b200 as rb

    ctx = rb.Context(0)
    yield ctx
    ctx.close()
