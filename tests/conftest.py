"""Shared test configuration.

Tests marked ``gpu`` need a B200 (sm_100a) and the built libpfrt_cuda.so; the
rest run on any machine (oracle pinning, host-side checks, the C ABI's symbol
table, multi-process host logic over gloo)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def ctx():
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    from pyflamert_b200 import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = np.load(os.path.join(ROOT, "tests", "golden", "golden_ref.npz"))
    return {k[:-3]: d[k] for k in d.files if k.endswith("__y")}, \
           {k[:-5]: bytes(d[k]).decode() for k in d.files if k.endswith("__sha")}
