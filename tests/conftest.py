import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import __graft_entry__ as ge  # noqa: E402

PKG = ge.load_package()
ORACLE = ge.load_oracle()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    return PKG


@pytest.fixture(scope="session")
def oracle():
    ORACLE.build()
    return ORACLE


@pytest.fixture(scope="session")
def ctx():
    from decision_js_b200._lib import Context
    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def dev():
    import torch
    return torch.device("cuda", 0)


def to_dev(a, dev):
    """numpy -> torch on the GPU (float16 kept as raw 16-bit words)."""
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        a = a.view(np.int16)
    elif a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(dev)


def f16_of(t):
    """torch int16 / float16 tensor -> numpy float32 of its f16 values."""
    return t.detach().cpu().numpy().view(np.float16).astype(np.float32)


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))
