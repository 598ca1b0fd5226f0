import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_oracle, load_package  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")


@pytest.fixture(scope="session")
def qq3():
    return load_package()


@pytest.fixture(scope="session")
def orc():
    return load_oracle()


@pytest.fixture(scope="session")
def torch():
    import torch as t

    assert t.cuda.is_available()
    return t


@pytest.fixture(scope="session")
def gpu_ctx(qq3):
    qq3.build.build_all()
    ctx = qq3.runtime.Context(int(os.environ.get("QQ3_TEST_DEVICE", "0")))
    yield ctx
    ctx.close()


def rel_err(got, want):
    """max |got - want| / max |want| (the 1e-2 'max relative error' of the parity bar)."""
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    den = max(float(np.abs(want).max()), 1e-30)
    return float(np.abs(got - want).max()) / den
