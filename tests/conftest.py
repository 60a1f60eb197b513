import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from redukt_b200 import rbin  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: full-size Mamba-130M cases")


def logsoftmax64(logits: np.ndarray) -> np.ndarray:
    l = logits.astype(np.float64)
    m = l.max(axis=-1, keepdims=True)
    return l - m - np.log(np.exp(l - m).sum(axis=-1, keepdims=True))


def max_dlogp(a: np.ndarray, b: np.ndarray) -> float:
    return float(np.max(np.abs(logsoftmax64(a) - logsoftmax64(b))))


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("REDUKT_B200_MODEL_CACHE")
    if d:
        os.makedirs(d, exist_ok=True)
        return d
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def ref_test_rbin(model_dir):
    """The reference's own unit-test model (synthetic_model(64, 2, 1200))."""
    return rbin.ensure_model(os.path.join(model_dir, "reftest.rbin"), rbin.REFERENCE_TEST_DIMS, kind="reference_test")


@pytest.fixture(scope="session")
def small_gauss_rbin(model_dir):
    dims = rbin.MambaDims(vocab=2000, d_model=128, n_layer=3)
    return rbin.ensure_model(os.path.join(model_dir, "gauss_small.rbin"), dims, kind="gaussian", seed=12345)


@pytest.fixture(scope="session")
def mamba130m_rbin(model_dir):
    return rbin.ensure_model(os.path.join(model_dir, "mamba130m.rbin"), rbin.MAMBA_130M, kind="gaussian")


_SHARED_BACKEND = {}


def shared_backend(path: str):
    """The plugin is a process-global singleton: every GPU test module goes through this one cache,
    so a module never holds a handle to a model another module has replaced."""
    from redukt_b200.plugin import PluginBackend
    b = _SHARED_BACKEND.get("b")
    if b is not None and _SHARED_BACKEND.get("path") == path and not b._closed:
        return b
    if b is not None and not b._closed:
        b.close()
    b = PluginBackend(path)
    _SHARED_BACKEND.update(b=b, path=path)
    return b


def q8(path: str, per_row: bool = False) -> str:
    flags = rbin.FLAG_Q8 | (rbin.FLAG_Q8_PER_ROW if per_row else 0)
    suffix = ".q8row.rbin" if per_row else ".q8.rbin"
    return rbin.with_flags(path, path[:-5] + suffix, flags)
