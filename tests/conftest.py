"""pytest configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs on any machine (oracle pins, host logic, C-ABI exports);
``-m gpu`` needs an sm_100 GPU and the in-tree ``libs1c.so``.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libs1c.so")


@pytest.fixture(scope="session")
def cuda_lib():
    """The built library; on a GPU box a missing library is a failure, never a skip."""
    from sys1rust_b200 import build as b
    b.build()
    from sys1rust_b200.backend import lib
    return lib()


_BACKENDS = {}


def get_backend(name: str):
    """Session-cached backends keyed by config name ('small' or 'large') and weight seed."""
    if name in _BACKENDS:
        return _BACKENDS[name]
    from sys1rust_b200.backend import CudaBackend
    from sys1rust_b200.config import large_model, small_model
    from sys1rust_b200.weights import SyntheticWeights
    cfg_name, seed = name.split(":")
    cfg = small_model() if cfg_name == "small" else large_model()
    w = SyntheticWeights(cfg, seed=int(seed))
    be = CudaBackend.from_synthetic(cfg, w.tensors)
    _BACKENDS[name] = (cfg, w, be)
    return _BACKENDS[name]
