"""Shared test set-up.

Markers: ``gpu`` tests need a B200 and call the CUDA library through its C
ABI; everything else runs on the CPU (oracle, host logic, ABI symbols).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("llama3.go_b200", "oracle", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libl3g.so")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle


_models = {}


def synthetic_model(name, seed=0):
    """Cached synthetic model tensors for a config name."""
    import synthetic
    key = (name, seed)
    if key not in _models:
        _models[key] = synthetic.make_model(synthetic.CONFIGS[name], seed=seed)
    return synthetic.CONFIGS[name], _models[key]


@pytest.fixture(scope="session")
def gpu_lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import build
    build.build(quiet=True)
    import l3g
    l3g.lib()
    return l3g
