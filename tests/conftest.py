"""Shared fixtures. `gpu` tests need a B200; everything else runs on the CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "webgpu-gemma_b200"))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.build()
    return oracle


_MODELS = {}


def synthetic(shape_name: str, seed: int):
    """(config, tensors) of a seeded synthetic model, cached per session."""
    key = (shape_name, seed)
    if key not in _MODELS:
        from gemma_b200 import synth
        shape = synth.SHAPES[shape_name]
        _MODELS[key] = (shape.config(), synth.make_tensors(shape, seed))
    return _MODELS[key]


@pytest.fixture(scope="session")
def tiny_model():
    return synthetic("tiny", 7)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
