"""Shared test setup: paths, the `gpu` marker, synthetic models.

CPU tests (`-m "not gpu"`) cover the oracle against golden vectors, host logic and the C ABI
surface. GPU tests (`-m gpu`) compare the CUDA library with the oracle through the C ABI.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "gsv.cpp_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

MODEL_CACHE = os.environ.get("GSVCU_MODEL_CACHE", "/tmp/gsvcu_models")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def model_small():
    """2-layer synthetic Q8_0 model (fast oracle)."""
    import gsv_synth
    return gsv_synth.cached_model(MODEL_CACHE, seed=11, n_layer=2)


@pytest.fixture(scope="session")
def model_full():
    """Full 24-layer synthetic Q8_0 model (BASELINE dims)."""
    import gsv_synth
    return gsv_synth.cached_model(MODEL_CACHE, seed=0, n_layer=24)


@pytest.fixture(scope="session")
def model_f32_small():
    """2-layer model whose attention/FFN matrices are F32 (no activation quantization)."""
    import gsv_synth
    return gsv_synth.cached_model(MODEL_CACHE, seed=5, n_layer=2, mat_type="f32")


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-30))
