import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# parity bar of BASELINE.json's north star: layer output within max-abs 2e-2 and cosine >= 0.9999
MAX_ABS_TOL = 2e-2
COS_TOL = 0.9999


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build
    build()
    return Oracle()


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def cosine(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    return float(a @ b / np.sqrt(max((a @ a) * (b @ b), 1e-300)))


def assert_close_layer(got, ref, what=""):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    err = float(np.abs(got - ref).max()) if got.size else 0.0
    cos = cosine(got, ref) if got.size and np.abs(ref).max() > 0 else 1.0
    assert err <= MAX_ABS_TOL, f"{what}: max abs err {err} > {MAX_ABS_TOL}"
    assert cos >= COS_TOL, f"{what}: cosine {cos} < {COS_TOL}"
    return err, cos
