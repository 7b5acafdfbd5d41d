import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA kernels)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc
    orc.build()
    return orc


@pytest.fixture(scope="session")
def ob():
    return importlib.import_module("onnx-rs_b200")


@pytest.fixture(scope="session")
def handle(ob):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    h = ob.Handle(0, precision="3xtf32")
    yield h
    h.close()


def compare(actual, expected, rtol, atol):
    """The reference's comparison rule (src/tools/comparison.rs:1298-1321): an element
    passes if |a-b| <= atol or |a-b|/|b| <= rtol (relative only when |b| > 1e-6).
    Returns (n_fail, max_abs, max_rel)."""
    a = np.asarray(actual, np.float64)
    b = np.asarray(expected, np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    d = np.abs(a - b)
    rel = np.where(np.abs(b) > 1e-6, d / np.maximum(np.abs(b), 1e-30), np.inf)
    ok = (d <= atol) | (rel <= rtol)
    ok &= ~(np.isnan(a) ^ np.isnan(b))
    finite_rel = rel[np.isfinite(rel)]
    return int((~ok).sum()), float(d.max() if d.size else 0.0), float(finite_rel.max() if finite_rel.size else 0.0)


def assert_close(actual, expected, rtol, atol, what=""):
    n, ma, mr = compare(actual, expected, rtol, atol)
    assert n == 0, f"{what}: {n} elements outside rtol={rtol}/atol={atol} (max abs {ma:.3g}, max rel {mr:.3g})"


@pytest.fixture(scope="session")
def close():
    return assert_close
