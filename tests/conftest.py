"""Shared test set-up: import paths, the `gpu` marker and small helpers.

Tests marked `gpu` need a B200 and the built library (colabfold-legacy-kernels_b200/build.py);
everything else runs on the CPU.
"""

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_SRC = REPO / "colabfold-legacy-kernels_b200" / "src"
for p in (str(REPO), str(PKG_SRC)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built sm_100a library")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (it is marked gpu)")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail("this test needs a compute capability 10.0 device, got %d.%d" % (major, minor))
    return torch.device("cuda", 0)


def assert_close_bf16(actual, expected, what, rtol=2e-2, atol=2e-2):
    """bf16/fp16 outputs and gradients: |a - e| <= atol + rtol * |e| elementwise."""
    import torch
    a = actual.double().cpu()
    e = expected.double().cpu()
    err = (a - e).abs()
    bound = atol + rtol * e.abs()
    bad = err > bound
    if bad.any():
        idx = bad.nonzero()[0].tolist()
        raise AssertionError(
            "%s: %d of %d elements outside atol=%g rtol=%g; worst |err|=%.4g; first bad at %s: "
            "got %.6g expected %.6g" % (what, int(bad.sum()), bad.numel(), atol, rtol,
                                        float(err.max()), idx, float(a[tuple(idx)]),
                                        float(e[tuple(idx)])))


def assert_close_f32(actual, expected, what, rel=1e-4):
    """f32 outputs (lse, dbias, dgamma, dW): |a - e| <= rel * (|e| + max|e|) elementwise, i.e. an
    absolute error bound of 1e-4 of the tensor's largest magnitude plus a relative one."""
    import torch
    a = actual.double().cpu()
    e = expected.double().cpu()
    scale = float(e.abs().max()) if e.numel() else 0.0
    err = (a - e).abs()
    bound = rel * (e.abs() + scale)
    bad = err > bound
    if bad.any():
        idx = bad.nonzero()[0].tolist()
        raise AssertionError(
            "%s: %d of %d elements outside rel=%g (max|e|=%.4g); worst |err|=%.4g; first bad at "
            "%s: got %.8g expected %.8g" % (what, int(bad.sum()), bad.numel(), rel, scale,
                                            float(err.max()), idx, float(a[tuple(idx)]),
                                            float(e[tuple(idx)])))
