"""Shared test set-up.

Markers: ``gpu`` tests need a B200 and the built CUDA library; everything else
runs on the CPU (the oracle against the reference's golden vectors and its
compiled code, the C ABI surface, host-side logic).

Tolerance: bit-exact for data movement, dequantisation,
rel_shift and argmax; |a - b| <= max(2e-6, 1e-5 |b|) for the floating-point
reductions and transcendental ops (LayerNorm, softmax, Swish, GLU, tanh).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "parakeet-unified-en-0.6b-c_b200")
for p in (os.path.join(ROOT, "oracle"), os.path.join(PKG, "python"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

ATOL = 2e-6
RTOL = 1e-5
GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_vectors.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built library")


def close_mask(a, b, atol=ATOL, rtol=RTOL):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    both_nan = np.isnan(a) & np.isnan(b)
    return both_nan | (np.abs(a - b) <= np.maximum(atol, rtol * np.abs(b)))


def assert_close(a, b, what="", atol=ATOL, rtol=RTOL):
    a = np.asarray(a)
    b = np.asarray(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    ok = close_mask(a, b, atol, rtol)
    if not ok.all():
        idx = np.argwhere(~ok)[0]
        d = np.abs(a.astype(np.float64) - b.astype(np.float64))
        raise AssertionError(
            f"{what}: {int((~ok).sum())}/{ok.size} outside tolerance; first at {tuple(idx)}: "
            f"{a[tuple(idx)]!r} vs {b[tuple(idx)]!r}; max |diff| {np.nanmax(d):.3e}")


def assert_bitexact(a, b, what=""):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if a.dtype == np.float32:
        av, bv = a.view(np.uint32), b.view(np.uint32)
        # NaN payloads are not portable (x86 propagates the input NaN, the GPU
        # returns the canonical one): any NaN matches any NaN.
        neq = (av != bv) & ~(np.isnan(a) & np.isnan(b))
    else:
        neq = a != b
    if neq.any():
        idx = np.argwhere(neq)[0]
        raise AssertionError(f"{what}: {int(neq.sum())}/{a.size} elements differ; first at "
                             f"{tuple(idx)}: {a[tuple(idx)]!r} vs {b[tuple(idx)]!r}")


@pytest.fixture(scope="session")
def oracle():
    import pyoracle
    if not os.path.exists(pyoracle.LIB_ORACLE):
        pyoracle.build()
    return pyoracle.Oracle()


@pytest.fixture(scope="session")
def reference():
    import pyoracle
    if not pyoracle.ref_available():
        pytest.skip("oracle/_ref/libpkref.so not built (reference tree absent)")
    return pyoracle.Reference()


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(autouse=True)
def _release_device_arrays():
    """Device arrays a test created live until the test ends."""
    yield
    try:
        import gpuhelp
        if gpuhelp.ALIVE:
            import torch
            torch.cuda.synchronize()
            gpuhelp.ALIVE.clear()
    except ImportError:
        pass


@pytest.fixture(autouse=True)
def _no_wait_timeouts(request):
    """After every GPU test: no bounded device wait (bulk-copy kernels) ran out."""
    yield
    if request.node.get_closest_marker("gpu") is None or "cuda" not in request.fixturenames:
        return
    import ctypes as C
    import pkcuda
    n = C.c_uint(0)
    pkcuda.call("pkcu_wait_timeouts", C.byref(n), 1)
    assert n.value == 0, f"{n.value} device wait(s) ran out"


@pytest.fixture(scope="session")
def cuda():
    """The CUDA library and torch on cuda:0 (gpu tests only)."""
    import torch
    import pkcuda
    if not torch.cuda.is_available():
        pytest.fail("gpu test without a CUDA device")
    pkcuda.lib()
    torch.cuda.set_device(0)
    return pkcuda
