"""GPU: the drop-in host API (the prototypes of csrc/parakeet.h:231-262) with
host buffers, against the reference's own compiled functions and the
restatement."""
import numpy as np
import pytest

from conftest import assert_bitexact, assert_close

pytestmark = pytest.mark.gpu


def p(a):
    return a.ctypes.data


def test_dropin_layer_norm(cuda, oracle):
    L = cuda.lib()
    r = np.random.default_rng(1)
    for R, Dd in ((375, 1024), (1, 37), (3, 1024)):
        x = r.standard_normal((R, Dd)).astype(np.float32)
        g = (1 + 0.1 * r.standard_normal(Dd)).astype(np.float32)
        b = (0.1 * r.standard_normal(Dd)).astype(np.float32)
        out = np.empty_like(x)
        L.pk_layer_norm_rows(p(x), p(g), p(b), p(out), R, Dd)
        assert L.pk_cuda_status() == 0
        assert_close(out, oracle.layer_norm_rows(x, g, b), "rows")
        one = np.empty(Dd, np.float32)
        L.pk_layer_norm(p(x[0]), p(g), p(b), p(one), Dd)
        assert_close(one, out[0], "single")
        y = x.copy()
        L.pk_layer_norm_rows_inplace(p(y), p(g), p(b), R, Dd)
        assert_close(y, out, "inplace")


def test_dropin_vs_reference(cuda, oracle, reference):
    L = cuda.lib()
    r = np.random.default_rng(2)
    s = (3 * r.standard_normal((3000, 375))).astype(np.float32)
    y = s.copy()
    L.pk_softmax_rows(p(y), 3000, 375)
    assert_close(y, reference.softmax_rows(s), "softmax_rows")
    row = s[0].copy()
    L.pk_softmax(p(row), 375)
    assert_close(row, y[0], "softmax")
    h = (4 * r.standard_normal(375 * 4096 + 3)).astype(np.float32)
    hh = h.copy()
    L.pk_swish(p(hh), h.size)
    assert_close(hh, reference.swish(h), "swish")
    hr = h.copy()
    L.pk_relu(p(hr), h.size)
    assert_bitexact(hr, reference.relu(h), "relu")
    bias = r.standard_normal(4099).astype(np.float32)
    xb = r.standard_normal(4099).astype(np.float32)
    xx = xb.copy()
    L.pk_bias_add(p(xx), p(bias), 4099)
    assert_bitexact(xx, xb + bias, "bias")
    xc = r.standard_normal((1024, 375)).astype(np.float32)
    w = (0.3 * r.standard_normal((1024, 9))).astype(np.float32)
    bc = (0.1 * r.standard_normal(1024)).astype(np.float32)
    out = np.empty_like(xc)
    L.pk_depthwise_conv1d(p(xc), p(w), p(bc), p(out), 1024, 375, 9)
    assert_close(out, reference.depthwise_conv1d(xc, w, bc), "dwconv vs reference")
    assert_bitexact(out, oracle.depthwise_conv1d(xc, w, bc), "dwconv vs oracle")
    L.pk_depthwise_conv1d(p(xc), p(w), None, p(out), 1024, 375, 9)
    assert_bitexact(out, oracle.depthwise_conv1d(xc, w, None), "dwconv no bias")
    assert L.pk_cuda_status() == 0


def test_dropin_reports_errors(cuda):
    L = cuda.lib()
    L.pk_swish(None, 8)
    assert L.pk_cuda_status() == 1
    x = np.ones(8, np.float32)
    L.pk_swish(p(x), 8)
    assert L.pk_cuda_status() == 0
    L.pk_depthwise_conv1d(p(x), p(x), None, p(x), 1, 8, 500)   # K above the limit
    assert L.pk_cuda_status() == 1
    assert b"K must be" in L.pkcu_last_error()
