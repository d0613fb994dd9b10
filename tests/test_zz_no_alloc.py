"""GPU: pk_softmax_rows_noalloc, the softmax entry point for callers that
cannot let the library allocate device memory -- a real-time callback that
must not wait on cudaMalloc, or a process whose device memory is all handed
to its own pool in advance. It stages rows in a fixed static device array
instead of a cudaMalloc'd workspace.

Checked through the C ABI on two calls in a row (different shapes, so the
second call runs over what the first left in the shared array): bit for bit
against the allocating drop-in pk_softmax_rows, and within the softmax
tolerance against the reference's own pk_softmax_rows (csrc/tensor_ops.c:346)
built from its source. Also the size limit and the empty call. This file is collected
last so that a run stopping at its first failure has run everything else; it
also passes on its own in a fresh process."""
import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu

MAX_FLOATS = 4 << 20


def _rows(seed, shape):
    return (3 * np.random.default_rng(seed).standard_normal(shape)).astype(np.float32)


def test_noalloc_matches_allocating_dropin_twice(cuda, reference):
    L = cuda.lib()
    for seed, shape in ((1, (3000, 375)), (2, (256, 33))):   # second call: smaller, stale tail
        x = _rows(seed, shape)
        want = x.copy()
        L.pk_softmax_rows(want.ctypes.data, shape[0], shape[1])
        assert L.pk_cuda_status() == 0
        got = x.copy()
        assert L.pk_softmax_rows_noalloc(got.ctypes.data, shape[0], shape[1]) == 0
        assert_close(got, reference.softmax_rows(x), f"noalloc vs the reference {shape}")
        assert_close(got, want, f"noalloc vs drop-in {shape}")
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_noalloc_empty_call(cuda):
    L = cuda.lib()
    assert L.pk_softmax_rows_noalloc(None, 0, 375) == 0
    assert L.pk_softmax_rows_noalloc(None, 12, 0) == 0
    assert L.pk_softmax_rows_noalloc(None, 12, 375) == 1     # rows to do but no x
    assert L.pk_softmax_rows_noalloc(None, -1, 375) == 1


def test_noalloc_rejects_oversize(cuda):
    L = cuda.lib()
    x = np.zeros(8, np.float32)
    assert L.pk_softmax_rows_noalloc(x.ctypes.data, MAX_FLOATS // 1024 + 1, 1024) == 1
    assert b"static buffer" in L.pkcu_last_error()
    # the largest allowed size still works
    big = _rows(3, (MAX_FLOATS // 1024, 1024))
    want = big.copy()
    L.pk_softmax_rows(want.ctypes.data, big.shape[0], big.shape[1])
    assert L.pk_softmax_rows_noalloc(big.ctypes.data, big.shape[0], big.shape[1]) == 0
    assert np.array_equal(big.view(np.uint32), want.view(np.uint32))
