"""The split-operand kernels (csrc/k_split.cu) behind the encoder model's
fp32-accurate bf16 GEMMs, bit-exact against the numpy restatement of the
three-part split (oracle/pyoracle.py: split3_bf16), through their C entry
points: activation rows to [a0 | a1 | a2], weights to the stack [w2; w1; w0],
channel-first inputs to [x2; x1; x0] at a padded pitch, and the copy that
drops the pad columns of a product."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import pyoracle as po
from conftest import assert_bitexact
from gpuhelp import dev

pytestmark = pytest.mark.gpu

VP, I, LL = C.c_void_p, C.c_int, C.c_longlong


def _lib(cuda):
    L = cuda.lib()
    L.pk_split_rows_bf16x3.argtypes = [VP, VP, LL, I, VP]
    L.pk_split_stack_bf16x3.argtypes = [VP, VP, I, I, VP]
    L.pk_split_cols_bf16x3.argtypes = [VP, VP, LL, I, I, I, VP]
    L.pk_depad_rows.argtypes = [VP, VP, LL, I, I, VP]
    return L


def _values(rng, shape):
    """Normal values spread over many binades (every part then matters)."""
    n = int(np.prod(shape))
    return (rng.standard_normal(n) * np.exp(rng.uniform(-12, 12, n))).astype(np.float32).reshape(shape)


def _parts_u16(t, shape):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint16).reshape(shape)


def test_split_rows_bitexact(cuda):
    import torch
    L = _lib(cuda)
    M, K = 37, 1024
    a = _values(np.random.default_rng(51), (M, K))
    out = torch.empty(M * 3 * K, dtype=torch.int16, device="cuda")
    assert L.pk_split_rows_bf16x3(dev(a).data_ptr(), out.data_ptr(), M, K, None) == 0
    got = _parts_u16(out, (M, 3, K))
    for i, p in enumerate(po.split3_bf16(a)):
        assert_bitexact(got[:, i, :], p, f"part {i}")


def test_split_stack_bitexact(cuda):
    import torch
    L = _lib(cuda)
    K, N = 64, 96
    w = _values(np.random.default_rng(52), (K, N))
    out = torch.empty(3 * K * N, dtype=torch.int16, device="cuda")
    assert L.pk_split_stack_bf16x3(dev(w).data_ptr(), out.data_ptr(), K, N, None) == 0
    got = _parts_u16(out, (3, K, N))
    p0, p1, p2 = po.split3_bf16(w)
    for i, p in enumerate((p2, p1, p0)):   # the stack [w2; w1; w0]
        assert_bitexact(got[i], p, f"stack part {i}")


def test_split_cols_and_depad_bitexact(cuda):
    import torch
    L = _lib(cuda)
    items, K, T = 3, 40, 13
    Tp = (T + 7) & ~7
    x = _values(np.random.default_rng(53), (items, K, T))
    out = torch.empty(items * 3 * K * Tp, dtype=torch.int16, device="cuda")
    assert L.pk_split_cols_bf16x3(dev(x).data_ptr(), out.data_ptr(), items, K, T, Tp,
                                  None) == 0
    got = _parts_u16(out, (items, 3, K, Tp))[..., :T]   # pad columns are unspecified
    p0, p1, p2 = po.split3_bf16(x)
    for i, p in enumerate((p2, p1, p0)):   # [x2; x1; x0] per item
        assert_bitexact(got[:, i], p, f"column part {i}")
    padded = _values(np.random.default_rng(54), (7, Tp))
    dst = torch.empty(7 * T, dtype=torch.float32, device="cuda")
    assert L.pk_depad_rows(dev(padded).data_ptr(), dst.data_ptr(), 7, T, Tp, None) == 0
    torch.cuda.synchronize()
    assert_bitexact(dst.cpu().numpy().reshape(7, T), padded[:, :T], "depad")


def test_split_entry_points_reject_bad_arguments(cuda):
    L = _lib(cuda)
    ERR_ARG = 1
    assert L.pk_split_rows_bf16x3(None, None, 4, 1024, None) == ERR_ARG
    assert L.pk_split_stack_bf16x3(None, None, 4, 8, None) == ERR_ARG
    assert L.pk_split_cols_bf16x3(None, None, 1, 4, 5, 4, None) == ERR_ARG   # Tp < T as well
    assert L.pk_depad_rows(None, None, 1, 5, 8, None) == ERR_ARG
