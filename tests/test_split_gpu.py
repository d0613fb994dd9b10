"""The operand preparation of the library's tcgen05 GEMM, bit-exact against
the numpy restatement of the three-part split (oracle/pyoracle.py:
split3_bf16) through the C entry points: activation rows to [a0 | a1 | a2]
(k_split.cu); a [K, N] weight transposed to K-major planes [N, 3K], an int8
weight's q to [N, K] bf16 (k_tcgemm.cu); a pointwise weight's rows to
[N, 3K] with the GLU interleave; channel-first items to time-first parts."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import pyoracle as po
from conftest import assert_bitexact
from gpuhelp import dev

pytestmark = pytest.mark.gpu

VP, I, LL, F = C.c_void_p, C.c_int, C.c_longlong, C.c_float


def _lib(cuda):
    L = cuda.lib()
    L.pk_split_rows_bf16x3.argtypes = [VP, VP, LL, I, VP]
    L.pk_tc_prepare.argtypes = [VP, I, F, I, I, VP, C.POINTER(F), VP]
    L.pk_tc_prepare_rows.argtypes = [VP, I, I, I, VP, VP]
    L.pk_split_cf_t.argtypes = [VP, VP, I, VP, VP]
    return L


def _values(rng, shape):
    """Normal values spread over many binades (every part then matters)."""
    n = int(np.prod(shape))
    return (rng.standard_normal(n) * np.exp(rng.uniform(-12, 12, n))).astype(np.float32).reshape(shape)


def _u16(t, shape):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint16).reshape(shape)


def _empty16(n):
    import torch
    from gpuhelp import ALIVE
    t = torch.empty(n, dtype=torch.int16, device="cuda")
    ALIVE.append(t)
    return t


def _rows_parts(a):
    """[R, K] fp32 -> [R, 3K] bf16 bits, row = [a0 | a1 | a2]."""
    p0, p1, p2 = po.split3_bf16(a)
    return np.concatenate([p0, p1, p2], axis=-1)


def test_split_rows_bitexact(cuda):
    L = _lib(cuda)
    M, K = 37, 1024
    a = _values(np.random.default_rng(1), (M, K))
    out = _empty16(M * 3 * K)
    assert L.pk_split_rows_bf16x3(dev(a).data_ptr(), out.data_ptr(), M, K, None) == 0
    assert_bitexact(_u16(out, (M, 3 * K)), _rows_parts(a), "rows [a0 | a1 | a2]")


@pytest.mark.parametrize("K,N", [(1024, 4096), (4096, 1024), (64, 96)])
def test_prepare_fp32_weight_bitexact(cuda, K, N):
    L = _lib(cuda)
    w = _values(np.random.default_rng(K + N), (K, N))
    out = _empty16(N * 3 * K)
    alpha = F(0)
    assert L.pk_tc_prepare(dev(w).data_ptr(), 32, 0.0, K, N, out.data_ptr(), C.byref(alpha), None) == 0
    assert alpha.value == 1.0
    assert_bitexact(_u16(out, (N, 3 * K)), _rows_parts(np.ascontiguousarray(w.T)), "planes [N, 3K]")


def test_prepare_int8_weight_exact(cuda):
    L = _lib(cuda)
    K, N = 1024, 3072
    q = np.random.default_rng(2).integers(-127, 128, (K, N)).astype(np.int8)
    out = _empty16(N * K)
    alpha = F(0)
    assert L.pk_tc_prepare(dev(q).data_ptr(), 8, 0.004, K, N, out.data_ptr(), C.byref(alpha), None) == 0
    assert alpha.value == np.float32(0.004)
    want = po.split3_bf16(np.ascontiguousarray(q.T).astype(np.float32))
    assert_bitexact(_u16(out, (N, K)), want[0], "q as bf16 [N, K]")
    assert not want[1].any()   # q is exact in one bf16 part


@pytest.mark.parametrize("glu", [0, 1])
def test_prepare_pointwise_rows(cuda, glu):
    L = _lib(cuda)
    N, K = 2048, 1024
    w = _values(np.random.default_rng(3 + glu), (N, K))
    out = _empty16(N * 3 * K)
    assert L.pk_tc_prepare_rows(dev(w).data_ptr(), N, K, glu, out.data_ptr(), None) == 0
    src = np.arange(N)
    if glu:   # rows 64k .. 64k + 31: value channels 32k ..; the next 32: their gates
        n = np.arange(N)
        blk, r = n // 64, n % 64
        src = np.where(r < 32, blk * 32 + r, N // 2 + blk * 32 + r - 32)
    assert_bitexact(_u16(out, (N, 3 * K)), _rows_parts(w[src]), "pointwise planes")


def test_split_channel_first_items_to_time_first(cuda):
    L = _lib(cuda)
    Cc = 1024
    lengths = [375, 7, 416]
    rng = np.random.default_rng(4)
    xs = [_values(rng, (Cc, T)) for T in lengths]
    out = _empty16(sum(lengths) * 3 * Cc)
    with cuda.Seq(lengths) as seq:
        assert L.pk_split_cf_t(dev(np.concatenate([x.reshape(-1) for x in xs])).data_ptr(), out.data_ptr(),
                               Cc, seq.handle, None) == 0
        got = _u16(out, (sum(lengths), 3 * Cc))
    want = np.concatenate([_rows_parts(np.ascontiguousarray(x.T)) for x in xs])
    assert_bitexact(got, want, "time-first parts")


def test_split_entry_points_reject_bad_arguments(cuda):
    L = _lib(cuda)
    ERR_ARG = 1
    assert L.pk_split_rows_bf16x3(None, None, 4, 1024, None) == ERR_ARG
    assert L.pk_split_cf_t(None, None, 1024, None, None) == ERR_ARG
