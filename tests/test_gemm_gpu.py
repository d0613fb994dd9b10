"""GPU parity of the GEMMs with fused epilogues (pkcu_gemm_bias_swish,
pkcu_gemm_bias_residual) against the reference's own CPU path: pk_wmatmul
with an fp32 Weight (its register-blocked sgemm, csrc/blas.c), the per-row
pk_bias_add, then pk_swish (csrc/encoder.c:193-196) or the residual add
(x + 0.5 out, :198-216; x + out, :418-434).

Tolerance: two fp32 GEMMs that sum in different orders differ by up to a few
units of K * 2^-24 * sum_k |a_ik| |w_kj|, so each entry must satisfy
|gpu - ref| <= 1e-5 * (|A| |W|)_ij + 2e-6 (plus 1e-6 |x| for the residual
add). The tensor-core path keeps fp32 accuracy (three bf16 parts per operand,
nine MMAs per product); a bf16 or tf32 GEMM would miss this bound by orders of
magnitude.
"""
import numpy as np
import pytest

from gpuhelp import dev, empty, host

pytestmark = pytest.mark.gpu


def bound(A, W):
    return 1e-5 * (np.abs(A).astype(np.float64) @ np.abs(W).astype(np.float64)) + 2e-6


def check(got, want, tol, what):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    bad = err > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{bad.size} outside the GEMM bound; max err "
                           f"{err.max():.3e}, max err / bound {(err / tol).max():.3f}")


def inputs(rng, M, N, K):
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    return A, W, b


@pytest.mark.parametrize("M,N,K", [(1, 4096, 1024), (37, 4096, 1024), (416, 4096, 1024),
                                   (300, 256, 64)])
def test_gemm_bias_swish(cuda, reference, M, N, K):
    A, W, b = inputs(np.random.default_rng(M + N + K), M, N, K)
    D = empty(M * N)
    cuda.call("pkcu_gemm_bias_swish", dev(A).data_ptr(), dev(W).data_ptr(), dev(b).data_ptr(),
              D.data_ptr(), M, N, K, None)
    check(host(D).reshape(M, N), reference.ff_linear1(A, W, b), bound(A, W), "Swish(A W + b)")


@pytest.mark.parametrize("M,N,K,scale", [(1, 1024, 4096, 0.5), (37, 1024, 4096, 0.5),
                                         (416, 1024, 1024, 1.0), (129, 640, 1024, 1.0)])
def test_gemm_bias_residual(cuda, reference, M, N, K, scale):
    rng = np.random.default_rng(7 * M + N + K)
    A, W, b = inputs(rng, M, N, K)
    x = rng.standard_normal((M, N)).astype(np.float32)
    X = dev(x)
    cuda.call("pkcu_gemm_bias_residual", dev(A).data_ptr(), dev(W).data_ptr(), dev(b).data_ptr(),
              X.data_ptr(), scale, M, N, K, None)
    want = reference.linear_residual(x, A, W, b, scale)
    check(host(X).reshape(M, N), want, scale * bound(A, W) + 1e-6 * np.abs(x), "X + s (A W + b)")


def test_gemm_matches_unfused_gpu_path(cuda):
    """The fused Swish GEMM against torch's fp32 GEMM (TF32 off) followed by
    this library's bias + Swish kernel: the two differ only by GEMM rounding."""
    import torch
    M, N, K = 512, 4096, 1024
    A, W, b = inputs(np.random.default_rng(3), M, N, K)
    Ad, Wd, bd = dev(A), dev(W), dev(b)
    D = empty(M * N)
    cuda.call("pkcu_gemm_bias_swish", Ad.data_ptr(), Wd.data_ptr(), bd.data_ptr(), D.data_ptr(),
              M, N, K, None)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        H = (Ad.view(M, K) @ Wd.view(K, N)).contiguous()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    cuda.call("pkcu_bias_swish_rows", H.data_ptr(), bd.data_ptr(), H.data_ptr(), M, N, None)
    check(host(D).reshape(M, N), host(H), bound(A, W), "fused vs unfused")
