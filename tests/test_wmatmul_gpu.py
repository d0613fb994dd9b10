"""GPU parity of the weight products on the library's own tcgen05 GEMM
(pkcu_weight_create + pkcu_wmatmul / _bias_swish / _bias_residual / _qkv)
against the reference's own CPU path, for the reference's three weight
storages (Weight, csrc/parakeet.h:52-57):

* float32 and int8 (per-tensor scale): the reference's pk_wmatmul
  (csrc/tensor_ops.c:50-61; cblas_sgemm_st / cblas_sgemm_qb with its
  dequantise-while-packing, csrc/blas.c:526-558, 759) on the same operands;
* GPTQ int4: pk_wmatmul on the fp32 weights the restatement's dequantisation
  gives (bit-exact to the format, extract_weights.py:589-594; the reference's
  AVX2 int4 unpack misreads nibbles, so its own int4 GEMM is not the oracle),
  for the reference's groups (32 along N) and config 5's (128 along K);
* the fused epilogues against pk_wmatmul followed by the reference's own
  pk_bias_add and pk_swish (csrc/encoder.c:193-196), the residual adds
  (:198-216, :418-434) and the QKV bias + head split + pos_bias_u/v
  (:313-356, the restatement's qkv_split_uv) on a ragged batch.

Tolerance: two fp32 GEMMs that sum in different orders differ by a few units
of K 2^-24 sum_k |a_ik| |w_kj|: every entry must satisfy
|gpu - ref| <= 1e-5 (|A| |W|)_ij + 2e-6."""
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
    return float((err / tol).max())


def work(cuda, M, K):
    return empty(int(cuda.lib().pkcu_wmatmul_work_bytes(M, K)) // 4 + 64)


def weights(kind, rng, K, N, oracle):
    """(device args for pkcu_weight_create, fp32 [K, N] values, int8 q or None, scale)."""
    if kind == "f32":
        W = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
        return dict(data=dev(W), bits=32), W, None, None
    if kind == "i8":
        q = rng.integers(-127, 128, (K, N)).astype(np.int8)
        s = np.float32(rng.uniform(1e-3, 1e-2))
        return dict(data=dev(q), bits=8, scale=float(s)), oracle.dequant_i8(q, s), q, s
    G, axis = {"i4_g32_n": (32, 1), "i4_g128_k": (128, 0)}[kind]
    packed = rng.integers(0, 256, (K, N // 2)).astype(np.uint8)
    ns = K * N // G
    scales = rng.uniform(1e-3, 2e-2, ns).astype(np.float32)
    W = oracle.dequant_i4(packed, scales, K, N, G, axis)
    return dict(data=dev(packed), bits=4, scales=dev(scales), group=G, axis=axis), W, None, None


def make_weight(cuda, args, K, N):
    return cuda.Weight(args.pop("data"), args.pop("bits"), K, N, **args)


# (8000, 640, 1024) takes the 128-wide tiles (640 columns pad to 768 in 256-wide ones)
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 1024, 1024), (300, 4096, 1024),
                                   (37, 1024, 4096), (1000, 3072, 1024), (8000, 640, 1024)])
@pytest.mark.parametrize("kind", ["f32", "i8", "i4_g32_n", "i4_g128_k"])
def test_wmatmul_matches_reference(cuda, reference, oracle, kind, M, N, K):
    if kind == "i4_g128_k" and K % 128:
        pytest.skip("groups of 128 along K need K % 128 == 0")
    rng = np.random.default_rng(M + N + K + len(kind))
    A = rng.standard_normal((M, K)).astype(np.float32)
    args, W, q, s = weights(kind, rng, K, N, oracle)
    want = reference.wmatmul(A, q, scale=s) if q is not None else reference.wmatmul(A, W)
    C = empty(M * N)
    with make_weight(cuda, args, K, N) as w:
        cuda.call("pkcu_wmatmul", dev(A).data_ptr(), w.handle, C.data_ptr(), M, 1.0, 0.0,
                  work(cuda, M, K).data_ptr(), None)
        got = host(C).reshape(M, N)
    check(got, want, bound(A, W), f"{kind} A W")


def test_wmatmul_alpha_beta(cuda, reference, oracle):
    """C = alpha A W + beta C, the reference's own alpha / beta semantics."""
    rng = np.random.default_rng(11)
    M, N, K = 200, 1024, 1024
    A = rng.standard_normal((M, K)).astype(np.float32)
    args, W, q, s = weights("i8", rng, K, N, oracle)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    want = reference.wmatmul(A, q, scale=s, alpha=0.75, beta=0.5, C_in=C0)
    C = dev(C0)
    with make_weight(cuda, args, K, N) as w:
        cuda.call("pkcu_wmatmul", dev(A).data_ptr(), w.handle, C.data_ptr(), M, 0.75, 0.5,
                  work(cuda, M, K).data_ptr(), None)
        got = host(C).reshape(M, N)
    check(got, want, 0.75 * bound(A, W) + 1e-6 * np.abs(C0), "alpha A W + beta C")


@pytest.mark.parametrize("kind", ["i8", "f32", "i4_g32_n"])
def test_wmatmul_bias_swish(cuda, reference, oracle, kind):
    rng = np.random.default_rng(5 + len(kind))
    M, N, K = 416, 4096, 1024
    A = rng.standard_normal((M, K)).astype(np.float32)
    args, W, q, s = weights(kind, rng, K, N, oracle)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    want = reference.ff_linear1(A, W, b)   # pk_wmatmul + pk_bias_add + pk_swish
    D = empty(M * N)
    with make_weight(cuda, args, K, N) as w:
        cuda.call("pkcu_wmatmul_bias_swish", dev(A).data_ptr(), w.handle, dev(b).data_ptr(), D.data_ptr(),
                  M, work(cuda, M, K).data_ptr(), None)
        got = host(D).reshape(M, N)
    # Swish is 1-Lipschitz up to 1.1: the GEMM bound carries over
    check(got, want, 1.1 * bound(A, W) + 1e-6 * np.abs(want), f"{kind} Swish(A W + b)")


@pytest.mark.parametrize("kind,M,N,K,scale", [("i8", 416, 1024, 4096, 0.5), ("i8", 37, 1024, 1024, 1.0),
                                              ("f32", 300, 1024, 4096, 0.5), ("i4_g128_k", 129, 1024, 4096, 0.5)])
def test_wmatmul_bias_residual(cuda, reference, oracle, kind, M, N, K, scale):
    rng = np.random.default_rng(7 * M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    args, W, q, s = weights(kind, rng, K, N, oracle)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    x = rng.standard_normal((M, N)).astype(np.float32)
    want = reference.linear_residual(x, A, W, b, scale)
    X = dev(x)
    with make_weight(cuda, args, K, N) as w:
        cuda.call("pkcu_wmatmul_bias_residual", dev(A).data_ptr(), w.handle, dev(b).data_ptr(), X.data_ptr(),
                  scale, M, work(cuda, M, K).data_ptr(), None)
        got = host(X).reshape(M, N)
    check(got, want, scale * bound(A, W) + 1e-6 * np.abs(x), f"{kind} X + s (A W + b)")


@pytest.mark.parametrize("lengths", [[375, 375], [408, 416, 7, 129]])
def test_wmatmul_qkv(cuda, reference, oracle, lengths):
    """The fused QKV projection with its epilogue against pk_wmatmul on the
    fused int8 weight, then the bias + head split + u/v of each utterance."""
    D = 1024
    rng = np.random.default_rng(sum(lengths))
    F = sum(lengths)
    A = rng.standard_normal((F, D)).astype(np.float32)
    args, W, q, s = weights("i8", rng, D, 3 * D, oracle)
    bqkv = (0.1 * rng.standard_normal(3 * D)).astype(np.float32)
    u = (0.1 * rng.standard_normal(D)).astype(np.float32)
    v = (0.1 * rng.standard_normal(D)).astype(np.float32)
    qkv = reference.wmatmul(A, q, scale=s)
    outs = [empty(F * D) for _ in range(4)]
    with make_weight(cuda, args, D, 3 * D) as w, cuda.Seq(lengths) as seq:
        cuda.call("pkcu_wmatmul_qkv", dev(A).data_ptr(), w.handle, dev(bqkv).data_ptr(), dev(u).data_ptr(),
                  dev(v).data_ptr(), *[o.data_ptr() for o in outs], seq.handle,
                  work(cuda, F, D).data_ptr(), None)
        got = [host(o) for o in outs]
    tol_rows = bound(A, W)
    f0 = 0
    for T in lengths:
        want = oracle.qkv_split_uv(qkv[f0:f0 + T], bqkv, u, v)   # Qu, Qv, K, V as [8, T, 128]
        tol = tol_rows[f0:f0 + T]
        for name, g, wv, cols in zip(("Qu", "Qv", "K", "V"), got, want, (0, 0, 1, 2)):
            gt = g[f0 * D:(f0 + T) * D].reshape(8, T, 128)
            tt = tol[:, cols * D:(cols + 1) * D].reshape(T, 8, 128).transpose(1, 0, 2)
            check(gt, wv, tt + 1e-6 * np.abs(wv), f"{name} of the {T}-frame item")
        f0 += T


def test_bad_arguments(cuda):
    import ctypes as C
    L = cuda.lib()
    h = C.c_void_p()
    x = empty(64)
    assert L.pkcu_weight_create(x.data_ptr(), 32, 0.0, None, 32, 1, 48, 64, None, C.byref(h)) == 1   # K % 32
    assert L.pkcu_weight_create(x.data_ptr(), 16, 0.0, None, 32, 1, 32, 64, None, C.byref(h)) == 1   # bits
    assert L.pkcu_weight_create(x.data_ptr(), 8, 0.0, None, 32, 1, 32, 64, None, C.byref(h)) == 1    # scale
    assert L.pkcu_wmatmul(None, None, None, 1, 1.0, 0.0, None, None) == 1


def conv_bound(w, x):
    return 1e-5 * (np.abs(w).astype(np.float64) @ np.abs(x).astype(np.float64)) + 2e-6


@pytest.mark.parametrize("Cout,T", [(1024, 375), (2048, 33), (1024, 1)])
def test_pointwise_conv1d(cuda, reference, Cout, T):
    """pkcu_pointwise_conv1d against the reference's pk_pointwise_conv1d
    (csrc/tensor_ops.c:579-590): out = W x + b, channel-first."""
    Cin = 1024
    rng = np.random.default_rng(Cout + T)
    x = rng.standard_normal((Cin, T)).astype(np.float32)
    w = (rng.standard_normal((Cout, Cin)) / np.sqrt(Cin)).astype(np.float32)
    b = (0.1 * rng.standard_normal(Cout)).astype(np.float32)
    want = reference.pointwise_conv1d(x, w, b)
    out = empty(Cout * T)
    with cuda.ConvWeight(dev(w), Cout, Cin, glu=False) as W:
        cuda.call("pkcu_pointwise_conv1d", dev(x).data_ptr(), W.handle, dev(b).data_ptr(), out.data_ptr(), T,
                  work(cuda, T, Cin).data_ptr(), None)
        got = host(out).reshape(Cout, T)
    check(got, want, conv_bound(w, x), "W x + b")


@pytest.mark.parametrize("T", [375, 129])
def test_pointwise_conv1d_glu(cuda, reference, oracle, T):
    """The first pointwise convolution with the GLU in its epilogue against
    pk_pointwise_conv1d then the GLU restatement (csrc/encoder.c:457-465);
    the GLU is 1-Lipschitz in a and 0.25 |a| in g, so the bound carries over."""
    C2, Cin = 2048, 1024
    rng = np.random.default_rng(T)
    x = rng.standard_normal((Cin, T)).astype(np.float32)
    w = (rng.standard_normal((C2, Cin)) / np.sqrt(Cin)).astype(np.float32)
    b = (0.1 * rng.standard_normal(C2)).astype(np.float32)
    pw1 = reference.pointwise_conv1d(x, w, b)
    want = oracle.glu_channel_first(pw1)
    out = empty(C2 // 2 * T)
    with cuda.ConvWeight(dev(w), C2, Cin, glu=True) as W:
        cuda.call("pkcu_pointwise_conv1d_glu", dev(x).data_ptr(), W.handle, dev(b).data_ptr(), out.data_ptr(),
                  T, work(cuda, T, Cin).data_ptr(), None)
        got = host(out).reshape(C2 // 2, T)
    tb = conv_bound(w, x)
    tol = tb[:C2 // 2] + 0.25 * np.abs(pw1[:C2 // 2]) * tb[C2 // 2:] + 1e-5 * np.abs(want) + 2e-6
    check(got, want, tol, "GLU(W x + b)")

