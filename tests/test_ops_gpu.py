"""GPU parity: every device-API op against the CPU restatement (oracle/) on
the same seeded inputs, through the C ABI.

Exact ops (data movement, adds, the polynomial Swish body, the depthwise FMA
chain, dequantisation, argmax) must match bit for bit; LayerNorm, softmax,
GLU and tanh within |diff| <= max(2e-6, 1e-5 |ref|)."""
import numpy as np
import pytest

from conftest import assert_bitexact, assert_close
from gpuhelp import D, DH, FF, H, Layout, dev, empty, host

pytestmark = pytest.mark.gpu

RAGGED = [[1, 7, 3, 32], [408, 416, 416, 408], [9], [375, 375]]
# enough 32-frame tiles for every SM: the transposing kernels' 32-frame path
# (the cases above take the 16-frame one)
WIDE = [[375] * 13 + [1, 37, 16, 17]]


def rng(seed):
    return np.random.default_rng(seed)


def test_selftest_reciprocal(cuda):
    """Every float d in [1, 2^126): fast reciprocal == correctly rounded 1/d."""
    import ctypes as C
    bad = C.c_ulonglong(12345)
    cuda.call("pkcu_selftest", C.byref(bad))
    assert bad.value == 0


def test_selftest_wait_bound(cuda, oracle):
    """A bounded device wait on a copy that never comes gives up after 20 ms,
    reports it, and the context stays usable."""
    import ctypes as C
    t = C.c_int(-1)
    cuda.call("pkcu_selftest_wait", C.byref(t))
    assert t.value == 1
    x = rng(5).standard_normal(4096).astype(np.float32)
    g = dev(x)
    cuda.call("pkcu_swish", g.data_ptr(), x.size, cuda.stream_handle())
    assert_bitexact(host(g), oracle.swish(x), "swish after the timed-out wait")


def test_swish_dense_sweep(cuda, oracle):
    """Swish body bit-exact against the restatement on a dense sweep of
    [-100, 100] (every 509th float of that range)."""
    u = np.arange(0, 0x42C80000, 509, dtype=np.uint32)     # [+0, 100)
    pos = u.view(np.float32)
    x = np.concatenate([pos, -pos]).astype(np.float32)
    x = x[: x.size & ~7]
    xd = dev(x)
    cuda.call("pkcu_swish", xd.data_ptr(), x.size, cuda.stream_handle())
    assert_bitexact(host(xd), oracle.swish(x), "swish sweep")


def exp_rounding_ties():
    """Floats x in [-87, 87] whose float32 product x * log2(e) is exactly
    k + 1/2: the inputs on which the reference's exp (pk_exp_avx2,
    csrc/tensor_ops.c:97-121: the product rounded, then rounded to an integer,
    ties to even) and an exp that fuses the product into the rounding add
    choose different k."""
    l2e = np.float32(1.44269504088896341)
    found = []
    for t in np.arange(126, dtype=np.float32) + np.float32(0.5):   # |k + 1/2|
        b0 = int(np.array([t / l2e], np.float32).view(np.int32)[0])
        xs = np.arange(b0 - 64, b0 + 65, dtype=np.int32).view(np.float32)
        found.extend(xs[(xs * l2e) == t].tolist())
    x = np.array(found, np.float32)
    x = x[x <= np.float32(87.0)]
    return np.concatenate([x, -x])


def test_swish_exp_rounding_ties(cuda, oracle):
    """Swish bit-exact against the restatement on every input whose exp
    argument sits on a rounding tie of x * log2(e) (and its two float
    neighbours): the packed f32x2 arithmetic must round the product and the
    shifter add separately, as the reference does."""
    ties = exp_rounding_ties()
    assert ties.size > 200
    near = np.concatenate([np.nextafter(ties, np.float32(np.inf)), np.nextafter(ties, np.float32(-np.inf))])
    v = -np.concatenate([ties, near]).astype(np.float32)   # Swish takes exp(-v)
    v = np.concatenate([v, np.zeros((-v.size) % 8, np.float32)])
    vd = dev(v)
    cuda.call("pkcu_swish", vd.data_ptr(), v.size, cuda.stream_handle())
    assert_bitexact(host(vd), oracle.swish(v), "swish on exp rounding ties")


def test_glu_gate_dense_sweep(cuda, oracle):
    """The GLU gate's own exp (ex2-based, pk_common.cuh glu_gate) on a dense
    sweep of gate values in [-100, 100] (every 509th float) plus the clamp
    edges and NaN: a * 1/(1 + exp(-g)) with a = 1 against the restatement
    (glibc expf, as the reference computes it) within the GLU tolerance, and
    against the float64 sigmoid within 4 units in the last place inside the
    clamp (|g| <= 86) where the result is a normal float."""
    u = np.arange(0, 0x42C80000, 509, dtype=np.uint32)     # [+0, 100)
    pos = u.view(np.float32)
    g = np.concatenate([pos, -pos, np.float32([86.0, -86.0, 85.99, -86.01, 88.7, -88.8, 1e30, -1e30])])
    g = g.astype(np.float32)
    n = (g.size + D - 1) // D * D
    g = np.concatenate([g, np.zeros(n - g.size, np.float32)])
    rows = n // D
    tf = np.empty((rows, 2 * D), np.float32)
    tf[:, :D] = 1.0
    tf[:, D:] = g.reshape(rows, D)
    out = empty((rows, D))
    with cuda.Seq([rows]) as seq:
        cuda.call("pkcu_glu", dev(tf).data_ptr(), None, out.data_ptr(), D, cuda.PKCU_TIME_FIRST,
                  seq.handle, cuda.stream_handle())
        got = host(out).reshape(-1)
    assert_close(got, oracle.glu_time_first(tf).reshape(-1), "gate vs glibc expf")
    exact = 1.0 / (1.0 + np.exp(-g.astype(np.float64)))
    normal = (exact >= np.finfo(np.float32).tiny) & (np.abs(g) <= 86.0)   # inside the clamp
    ulp = np.spacing(exact[normal].astype(np.float32)).astype(np.float64)
    err_ulp = np.abs(got[normal].astype(np.float64) - exact[normal]) / ulp
    assert err_ulp.max() <= 4.0, err_ulp.max()
    # a NaN gate gives NaN (1/(1 + expf(NaN)) in the reference)
    tf[0, D] = np.nan
    with cuda.Seq([rows]) as seq:
        cuda.call("pkcu_glu", dev(tf).data_ptr(), None, out.data_ptr(), D, cuda.PKCU_TIME_FIRST,
                  seq.handle, cuda.stream_handle())
        assert np.isnan(host(out)[0, 0])


# ── LayerNorm family ──────────────────────────────────────────────────────────

@pytest.mark.parametrize("R,Dd,offset", [(1, 1024, 0), (7, 1024, 0), (375, 1024, 0),
                                         (1000, 1024, 0), (8000, 1024, 0), (5, 37, 0),
                                         (4, 1024, 1), (3, 2048, 0), (2, 1, 0)])
def test_layer_norm_rows(cuda, oracle, R, Dd, offset):
    r = rng(R * Dd + offset)
    x = r.standard_normal((R, Dd)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(Dd)).astype(np.float32)
    b = (0.1 * r.standard_normal(Dd)).astype(np.float32)
    buf = dev(np.concatenate([np.zeros(offset, np.float32), x.reshape(-1)]))
    xd = buf[offset:]
    out = empty(R * Dd)
    cuda.call("pkcu_layer_norm_rows", xd.data_ptr(), dev(g).data_ptr(), dev(b).data_ptr(),
              out.data_ptr(), R, Dd, cuda.stream_handle())
    want = oracle.layer_norm_rows(x, g, b)
    assert_close(host(out).reshape(R, Dd), want, "ln")
    # in place (pk_layer_norm_rows_inplace)
    cuda.call("pkcu_layer_norm_rows", xd.data_ptr(), dev(g).data_ptr(), dev(b).data_ptr(),
              xd.data_ptr(), R, Dd, cuda.stream_handle())
    assert_close(host(xd).reshape(R, Dd), want, "ln inplace")


@pytest.mark.parametrize("R", [777, 7501])
def test_residual_layer_norm(cuda, oracle, R):
    r = rng(3 + R)
    x = r.standard_normal((R, D)).astype(np.float32)
    y = r.standard_normal((R, D)).astype(np.float32)
    bias = (0.1 * r.standard_normal(D)).astype(np.float32)
    g1, g2 = ((1 + 0.1 * r.standard_normal(D)).astype(np.float32) for _ in range(2))
    b1, b2 = ((0.1 * r.standard_normal(D)).astype(np.float32) for _ in range(2))
    for alpha in (0.5, 1.0):
        xr = oracle.residual(x, oracle.bias_add_rows(y, bias), alpha)
        xd, ln = dev(x), empty((R, D))
        cuda.call("pkcu_residual_layer_norm", xd.data_ptr(), dev(y).data_ptr(),
                  dev(bias).data_ptr(), alpha, dev(g1).data_ptr(), dev(b1).data_ptr(),
                  ln.data_ptr(), R, cuda.stream_handle())
        assert_bitexact(host(xd), xr, "x")
        assert_close(host(ln), oracle.layer_norm_rows(xr, g1, b1), "ln")
    # residual + LN_out in place + next block's LN
    xr = oracle.residual(x, oracle.bias_add_rows(y, bias), 0.5)
    x2 = oracle.layer_norm_rows(xr, g1, b1)
    xd, ln = dev(x), empty((R, D))
    cuda.call("pkcu_residual_layer_norm2", xd.data_ptr(), dev(y).data_ptr(), dev(bias).data_ptr(),
              0.5, dev(g1).data_ptr(), dev(b1).data_ptr(), dev(g2).data_ptr(), dev(b2).data_ptr(),
              ln.data_ptr(), R, cuda.stream_handle())
    assert_close(host(xd), x2, "x after LN_out")
    assert_close(host(ln), oracle.layer_norm_rows(host(xd), g2, b2), "LN_next")
    # without the next LN
    xd = dev(x)
    cuda.call("pkcu_residual_layer_norm2", xd.data_ptr(), dev(y).data_ptr(), None, 1.0,
              dev(g1).data_ptr(), dev(b1).data_ptr(), None, None, None, R, cuda.stream_handle())
    assert_close(host(xd), oracle.layer_norm_rows(oracle.residual(x, y, 1.0), g1, b1), "no next")


@pytest.mark.parametrize("lengths", RAGGED + WIDE)
def test_layer_norm_transpose(cuda, oracle, lengths):
    r = rng(sum(lengths))
    L = Layout(lengths)
    F = L.frames
    x = r.standard_normal((F, D)).astype(np.float32)
    y = r.standard_normal((F, D)).astype(np.float32)
    bias = (0.1 * r.standard_normal(D)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(D)).astype(np.float32)
    b = (0.1 * r.standard_normal(D)).astype(np.float32)
    with cuda.Seq(lengths) as seq:
        cf = empty(F * D)
        cuda.call("pkcu_layer_norm_transpose", dev(x).data_ptr(), dev(g).data_ptr(),
                  dev(b).data_ptr(), cf.data_ptr(), seq.handle, cuda.stream_handle())
        got = host(cf)
        for i, T in enumerate(lengths):
            want = oracle.transpose(oracle.layer_norm_rows(L.frames_of(x, i), g, b))
            assert_close(L.chunk(got, i, D, (D, T)), want, f"item {i}")
        # fused with the attention residual
        xd, cf = dev(x), empty(F * D)
        cuda.call("pkcu_residual_layer_norm_transpose", xd.data_ptr(), dev(y).data_ptr(),
                  dev(bias).data_ptr(), 1.0, dev(g).data_ptr(), dev(b).data_ptr(), cf.data_ptr(),
                  seq.handle, cuda.stream_handle())
        xr = oracle.residual(x, oracle.bias_add_rows(y, bias), 1.0)
        assert_bitexact(host(xd), xr, "x")
        got = host(cf)
        for i, T in enumerate(lengths):
            want = oracle.transpose(oracle.layer_norm_rows(L.frames_of(xr, i), g, b))
            assert_close(L.chunk(got, i, D, (D, T)), want, f"res item {i}")


@pytest.mark.parametrize("lengths", RAGGED + WIDE)
def test_transpose_add_layer_norm(cuda, oracle, lengths):
    r = rng(7 + sum(lengths))
    L = Layout(lengths)
    F = L.frames
    x = r.standard_normal((F, D)).astype(np.float32)
    y = r.standard_normal(F * D).astype(np.float32)       # per item [D, T]
    bias = (0.1 * r.standard_normal(D)).astype(np.float32)
    g = (1 + 0.1 * r.standard_normal(D)).astype(np.float32)
    b = (0.1 * r.standard_normal(D)).astype(np.float32)
    want_x = np.empty_like(x)
    for i, T in enumerate(lengths):
        pw2 = oracle.pointwise_bias(L.chunk(y, i, D, (D, T)), bias)
        want_x[L.frame[i]:L.frame[i + 1]] = oracle.transpose_add(L.frames_of(x, i), pw2)
    with cuda.Seq(lengths) as seq:
        xd = dev(x)
        cuda.call("pkcu_transpose_add", xd.data_ptr(), dev(y).data_ptr(), dev(bias).data_ptr(),
                  seq.handle, cuda.stream_handle())
        assert_bitexact(host(xd), want_x, "transpose_add")
        xd, ln = dev(x), empty((F, D))
        cuda.call("pkcu_transpose_add_layer_norm", xd.data_ptr(), dev(y).data_ptr(),
                  dev(bias).data_ptr(), dev(g).data_ptr(), dev(b).data_ptr(), ln.data_ptr(),
                  seq.handle, cuda.stream_handle())
        assert_bitexact(host(xd), want_x, "x")
        assert_close(host(ln), oracle.layer_norm_rows(want_x, g, b), "ln")


# ── softmax and the relative-position scores ─────────────────────────────────

@pytest.mark.parametrize("R,n", [(3, 1), (5, 7), (9, 8), (4, 31), (4, 33), (3000, 375),
                                 (64, 416), (8, 1000), (6, 1025), (3, 5000), (7, 300),
                                 (5, 200), (3, 500), (17, 129)])
def test_softmax_rows(cuda, oracle, R, n):
    x = (3 * rng(R + n).standard_normal((R, n))).astype(np.float32)
    xd = dev(x)
    cuda.call("pkcu_softmax_rows", xd.data_ptr(), R, n, cuda.stream_handle())
    assert_close(host(xd), oracle.softmax_rows(x), f"softmax {R}x{n}")


@pytest.mark.parametrize("lengths", RAGGED + [[1100, 33], [600, 7], [512, 1], [1000, 12, 13, 15],
                                     [129, 130, 131, 126]])
def test_relpos_scores(cuda, oracle, lengths):
    r = rng(11 + sum(lengths))
    L = Layout(lengths)
    ac = r.standard_normal(L.score[-1]).astype(np.float32) * 4
    bd = r.standard_normal(L.bd[-1]).astype(np.float32) * 4
    scale = np.float32(1.0) / np.sqrt(np.float32(128.0))
    with cuda.Seq(lengths) as seq:
        acd, bdd = dev(ac), dev(bd)
        out = empty(L.score[-1])
        cuda.call("pkcu_relative_shift", bdd.data_ptr(), out.data_ptr(), seq.handle,
                  cuda.stream_handle())
        got = host(out)
        for i in range(len(lengths)):
            assert_bitexact(L.scores(got, i), oracle.relative_shift(L.bds(bd, i)), f"shift {i}")
        cuda.call("pkcu_relpos_combine", acd.data_ptr(), bdd.data_ptr(), out.data_ptr(),
                  float(scale), seq.handle, cuda.stream_handle())
        got = host(out)
        comb = [oracle.relpos_combine(L.scores(ac, i), L.bds(bd, i), float(scale))
                for i in range(len(lengths))]
        for i in range(len(lengths)):
            assert_bitexact(L.scores(got, i), comb[i], f"combine {i}")
        cuda.call("pkcu_relpos_combine_softmax", acd.data_ptr(), bdd.data_ptr(), out.data_ptr(),
                  float(scale), seq.handle, cuda.stream_handle())
        got = host(out)
        for i, T in enumerate(lengths):
            want = oracle.softmax_rows(comb[i].reshape(H * T, T)).reshape(H, T, T)
            assert_close(L.scores(got, i), want, f"softmax {i}")
        # in place (S == ac), as the reference overwrites ac
        cuda.call("pkcu_relpos_combine_softmax", acd.data_ptr(), bdd.data_ptr(), acd.data_ptr(),
                  float(scale), seq.handle, cuda.stream_handle())
        assert_bitexact(host(acd), got, "in place")


# Batches with enough score rows for the pipelined kernel (the cases above
# are short enough for the one-warp-per-row kernel): one case per chunk
# configuration of the dispatch, ragged where it matters.
@pytest.mark.parametrize("lengths", [[50] * 150, [120] * 60, [250] * 29, [375] * 19 + [1],
                                     [416] * 17 + [408], [700] * 11, [1000] * 7 + [999]])
def test_relpos_scores_pipelined(cuda, oracle, lengths):
    r = rng(17 + sum(lengths))
    L = Layout(lengths)
    ac = r.standard_normal(L.score[-1]).astype(np.float32) * 4
    bd = r.standard_normal(L.bd[-1]).astype(np.float32) * 4
    scale = np.float32(1.0) / np.sqrt(np.float32(128.0))
    with cuda.Seq(lengths) as seq:
        acd, bdd = dev(ac), dev(bd)
        out = empty(L.score[-1])
        cuda.call("pkcu_relpos_combine", acd.data_ptr(), bdd.data_ptr(), out.data_ptr(),
                  float(scale), seq.handle, cuda.stream_handle())
        got = host(out)
        comb = [oracle.relpos_combine(L.scores(ac, i), L.bds(bd, i), float(scale))
                for i in range(len(lengths))]
        for i in range(len(lengths)):
            assert_bitexact(L.scores(got, i), comb[i], f"combine {i}")
        cuda.call("pkcu_relpos_combine_softmax", acd.data_ptr(), bdd.data_ptr(), out.data_ptr(),
                  float(scale), seq.handle, cuda.stream_handle())
        got = host(out)
        for i, T in enumerate(lengths):
            want = oracle.softmax_rows(comb[i].reshape(H * T, T)).reshape(H, T, T)
            assert_close(L.scores(got, i), want, f"softmax {i}")


# ── head layouts ──────────────────────────────────────────────────────────────

@pytest.mark.parametrize("lengths", RAGGED)
def test_head_layouts(cuda, oracle, lengths):
    r = rng(13 + sum(lengths))
    L = Layout(lengths)
    F = L.frames
    qkv = r.standard_normal((F, 3 * D)).astype(np.float32)
    bqkv = (0.1 * r.standard_normal(3 * D)).astype(np.float32)
    u = (0.1 * r.standard_normal((H, DH))).astype(np.float32)
    v = (0.1 * r.standard_normal((H, DH))).astype(np.float32)
    P = r.standard_normal((int(L.pos[-1]), D)).astype(np.float32)
    ah = r.standard_normal(F * D).astype(np.float32)
    with cuda.Seq(lengths) as seq:
        outs = [empty(F * D) for _ in range(4)]
        cuda.call("pkcu_qkv_split_uv", dev(qkv).data_ptr(), dev(bqkv).data_ptr(), dev(u).data_ptr(),
                  dev(v).data_ptr(), *[o.data_ptr() for o in outs], seq.handle,
                  cuda.stream_handle())
        got = [host(o) for o in outs]
        for i, T in enumerate(lengths):
            want = oracle.qkv_split_uv(L.frames_of(qkv, i, 3 * D), bqkv, u, v)
            for name, gg, w in zip(("Qu", "Qv", "K", "V"), got, want):
                assert_bitexact(L.chunk(gg, i, D, (H, T, DH)), w, f"{name} item {i}")
        ph = empty(int(L.pos[-1]) * D)
        cuda.call("pkcu_pos_head_split", dev(P).data_ptr(), ph.data_ptr(), seq.handle,
                  cuda.stream_handle())
        got = host(ph)
        for i, T in enumerate(lengths):
            Li = 2 * T - 1
            gi = got[L.pos[i] * D:L.pos[i + 1] * D].reshape(H, Li, DH)
            assert_bitexact(gi, oracle.pos_head_split(L.posrows(P, i)), f"P_h item {i}")
        at = empty((F, D))
        cuda.call("pkcu_head_concat", dev(ah).data_ptr(), at.data_ptr(), seq.handle,
                  cuda.stream_handle())
        got = host(at)
        for i, T in enumerate(lengths):
            assert_bitexact(L.frames_of(got, i), oracle.head_concat(L.chunk(ah, i, D, (H, T, DH))),
                            f"concat item {i}")


# ── elementwise ───────────────────────────────────────────────────────────────

@pytest.mark.parametrize("n,offset", [(1, 0), (7, 0), (8, 0), (1003, 0), (375 * 4096, 0),
                                      (1003, 1), (4096, 3)])
def test_swish(cuda, oracle, n, offset):
    x = (4 * rng(n + offset).standard_normal(n)).astype(np.float32)
    buf = dev(np.concatenate([np.zeros(offset, np.float32), x]))
    xd = buf[offset:]
    cuda.call("pkcu_swish", xd.data_ptr(), n, cuda.stream_handle())
    got, want = host(xd), oracle.swish(x)
    n8 = n & ~7
    assert_bitexact(got[:n8], want[:n8], "polynomial body")
    assert_close(got[n8:], want[n8:], "expf tail")


def test_relu(cuda, oracle):
    x = rng(5).standard_normal(1003).astype(np.float32)
    x[[0, 5, 999, 1001]] = [np.nan, -0.0, np.nan, -0.0]
    for off in (0, 1):
        buf = dev(np.concatenate([np.zeros(off, np.float32), x]))
        xd = buf[off:]
        cuda.call("pkcu_relu", xd.data_ptr(), x.size, cuda.stream_handle())
        assert_bitexact(host(xd), oracle.relu(x), f"relu off={off}")


@pytest.mark.parametrize("R,n", [(375, 4096), (7, 3072), (5, 37), (1, 1)])
def test_bias_rows(cuda, oracle, R, n):
    r = rng(R * n)
    x = r.standard_normal((R, n)).astype(np.float32)
    b = r.standard_normal(n).astype(np.float32)
    y = r.standard_normal((R, n)).astype(np.float32)
    xd = dev(x)
    cuda.call("pkcu_bias_add_rows", xd.data_ptr(), dev(b).data_ptr(), R, n, cuda.stream_handle())
    assert_bitexact(host(xd), oracle.bias_add_rows(x, b), "bias")
    out = empty((R, n))
    cuda.call("pkcu_bias_swish_rows", dev(x).data_ptr(), dev(b).data_ptr(), out.data_ptr(), R, n,
              cuda.stream_handle())
    want = oracle.swish(oracle.bias_add_rows(x, b))
    n8 = (R * n) & ~7
    assert_bitexact(host(out).reshape(-1)[:n8], want.reshape(-1)[:n8], "bias+swish")
    assert_close(host(out), want, "bias+swish")
    xd = dev(x)
    cuda.call("pkcu_residual_add", xd.data_ptr(), dev(y).data_ptr(), dev(b).data_ptr(), 0.5, R, n,
              cuda.stream_handle())
    assert_bitexact(host(xd), oracle.residual(x, oracle.bias_add_rows(y, b), 0.5), "residual")


# ── conv module ───────────────────────────────────────────────────────────────

@pytest.mark.parametrize("lengths", RAGGED)
def test_glu(cuda, oracle, lengths):
    r = rng(17 + sum(lengths))
    L = Layout(lengths)
    F = L.frames
    pw1 = r.standard_normal(2 * F * D).astype(np.float32) * 3
    bias = (0.1 * r.standard_normal(2 * D)).astype(np.float32)
    with cuda.Seq(lengths) as seq:
        out = empty(F * D)
        cuda.call("pkcu_glu", dev(pw1).data_ptr(), dev(bias).data_ptr(), out.data_ptr(), D,
                  cuda.PKCU_CHANNEL_FIRST, seq.handle, cuda.stream_handle())
        got = host(out)
        for i, T in enumerate(lengths):
            item = L.chunk(pw1, i, 2 * D, (2 * D, T))
            want = oracle.glu_channel_first(oracle.pointwise_bias(item, bias))
            assert_close(L.chunk(got, i, D, (D, T)), want, f"glu item {i}")
        tf = r.standard_normal((F, 2 * D)).astype(np.float32)
        out = empty((F, D))
        cuda.call("pkcu_glu", dev(tf).data_ptr(), None, out.data_ptr(), D, cuda.PKCU_TIME_FIRST,
                  seq.handle, cuda.stream_handle())
        assert_close(host(out), oracle.glu_time_first(tf), "glu time-first")


@pytest.mark.parametrize("C,T,K,bias,offset", [
    (1024, 375, 9, True, 0), (16, 1, 9, True, 0), (16, 2, 9, False, 0), (8, 5, 3, True, 0),
    (32, 129, 9, True, 0), (4, 300, 31, True, 0), (6, 40, 1, True, 0), (1024, 32, 9, True, 0),
    (8, 7, 9, True, 0), (8, 11, 9, True, 0), (8, 15, 9, True, 0), (8, 16, 9, True, 0),
    (64, 375, 9, True, 1), (24, 642, 9, True, 0), (24, 645, 9, True, 0), (24, 646, 9, True, 0),
    (16, 900, 9, True, 0)])
def test_depthwise_conv1d(cuda, oracle, C, T, K, bias, offset):
    """offset != 0 misaligns x (the bulk-copy path needs 16-byte aligned rows); T = 646 and
    900 exceed the shared-memory row and take the chunked path."""
    r = rng(C * T + K)
    x = r.standard_normal((C, T)).astype(np.float32)
    w = (0.3 * r.standard_normal((C, K))).astype(np.float32)
    b = (0.1 * r.standard_normal(C)).astype(np.float32) if bias else None
    buf = dev(np.concatenate([np.zeros(offset, np.float32), x.reshape(-1)]))
    out = empty((C, T))
    cuda.call("pkcu_depthwise_conv1d", buf[offset:].data_ptr(), dev(w).data_ptr(),
              dev(b).data_ptr() if bias else None, out.data_ptr(), C, T, K, cuda.stream_handle())
    assert_bitexact(host(out), oracle.depthwise_conv1d(x, w, b), "dwconv")


@pytest.mark.parametrize("lengths", RAGGED)
@pytest.mark.parametrize("with_bn", [False, True])
def test_dwconv_bn_swish(cuda, oracle, lengths, with_bn):
    r = rng(19 + sum(lengths))
    L = Layout(lengths)
    F = L.frames
    x = r.standard_normal(F * D).astype(np.float32)
    w = (0.3 * r.standard_normal((D, 9))).astype(np.float32)
    b = (0.1 * r.standard_normal(D)).astype(np.float32)
    bn = np.concatenate([0.1 * r.standard_normal(D), r.uniform(0.5, 1.5, D),
                         1 + 0.1 * r.standard_normal(D), 0.1 * r.standard_normal(D)]).astype(np.float32)
    with cuda.Seq(lengths) as seq:
        out = empty(F * D)
        cuda.call("pkcu_dwconv_bn_swish", dev(x).data_ptr(), dev(w).data_ptr(), dev(b).data_ptr(),
                  dev(bn).data_ptr() if with_bn else None, 1e-5, 1, out.data_ptr(), D, 9,
                  seq.handle, cuda.stream_handle())
        got = host(out)
        for i, T in enumerate(lengths):
            y = oracle.depthwise_conv1d(L.chunk(x, i, D, (D, T)), w, b)
            if with_bn:
                y = oracle.batch_norm(y, bn[:D], bn[D:2 * D], bn[2 * D:3 * D], bn[3 * D:], 1e-5)
            assert_bitexact(L.chunk(got, i, D, (D, T)), oracle.swish(y), f"item {i}")


@pytest.mark.parametrize("lengths,K", [([408, 416, 416, 408], 9), ([9, 1, 4], 9), ([700], 9),
                                       ([33, 20], 5)])
@pytest.mark.parametrize("with_bias", [True, False])
def test_glu_dwconv_fused(cuda, oracle, lengths, K, with_bias):
    """GLU folded into the depthwise conv: bit-identical to GLU then conv."""
    r = rng(23 + sum(lengths) + K)
    L = Layout(lengths)
    F = L.frames
    pw1 = (3 * r.standard_normal(2 * F * D)).astype(np.float32)
    gb = (0.1 * r.standard_normal(2 * D)).astype(np.float32)
    w = (0.3 * r.standard_normal((D, K))).astype(np.float32)
    b = (0.1 * r.standard_normal(D)).astype(np.float32)
    with cuda.Seq(lengths) as seq:
        gated, two, fused = empty(F * D), empty(F * D), empty(F * D)
        gbd = dev(gb).data_ptr() if with_bias else None
        cuda.call("pkcu_glu", dev(pw1).data_ptr(), gbd, gated.data_ptr(), D, cuda.PKCU_CHANNEL_FIRST,
                  seq.handle, cuda.stream_handle())
        cuda.call("pkcu_dwconv_bn_swish", gated.data_ptr(), dev(w).data_ptr(), dev(b).data_ptr(), None,
                  0.0, 1, two.data_ptr(), D, K, seq.handle, cuda.stream_handle())
        cuda.call("pkcu_glu_dwconv_bn_swish", dev(pw1).data_ptr(), gbd, dev(w).data_ptr(),
                  dev(b).data_ptr(), None, 0.0, 1, fused.data_ptr(), D, K, seq.handle,
                  cuda.stream_handle())
        got = host(fused)
        assert_bitexact(got, host(two), "fused == GLU then conv")
        for i, T in enumerate(lengths):
            item = L.chunk(pw1, i, 2 * D, (2 * D, T))
            g = oracle.glu_channel_first(oracle.pointwise_bias(item, gb) if with_bias else item)
            want = oracle.swish(oracle.depthwise_conv1d(g, w, b))
            assert_close(L.chunk(got, i, D, (D, T)), want, f"item {i}")


# ── weights ───────────────────────────────────────────────────────────────────

@pytest.mark.parametrize("n,offset,out_off", [(1024 * 3072, 0, 0), (1003, 0, 0), (4099, 3, 1),
                                             (4102, 4, 0), (4101, 0, 1), (5, 0, 0)])
def test_dequant_i8(cuda, oracle, n, offset, out_off):
    """offset / out_off misalign the int8 input (by bytes) and the output (by
    floats): the vector path needs 4-byte int8 and 16-byte output alignment."""
    import torch
    r = rng(n)
    q = r.integers(-127, 128, size=n, dtype=np.int8)
    s = float(np.float32(r.uniform(1e-3, 1e-2)))
    buf = dev(np.concatenate([np.zeros(offset, np.int8), q]))
    out = empty(n + out_off)[out_off:]
    cuda.call("pkcu_dequant_i8", buf[offset:].data_ptr(), s, out.data_ptr(), n,
              cuda.stream_handle())
    assert_bitexact(host(out), oracle.dequant_i8(q, s), "int8")
    del torch


def test_requant_qkv(cuda, oracle):
    import ctypes as C
    import torch
    r = rng(23)
    K, Dd = 1024, 1024
    q, k, v = (r.integers(-127, 128, size=(K, Dd), dtype=np.int8) for _ in range(3))
    for sq, sk, sv in ((0.004, 0.0075, 0.006), (0.01, 0.01, 0.002), (0.003, 0.003, 0.003)):
        fused = empty((K, 3 * Dd), torch.int8)
        ms = C.c_float()
        cuda.call("pkcu_requant_qkv_i8", dev(q).data_ptr(), dev(k).data_ptr(), dev(v).data_ptr(),
                  sq, sk, sv, fused.data_ptr(), C.byref(ms), K, Dd, cuda.stream_handle())
        want, wms = oracle.requant_qkv_i8(q, k, v, sq, sk, sv)
        assert np.float32(ms.value) == np.float32(wms)
        assert_bitexact(host(fused), want, f"requant {sq},{sk},{sv}")


@pytest.mark.parametrize("K,N,G,axis", [(1024, 4096, 32, 1), (4096, 1024, 32, 1),
                                        (1024, 4096, 128, 0), (4096, 1024, 128, 0),
                                        (6, 18, 3, 1), (16, 10, 8, 0), (8, 24, 2, 1),
                                        (24, 40, 4, 0), (3, 8, 8, 1), (5, 16, 16, 1),
                                        (128, 72, 8, 1), (16, 512, 8, 1), (12, 512, 16, 1),
                                        (8, 768, 64, 1), (3, 256, 128, 1), (4, 256, 256, 1)])
def test_dequant_i4(cuda, oracle, K, N, G, axis):
    r = rng(K + N + G)
    q = r.integers(-8, 8, size=(K, N)).astype(np.int8)
    packed = ((q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
    shape = (K, N // G) if axis == 1 else (K // G, N)
    sc = r.uniform(1e-3, 2e-2, size=shape).astype(np.float32)
    out = empty((K, N))
    cuda.call("pkcu_dequant_i4", dev(packed).data_ptr(), dev(sc).data_ptr(), out.data_ptr(), K, N,
              G, axis, cuda.stream_handle())
    assert_bitexact(host(out), oracle.dequant_i4(packed, sc, K, N, G, axis), "int4")


def test_dequant_i4_qkv(cuda, oracle):
    r = rng(29)
    K, Dd, G = 1024, 1024, 32
    ps, ss = [], []
    for _ in range(3):
        q = r.integers(-8, 8, size=(K, Dd)).astype(np.int8)
        ps.append(((q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)).astype(np.uint8))
        ss.append(r.uniform(1e-3, 2e-2, size=(K, Dd // G)).astype(np.float32))
    out = empty((K, 3 * Dd))
    cuda.call("pkcu_dequant_i4_qkv", *[dev(p).data_ptr() for p in ps],
              *[dev(s).data_ptr() for s in ss], out.data_ptr(), K, Dd, G, cuda.stream_handle())
    assert_bitexact(host(out), oracle.dequant_i4_qkv(*ps, *ss, K, Dd, G), "int4 qkv")


# ── RNN-T joint ───────────────────────────────────────────────────────────────

@pytest.mark.parametrize("B,T,J", [(32, 416, 640), (2, 3, 6), (1, 1, 640)])
def test_joint_add_act(cuda, oracle, B, T, J):
    r = rng(B * T + J)
    enc = r.standard_normal((B, T, J)).astype(np.float32)
    pred = r.standard_normal((B, J)).astype(np.float32)
    enc.reshape(-1)[:2] = [-0.0, np.nan]
    out = empty((B, T, J))
    cuda.call("pkcu_joint_add_act", dev(enc).data_ptr(), dev(pred).data_ptr(), out.data_ptr(),
              B, T, J, cuda.PKCU_ACT_RELU, cuda.stream_handle())
    assert_bitexact(host(out), oracle.joint_add_act(enc, pred, 0), "relu")
    cuda.call("pkcu_joint_add_act", dev(enc).data_ptr(), dev(pred).data_ptr(), out.data_ptr(),
              B, T, J, cuda.PKCU_ACT_TANH, cuda.stream_handle())
    assert_close(host(out), oracle.joint_add_act(enc, pred, 1), "tanh")


@pytest.mark.parametrize("R,V", [(32 * 416, 1025), (7, 1), (5, 33), (3, 4000), (8, 100)])
def test_argmax_rows(cuda, oracle, R, V):
    import torch
    r = rng(R + V)
    lg = r.standard_normal((R, V)).astype(np.float32)
    if R >= 5 and V >= 4:
        lg[0, :] = 1.0                     # all tied -> 0
        lg[1, 0] = np.nan                  # NaN first -> 0
        lg[2, V // 2] = np.nan             # NaN elsewhere ignored
        lg[3, :] = -np.inf
        lg[4, V - 1] = lg[4, 1] = 50.0     # tie between 1 and V-1 -> 1
    if R >= 8 and V >= 70:
        lg[5, 35] = lg[5, 3] = np.inf      # tie inside one lane's entries (j, j + 32) -> 3
        lg[6, 2] = lg[6, 66] = 9.0         # same lane, first of the two -> 2
        lg[7, :] = np.nan                  # all NaN -> 0
    out = empty(R, torch.int32)
    cuda.call("pkcu_argmax_rows", dev(lg).data_ptr(), out.data_ptr(), R, V, cuda.stream_handle())
    assert_bitexact(host(out), oracle.argmax_rows(lg), "argmax")
