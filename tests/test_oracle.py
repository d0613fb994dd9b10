"""CPU: the restatement (oracle/) pinned against the reference.

Three kinds of evidence:
  * golden vectors produced by the reference's own compiled code
    (tests/golden/reference_vectors.npz, tests/golden/make_golden.py);
  * the reference library itself at the BASELINE shapes (T = 32, 375, 416),
    when oracle/_ref/libpkref.so was built;
  * known answers that follow from the reference code: the closed form of
    relative_shift, first-maximum argmax, int4 nibble order, requant rounding.
"""
import numpy as np
import pytest

from conftest import assert_bitexact, assert_close

import pyoracle as po


# ── golden vectors ───────────────────────────────────────────────────────────

def test_golden_layer_norm(oracle, golden):
    assert_close(oracle.layer_norm_rows(golden["ln_x"], golden["ln_g"], golden["ln_b"]),
                 golden["ln_out"], "ln")
    assert_close(oracle.layer_norm_rows(golden["ln37_x"], golden["ln37_g"], golden["ln37_b"]),
                 golden["ln37_out"], "ln D=37")


@pytest.mark.parametrize("name", ["sm7", "sm375", "sm32"])
def test_golden_softmax(oracle, golden, name):
    assert_close(oracle.softmax_rows(golden[name + "_x"]), golden[name + "_out"], name)


def test_golden_swish_relu(oracle, golden):
    assert_close(oracle.swish(golden["swish_x"]), golden["swish_out"], "swish")
    assert_bitexact(oracle.relu(golden["relu_x"]), golden["relu_out"], "relu")


def test_golden_dwconv(oracle, golden):
    assert_close(oracle.depthwise_conv1d(golden["dw_x"], golden["dw_w"], golden["dw_b"]),
                 golden["dw_out"], "dwconv k=9")
    assert_close(oracle.depthwise_conv1d(golden["dw5_x"], golden["dw5_w"], None),
                 golden["dw5_out"], "dwconv k=3 no bias")


@pytest.mark.parametrize("T", [1, 2, 3, 7])
def test_golden_relative_shift(oracle, golden, T):
    assert_bitexact(oracle.relative_shift(golden[f"rs{T}_bd"]), golden[f"rs{T}_out"], "rel_shift")


def test_golden_dequant(oracle, golden):
    assert_bitexact(oracle.dequant_i8(golden["i8_q"], float(golden["i8_scale"][0])),
                    golden["i8_out"], "int8")
    K, N = golden["i4_out"].shape
    assert_bitexact(oracle.dequant_i4(golden["i4_packed"], golden["i4_scales"], K, N, 32, 1),
                    golden["i4_out"], "int4")


def test_golden_requant(oracle, golden):
    sq, sk, sv, ms = (float(v) for v in golden["rq_scales"])
    fused, oms = oracle.requant_qkv_i8(golden["rq_q"], golden["rq_k"], golden["rq_v"], sq, sk, sv)
    assert np.float32(oms) == np.float32(ms)
    assert_bitexact(fused, golden["rq_fused"], "requant")


def test_int4_pack_roundtrip(oracle):
    """Exporter packing (extract_weights.py:589-594) then dequant gives q * scale."""
    rng = np.random.default_rng(5)
    for K, N, G, axis in ((8, 64, 32, 1), (256, 32, 128, 0), (3, 16, 2, 1)):
        q = rng.integers(-8, 8, size=(K, N)).astype(np.int8)
        packed = ((q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
        if axis == 1:
            sc = rng.uniform(1e-3, 2e-2, size=(K, N // G)).astype(np.float32)
            full = np.repeat(sc, G, axis=1)
        else:
            sc = rng.uniform(1e-3, 2e-2, size=(K // G, N)).astype(np.float32)
            full = np.repeat(sc, G, axis=0)
        assert_bitexact(oracle.dequant_i4(packed, sc, K, N, G, axis),
                        (q.astype(np.float32) * full).astype(np.float32), f"G={G} axis={axis}")


def _golden_block(golden):
    ps = {k: golden["blk_p_" + k] for k in po.PARAM_ROLES}
    si = {k: golden["blk_si_" + k] for k in po.STANDIN_ROLES}
    return ps, si, golden["blk_x"]


def test_golden_block(oracle, golden):
    ps, si, x = _golden_block(golden)
    xo, caps = oracle.conformer_block(x, ps, si)
    assert_close(xo, golden["blk_x_out"], "block x")
    for k in po.CAPTURE_ROLES:
        assert_close(caps[k], golden["blk_cap_" + k], "block " + k)


def _golden_pre(g):
    ps = {k: g["pre_p_" + k] for k in po.PRE_PARAM_ROLES}
    si = {k: g["pre_si_" + k] for k in ("y2", "y3", "proj")}
    return ps, si, g["pre_mel"]


def test_golden_pre_encode(oracle, golden):
    """Pre-encode subsampling + scaling (csrc/encoder.c:103-175, 578-593): every
    3x3 convolution, bias, ReLU, flatten and the sqrt(1024) scale bit for bit."""
    ps, si, mel = _golden_pre(golden)
    xo, caps = oracle.pre_encode(mel, ps, si)
    assert_bitexact(xo, golden["pre_x_out"], "pre x")
    for k in ("s2d", "s3d", "flat"):
        assert_bitexact(caps[k], golden["pre_cap_" + k], "pre " + k)


def test_golden_greedy_decode(oracle, golden):
    """The reference's own pk_greedy_decode (csrc/decoder.c:80-132) on 6 frames
    with stand-in products: tokens, joint evaluations, joint hidden rows bit
    for bit, LSTM state within the tolerance."""
    params = {k: golden["dec_p_" + k] for k in ("B0", "B1", "enc_b", "pred_b", "out_b")}
    embed = np.zeros((po.DEC_V, po.DEC_H), np.float32)
    embed[golden["dec_embed_rows"]] = golden["dec_embed"]
    params["embed"] = embed
    table = {k: golden["dec_t_" + k] for k in po.DEC_PRODUCTS}
    prod = po.DecodeProducts(table)
    tok, iters, _ = po.oracle_greedy_decode(6, params, prod)
    assert_bitexact(tok.astype(np.int32), golden["dec_tokens"], "tokens")
    assert iters == int(golden["dec_iters"][0])
    for k in range(iters):
        assert_bitexact(prod.inputs["out"][k], golden["dec_hidden"][k], f"hidden {k}")
        assert_close(prod.inputs["pred"][k], golden["dec_h1"][k], f"h1 {k}")


# ── the reference library at BASELINE shapes ─────────────────────────────────

def test_ref_layer_norm_T375(oracle, reference):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((375, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    b = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    assert_close(oracle.layer_norm_rows(x, g, b), reference.layer_norm_rows(x, g, b), "ln")
    assert_close(oracle.layer_norm_rows(x, g, b), reference.layer_norm_rows_inplace(x, g, b),
                 "ln inplace")


@pytest.mark.parametrize("T", [32, 375, 416])
def test_ref_softmax(oracle, reference, T):
    rng = np.random.default_rng(T)
    s = (3 * rng.standard_normal((8 * 16, T))).astype(np.float32)
    assert_close(oracle.softmax_rows(s), reference.softmax_rows(s), f"softmax T={T}")


def test_ref_requant_loader(oracle, reference):
    """Fused-QKV requant against the reference loader (csrc/weights.c:437-487)."""
    rng = np.random.default_rng(11)
    q, k, v = (rng.integers(-127, 128, size=(1024, 1024), dtype=np.int8) for _ in range(3))
    fused, scales = reference.load_fused_qkv_i8(q, k, v, 0.0031, 0.0092, 0.0092)
    mine, ms = oracle.requant_qkv_i8(q, k, v, *(float(s) for s in scales[:3]))
    assert np.float32(ms) == scales[3]
    assert_bitexact(mine, fused, "requant")


def test_ref_swish(oracle, reference):
    rng = np.random.default_rng(8)
    h = (4 * rng.standard_normal((375, 4096))).astype(np.float32)
    assert_close(oracle.swish(h), reference.swish(h), "swish")


def test_ref_dwconv(oracle, reference):
    rng = np.random.default_rng(9)
    for T in (1, 4, 8, 9, 375):
        x = rng.standard_normal((64, T)).astype(np.float32)
        w = (0.3 * rng.standard_normal((64, 9))).astype(np.float32)
        b = (0.1 * rng.standard_normal(64)).astype(np.float32)
        assert_close(oracle.depthwise_conv1d(x, w, b), reference.depthwise_conv1d(x, w, b),
                     f"dwconv T={T}")


@pytest.mark.parametrize("T", [1, 2, 32, 41])
def test_ref_block(oracle, reference, T):
    """The whole block: the reference's own conformer_block (GEMMs replaced by
    the same stand-ins) against the restatement, every GEMM input compared."""
    ps, si, x = po.random_block_inputs(np.random.default_rng(100 + T), T)
    xo, co = oracle.conformer_block(x, ps, si)
    xr, cr = reference.conformer_block(x, ps, si)
    assert_close(xo, xr, "x")
    for k in po.CAPTURE_ROLES:
        if k in ("Qu", "K", "Qv", "V", "P_h", "attn"):
            assert_bitexact(co[k], cr[k], k)
        else:
            assert_close(co[k], cr[k], k)


@pytest.mark.parametrize("T", [1, 2, 3, 4, 5, 8, 9, 33, 257, 3000])
def test_ref_pre_encode(oracle, reference, T):
    """The reference's own pre_encode_and_scale (its pk_conv2d, pk_relu, flatten
    and scaling; the 1x1 convolutions and projection as stand-ins) against the
    restatement: bit-exact, odd and even T, down to one mel frame."""
    ps, si, mel = po.random_pre_inputs(np.random.default_rng(300 + T), T)
    xo, co = oracle.pre_encode(mel, ps, si)
    xr, cr = reference.pre_encode(mel, ps, si)
    assert_bitexact(xo, xr, "x")
    for k in co:
        assert_bitexact(co[k], cr[k], k)


@pytest.mark.parametrize("T,p_blank", [(0, 0.5), (1, 0.5), (3, 1.0), (5, 0.0), (13, 0.6),
                                       (40, 0.8), (64, 0.9)])
def test_ref_greedy_decode(T, p_blank):
    """The reference's own pk_greedy_decode, pk_joint, pk_decoder_step and
    pk_lstm_step (matrix-vector products as stand-ins) against the
    restatement: same tokens and joint evaluations (the 10-symbol cap at
    p_blank 0, no symbol at 1), the same input for every product -- bit for
    bit for the embedding rows and joint hidden rows, within the tolerance for
    the LSTM states (glibc expf / tanhf under the reference's -ffast-math)."""
    if not po.ref_dec_available():
        pytest.skip("oracle/_ref/libpkref_dec.so not built (reference tree absent)")
    rng = np.random.default_rng(500 + T)
    params = po.random_dec_params(rng)
    table = po.random_dec_products(rng, T, p_blank)
    a, b = po.DecodeProducts(table), po.DecodeProducts(table)
    tok_o, it_o, _ = po.oracle_greedy_decode(T, params, a)
    tok_r, it_r = po.reference_greedy_decode(T, params, b)
    assert_bitexact(tok_o, tok_r, "tokens")
    assert it_o == it_r
    if p_blank == 0.0:
        assert len(tok_o) == 10 * T
    for g in po.DEC_PRODUCTS[1:]:
        assert sorted(a.inputs[g]) == sorted(b.inputs[g]), g
        for k in a.inputs[g]:
            if g in ("out", "l0_wi"):
                assert_bitexact(a.inputs[g][k], b.inputs[g][k], f"{g} {k}")
            else:
                assert_close(a.inputs[g][k], b.inputs[g][k], f"{g} {k}")


# ── known answers ────────────────────────────────────────────────────────────

@pytest.mark.parametrize("T", list(range(1, 71)))
def test_kat_relative_shift_closed_form(oracle, T):
    rng = np.random.default_rng(T)
    bd = rng.standard_normal((8, T, 2 * T - 1)).astype(np.float32)
    i, j = np.meshgrid(np.arange(T), np.arange(T), indexing="ij")
    assert_bitexact(oracle.relative_shift(bd), bd[:, i, T - 1 - i + j], f"T={T}")


def test_kat_argmax(oracle):
    nan = np.nan
    rows = np.array([
        [1, 3, 3, 2],          # tie -> first
        [nan, 5, 6, 7],        # NaN at 0 -> 0 (strict '>' against NaN)
        [1, nan, 0, 2],        # later NaN skipped
        [-np.inf, -np.inf, -np.inf, -np.inf],
        [0.0, -0.0, 0.0, -1],  # +0 == -0 -> first
        [-5, -4, -4, -9],
    ], np.float32)
    assert list(oracle.argmax_rows(rows)) == [1, 0, 3, 0, 0, 1]


def test_kat_int4_nibbles(oracle):
    # byte 0x8F: low nibble 0xF = -1 (column 0), high nibble 0x8 = -8 (column 1)
    packed = np.array([[0x8F, 0x71, 0x00, 0x07]], np.uint8)
    out = oracle.dequant_i4(packed, np.ones((1, 1), np.float32), 1, 8, 8, 1)
    assert list(out[0]) == [-1, -8, 1, 7, 0, 0, 7, 0]


def test_kat_requant(oracle):
    q = np.array([[127, -127, 3, -3, 1, 2, 0, 50]], np.int8)
    k = np.array([[127, -127, 3, -3, 1, 2, 0, 50]], np.int8)
    v = np.array([[127, -127, 3, -3, 1, 2, 0, 50]], np.int8)
    fused, ms = oracle.requant_qkv_i8(q, k, v, 0.5, 1.0, 0.25)
    assert ms == 1.0
    assert list(fused[0, 8:16]) == list(k[0])                      # s == ms: copied
    assert list(fused[0, :8]) == [64, -64, 2, -2, 1, 1, 0, 25]     # roundf half away from zero
    assert list(fused[0, 16:]) == [32, -32, 1, -1, 0, 1, 0, 13]


def test_kat_exp_poly_exact_points(oracle):
    # exp(0) = 1 exactly; the clamp saturates at +-87.
    assert oracle.exp_poly(0.0) == 1.0
    assert oracle.exp_poly(-1000.0) == oracle.exp_poly(-87.0)
    assert oracle.exp_poly(1000.0) == oracle.exp_poly(87.0)
    # degree-5 Taylor on |r| <= ln2/2: relative error below 2e-6 (r^6/720 at the edge)
    for x in (1.0, -3.5, 10.0, -20.25):
        assert abs(oracle.exp_poly(x) / np.exp(np.float64(x)) - 1) < 2e-6


def test_split3_bf16_properties():
    """The three-part bf16 split behind the split-operand GEMMs: the parts sum
    back to the fp32 value exactly, and the six kept part products of a
    1024-long product are within a few fp32 units of the float64 product
    (the three dropped ones are below 2^-23 of |a||w|)."""
    rng = np.random.default_rng(41)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    p0, p1, p2 = po.split3_bf16(x)
    back = (po.bf16_to_f32(p0).astype(np.float64) + po.bf16_to_f32(p1) + po.bf16_to_f32(p2))
    assert (back == x.astype(np.float64)).all()
    a = rng.standard_normal((64, 1024)).astype(np.float32)
    w = (rng.standard_normal((1024, 96)) / 32).astype(np.float32)
    exact = a.astype(np.float64) @ w.astype(np.float64)
    bound = np.abs(a).astype(np.float64) @ np.abs(w).astype(np.float64)
    err = np.abs(po.split_band_product(a, w) - exact) / bound
    assert err.max() < 2.0 ** -22, err.max()


def test_decode_restatement_matches_reference_with_weight_products():
    """The greedy-decode restatement against the reference's own
    pk_greedy_decode, both fed every product computed in float64 from the same
    seeded decoder weights (the oracle the fused decode is checked against):
    tokens and joint evaluations identical, on utterances that mix blanks,
    emissions and the 10-symbol cap."""
    if not po.ref_dec_available():
        pytest.skip("oracle/_ref/libpkref_dec.so not built (reference tree absent)")
    rng = np.random.default_rng(91)
    params = po.random_dec_params(rng)
    weights = po.random_dec_weights(rng)
    seen = set()
    for shift, T in ((3.5, 17), (3.5, 1), (0.0, 6), (8.0, 9)):
        p = dict(params)
        p["out_b"] = params["out_b"].copy()
        p["out_b"][po.DEC_BLANK] += shift
        enc = rng.standard_normal((T, po.DEC_H)).astype(np.float32)
        tok_o, it_o, _ = po.oracle_greedy_decode(T, p, po.WeightProducts(weights, enc, p["out_b"]))
        tok_r, it_r = po.reference_greedy_decode(T, p, po.WeightProducts(weights, enc, p["out_b"]))
        assert it_o == it_r and len(tok_o) == len(tok_r) and (tok_o == tok_r).all(), (shift, T)
        seen.add("cap" if len(tok_o) == 10 * T else "none" if len(tok_o) == 0 else "mixed")
    assert seen == {"cap", "none", "mixed"}, seen
