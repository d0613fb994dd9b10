"""Generate tests/golden/reference_vectors.npz from the reference's own code.

Runs the reference engine's compiled csrc/tensor_ops.c, blas.c and encoder.c
(oracle/_ref/libpkref.so, built by oracle/Makefile from the reference source
tree) on small seeded inputs and stores inputs and outputs. The fixture pins
this repository's CPU restatement (oracle/) and the CUDA kernels on machines
where the reference tree is not available.

    python tests/golden/make_golden.py      # needs oracle/_ref/libpkref.so

Seeds: numpy PCG64, one per case (listed below); inputs N(0,1) unless noted.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle as po  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_vectors.npz")


def main():
    R = po.Reference()
    L = R.L
    g = {}

    rng = np.random.default_rng(1001)  # LayerNorm
    x = rng.standard_normal((7, 1024)).astype(np.float32)
    gam = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    bet = (0.1 * rng.standard_normal(1024)).astype(np.float32)
    g["ln_x"], g["ln_g"], g["ln_b"] = x, gam, bet
    g["ln_out"] = R.layer_norm_rows(x, gam, bet)
    x37 = rng.standard_normal((3, 37)).astype(np.float32)
    g37 = (1 + 0.1 * rng.standard_normal(37)).astype(np.float32)
    b37 = (0.1 * rng.standard_normal(37)).astype(np.float32)
    g["ln37_x"], g["ln37_g"], g["ln37_b"] = x37, g37, b37
    g["ln37_out"] = R.layer_norm_rows(x37, g37, b37)

    rng = np.random.default_rng(1002)  # softmax, scale 3
    for name, shape in (("sm7", (16, 7)), ("sm375", (8, 375)), ("sm32", (8, 32))):
        s = (3 * rng.standard_normal(shape)).astype(np.float32)
        g[name + "_x"] = s
        g[name + "_out"] = R.softmax_rows(s)

    rng = np.random.default_rng(1003)  # swish / relu (scale 4, n = 1003: a 3-element tail)
    s = (4 * rng.standard_normal(1003)).astype(np.float32)
    g["swish_x"], g["swish_out"] = s, R.swish(s)
    r = s.copy()
    r[[0, 5, 1000, 1001]] = [np.nan, -0.0, np.nan, -0.0]  # vector body vs scalar tail semantics
    g["relu_x"], g["relu_out"] = r, R.relu(r)

    rng = np.random.default_rng(1004)  # depthwise conv
    xc = rng.standard_normal((16, 31)).astype(np.float32)
    w = (0.3 * rng.standard_normal((16, 9))).astype(np.float32)
    b = (0.1 * rng.standard_normal(16)).astype(np.float32)
    g["dw_x"], g["dw_w"], g["dw_b"] = xc, w, b
    g["dw_out"] = R.depthwise_conv1d(xc, w, b)
    # Odd K only: for even K the reference's interior loop [pad, T-pad) reads one
    # tap past the end of each channel row (csrc/tensor_ops.c:496-499, 518-523).
    xs = rng.standard_normal((8, 5)).astype(np.float32)
    ws = (0.3 * rng.standard_normal((8, 3))).astype(np.float32)
    g["dw5_x"], g["dw5_w"] = xs, ws
    g["dw5_out"] = R.depthwise_conv1d(xs, ws, None)

    rng = np.random.default_rng(1005)  # relative_shift
    for T in (1, 2, 3, 7):
        bd = rng.standard_normal((8, T, 2 * T - 1)).astype(np.float32)
        g[f"rs{T}_bd"], g[f"rs{T}_out"] = bd, R.relative_shift(bd)

    rng = np.random.default_rng(1006)  # int8 dequant through cblas_sgemm_qb with A = I
    K, N = 16, 48
    q = rng.integers(-127, 128, size=(K, N), dtype=np.int8)
    scale = np.float32(rng.uniform(1e-3, 1e-2))
    A = np.eye(K, dtype=np.float32)
    Cm = np.zeros((K, N), np.float32)
    L.cblas_sgemm_qb.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p, C.c_int,
                                 C.c_void_p, C.c_float, C.c_int, C.c_float, C.c_void_p, C.c_int]
    L.cblas_sgemm_qb(K, N, K, 1.0, A.ctypes.data, K, q.ctypes.data, scale, N, 0.0, Cm.ctypes.data, N)
    g["i8_q"], g["i8_scale"], g["i8_out"] = q, np.array([scale], np.float32), Cm

    rng = np.random.default_rng(1007)  # int4: packed with the exporter's format
    # (extract_weights.py:589-594: low nibble = even column). The reference's
    # AVX2 unpack (csrc/blas.c:812-831) mis-decodes odd columns, so the decode is
    # pinned by this round trip and the scalar formula of csrc/weights.c:505-515.
    K, N = 16, 64
    q4 = rng.integers(-8, 8, size=(K, N)).astype(np.int8)
    packed = ((q4[:, 0::2] & 0x0F) | ((q4[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
    sc = rng.uniform(1e-3, 2e-2, size=(K, N // 32)).astype(np.float32)
    g["i4_packed"], g["i4_scales"], g["i4_q"] = packed, sc, q4
    g["i4_out"] = (q4.astype(np.float32) * np.repeat(sc, 32, axis=1)).astype(np.float32)

    rng = np.random.default_rng(1009)  # fused-QKV int8 requant through pk_load_weights
    qkv = [rng.integers(-127, 128, size=(1024, 1024), dtype=np.int8) for _ in range(3)]
    fused, scales = R.load_fused_qkv_i8(*qkv, 0.004, 0.0075, 0.006)
    for nm, a in zip("qkv", qkv):
        g["rq_" + nm] = a[:16].copy()
    g["rq_scales"], g["rq_fused"] = scales, fused[:16].copy()

    rng = np.random.default_rng(1008)  # one conformer block, T = 9, all GEMM inputs captured
    T = 9
    ps, si, xb = po.random_block_inputs(rng, T)
    xo, caps = R.conformer_block(xb, ps, si)
    g["blk_x"], g["blk_x_out"] = xb, xo
    for k, v in ps.items():
        g["blk_p_" + k] = v
    for k, v in si.items():
        g["blk_si_" + k] = v
    for k, v in caps.items():
        g["blk_cap_" + k] = v

    rng = np.random.default_rng(1010)  # pre-encode subsampling + scaling, T = 11 mel frames
    # (H1 = 6, H2 = 3, T' = 2); the 1x1 convolutions and the projection are
    # stand-ins, their inputs captured.
    ps, si, mel = po.random_pre_inputs(rng, 11)
    xo, caps = R.pre_encode(mel, ps, si)
    g["pre_mel"], g["pre_x_out"] = mel, xo
    for k, v in ps.items():
        g["pre_p_" + k] = v
    for k, v in si.items():
        g["pre_si_" + k] = v
    for k, v in caps.items():
        g["pre_cap_" + k] = v

    rng = np.random.default_rng(1011)  # greedy RNN-T decode, T = 6 frames, p_blank 0.5
    # Values on a 1/64 grid keep the fixture compressible; only the embedding
    # rows the decode reads (blank + emitted tokens) and the product rows of
    # the iterations it ran are stored (the rest is zero / unused).
    def grid(a):
        return (np.round(a * 64) / 64).astype(np.float32)
    params = {k: grid(v) for k, v in po.random_dec_params(rng).items()}
    table = {k: grid(v) for k, v in po.random_dec_products(rng, 6, 0.5).items()}
    prod = po.DecodeProducts(table)
    tok, iters = po.reference_greedy_decode(6, params, prod)
    rows = np.unique(np.concatenate([[po.DEC_BLANK], tok])).astype(np.int32)
    g["dec_embed_rows"], g["dec_embed"] = rows, params["embed"][rows]
    for k in ("B0", "B1", "enc_b", "pred_b", "out_b"):
        g["dec_p_" + k] = params[k]
    for k, v in table.items():
        g["dec_t_" + k] = v if k == "enc" else v[:iters + 1]
    g["dec_tokens"], g["dec_iters"] = tok.astype(np.int32), np.array([iters], np.int32)
    g["dec_hidden"] = np.stack([prod.inputs["out"][k] for k in range(iters)])
    g["dec_h1"] = np.stack([prod.inputs["pred"][k] for k in range(iters)])

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {len(g)} arrays, {os.path.getsize(OUT) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
