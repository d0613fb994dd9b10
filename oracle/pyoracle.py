"""numpy front end for the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/liboracle.so`` (this repository's restatement of the
reference algorithms, ``pk_oracle.c`` / ``pk_oracle_weights.c``) and, when it
was built, ``oracle/_ref/libpkref.so`` (the reference's own tensor_ops.c,
blas.c, threadpool.c and encoder.c compiled from its source tree by
``oracle/Makefile``).  Only the test suite, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs import this module; the product path never does.

Array conventions: every function takes and returns C-contiguous numpy
arrays (float32 / int8 / uint8 / int32) and never modifies its inputs unless
its name ends in ``_`` (in place, as the reference function it mirrors).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_ORACLE = os.path.join(HERE, "liboracle.so")
LIB_REF = os.path.join(HERE, "_ref", "libpkref.so")
LIB_REF_DEC = os.path.join(HERE, "_ref", "libpkref_dec.so")
LIB_REF_FULL = os.path.join(HERE, "_ref", "libpkref_full.so")

D, H, DH, FF = 1024, 8, 128, 4096

# Stand-in GEMM outputs of one block, in the order ref_harness.c consumes them.
STANDIN_ROLES = ("ff1_h", "ff1_out", "qkv", "P", "ac", "bd", "attn_h", "att_out",
                 "pw1", "pw2", "ff2_h", "ff2_out")
# GEMM inputs one block produces (captured from the reference, produced by the oracle).
CAPTURE_ROLES = ("ln_ff1", "h1", "ln_sa", "Qu", "K", "Qv", "P_h", "S", "V", "attn",
                 "cf", "dw", "ln_ff2", "h2")
# Non-GEMM parameters of one block, in ref_harness.c fill_block order.
PARAM_ROLES = ("norm_ff1_w", "norm_ff1_b", "ff1_b1", "ff1_b2", "norm_sa_w", "norm_sa_b",
               "qkv_b", "pos_u", "pos_v", "out_b", "norm_conv_w", "norm_conv_b", "pw1_b",
               "dw_w", "dw_b", "pw2_b", "norm_ff2_w", "norm_ff2_b", "ff2_b1", "ff2_b2",
               "norm_out_w", "norm_out_b")

FP = C.POINTER(C.c_float)
I8P = C.POINTER(C.c_int8)
U8P = C.POINTER(C.c_uint8)
I32P = C.POINTER(C.c_int32)
FPP = C.POINTER(FP)


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (liboracle.so, and _ref/libpkref.so where the
    reference tree exists)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(FP)


def _ptr_array(arrs):
    arr = (FP * len(arrs))()
    for i, a in enumerate(arrs):
        arr[i] = _fp(a) if a is not None else FP()
    return arr


class _Lib:
    def __init__(self, path: str, sigs: dict):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        for name, (res, args) in sigs.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args


# Greedy RNN-T decode: the products it consumes, in the numbering of
# pk_oracle_decode.c / ref_dec_harness.c (OR_DEC_*).
DEC_H, DEC_V, DEC_BLANK = 640, 1025, 1024
DEC_PRODUCTS = ("enc", "pred", "out", "l0_wi", "l0_wr", "l1_wi", "l1_wr")
DEC_PARAM_ROLES = ("embed", "B0", "B1", "enc_b", "pred_b", "out_b")
DEC_GEMM_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_int, C.c_int, FP, C.c_int, FP, C.c_int)
_DEC_ARGS = [C.c_int, FP, FP, FP, FP, FP, FP, DEC_GEMM_FN, C.c_void_p, I32P, C.c_int]

_ORACLE_SIGS = {
    "or_greedy_decode": (C.c_int, _DEC_ARGS + [FP, I32P]),
    "or_pre_out_frames": (C.c_int, [C.c_int]),
    "or_pre_encode": (C.c_int, [FP, C.c_int, FPP, FP, FP, FP, FP, FP, FP, FP]),
    "or_exp_poly": (C.c_float, [C.c_float]),
    "or_layer_norm_rows": (None, [FP, FP, FP, FP, C.c_int, C.c_int]),
    "or_layer_norm_rows_inplace": (None, [FP, FP, FP, C.c_int, C.c_int]),
    "or_softmax_rows": (None, [FP, C.c_int, C.c_int]),
    "or_swish": (None, [FP, C.c_longlong]),
    "or_relu": (None, [FP, C.c_longlong]),
    "or_bias_add": (None, [FP, FP, C.c_int]),
    "or_depthwise_conv1d": (None, [FP, FP, FP, FP, C.c_int, C.c_int, C.c_int]),
    "or_relative_shift": (None, [FP, FP, C.c_int, C.c_int]),
    "or_relpos_combine": (None, [FP, FP, C.c_longlong, C.c_float]),
    "or_qkv_split_uv": (None, [FP, FP, FP, FP, FP, FP, FP, C.c_int]),
    "or_pos_head_split": (None, [FP, FP, C.c_int]),
    "or_head_concat": (None, [FP, FP, C.c_int]),
    "or_residual": (None, [FP, FP, C.c_float, C.c_longlong]),
    "or_transpose": (None, [FP, FP, C.c_int, C.c_int]),
    "or_pointwise_bias": (None, [FP, FP, C.c_int, C.c_int]),
    "or_glu_channel_first": (None, [FP, FP, C.c_int, C.c_int]),
    "or_glu_time_first": (None, [FP, FP, C.c_int, C.c_int]),
    "or_transpose_add": (None, [FP, FP, C.c_int, C.c_int]),
    "or_batch_norm": (None, [FP, FP, FP, FP, FP, C.c_float, C.c_int, C.c_int]),
    "or_conformer_block": (None, [FP, C.c_int, FPP, FPP, FPP]),
    "or_joint_add_act": (None, [FP, FP, FP, C.c_int, C.c_int, C.c_int, C.c_int]),
    "or_argmax_rows": (None, [FP, I32P, C.c_longlong, C.c_int]),
    "or_dequant_i8": (None, [I8P, C.c_float, FP, C.c_longlong]),
    "or_requant_qkv_i8": (C.c_float, [I8P, I8P, I8P, C.c_float, C.c_float, C.c_float,
                                      I8P, C.c_int, C.c_int]),
    "or_dequant_i4": (None, [U8P, FP, FP, C.c_int, C.c_int, C.c_int, C.c_int]),
    "or_dequant_i4_qkv": (None, [U8P, U8P, U8P, FP, FP, FP, FP, C.c_int, C.c_int, C.c_int]),
}

_REF_SIGS = {
    "pk_layer_norm": (None, [FP, FP, FP, FP, C.c_int]),
    "pk_layer_norm_rows": (None, [FP, FP, FP, FP, C.c_int, C.c_int]),
    "pk_layer_norm_rows_inplace": (None, [FP, FP, FP, C.c_int, C.c_int]),
    "pk_softmax": (None, [FP, C.c_int]),
    "pk_softmax_rows": (None, [FP, C.c_int, C.c_int]),
    "pk_swish": (None, [FP, C.c_int]),
    "pk_relu": (None, [FP, C.c_int]),
    "pk_bias_add": (None, [FP, FP, C.c_int]),
    "pk_depthwise_conv1d": (None, [FP, FP, FP, FP, C.c_int, C.c_int, C.c_int]),
    "pkref_relative_shift": (C.c_int, [FP, C.c_int, C.c_int]),
    "pkref_ws_floats": (C.c_size_t, [C.c_int]),
    "pkref_conformer_blocks": (C.c_int, [FP, C.c_int, C.c_int, FPP, FPP, FPP, C.c_int, FP]),
    "pkref_pool_threads": (C.c_int, []),
    "pkref_load_fused_qkv": (C.c_int, [C.c_char_p, C.c_char_p, C.c_void_p, C.c_size_t,
                                      FP, C.POINTER(C.c_int)]),
    "pkref_manifest_scales": (C.c_int, [C.c_char_p, C.POINTER(C.c_char_p), C.c_int, FP]),
    "pkref_pre_encode": (C.c_int, [FP, C.c_int, FPP, FP, FP, FP, FP, FP, FP, FP]),
    "pk_wmatmul": (None, [FP, C.c_void_p, FP, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float]),
    "pk_pointwise_conv1d": (None, [FP, FP, FP, FP, C.c_int, C.c_int, C.c_int]),
}


class RefWeight(C.Structure):
    """The reference's Weight (csrc/parakeet.h:52-57)."""
    _fields_ = [("data", C.c_void_p), ("scale", C.c_float), ("scales", FP), ("bits", C.c_int)]

_oracle = None
_ref = None
_ref_dec = None


def ref_dec_available() -> bool:
    return os.path.exists(LIB_REF_DEC)


def ref_dec_lib():
    global _ref_dec
    if _ref_dec is None:
        _ref_dec = _Lib(LIB_REF_DEC, {
            "pkref_greedy_decode": (C.c_int, _DEC_ARGS + [I32P]),
            "pkref_greedy_decode_static": (C.c_int, [C.c_int, FP, FP, FP, FP, FP, FP, FPP, I32P,
                                                     C.c_int, I32P])}).lib
    return _ref_dec


def oracle_lib():
    global _oracle
    if _oracle is None:
        _oracle = _Lib(LIB_ORACLE, _ORACLE_SIGS).lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(LIB_REF)


def ref_lib():
    global _ref
    if _ref is None:
        _ref = _Lib(LIB_REF, _REF_SIGS).lib
    return _ref


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ── restatement (liboracle.so) ────────────────────────────────────────────────

class Oracle:
    """The restatement, one method per reference op (csrc/ citations in pk_oracle.c)."""

    def __init__(self):
        self.L = oracle_lib()

    def exp_poly(self, x: float) -> float:
        return self.L.or_exp_poly(x)

    def layer_norm_rows(self, x, g, b):
        x, g, b = f32(x), f32(g), f32(b)
        out = np.empty_like(x)
        R, Dd = x.shape
        self.L.or_layer_norm_rows(_fp(x), _fp(g), _fp(b), _fp(out), R, Dd)
        return out

    def softmax_rows(self, x):
        y = f32(x).copy()
        self.L.or_softmax_rows(_fp(y), y.shape[0], y.shape[1])
        return y

    def swish(self, x):
        y = f32(x).copy()
        self.L.or_swish(_fp(y), y.size)
        return y

    def relu(self, x):
        y = f32(x).copy()
        self.L.or_relu(_fp(y), y.size)
        return y

    def bias_add_rows(self, x, b):
        y = f32(x).copy()
        b = f32(b)
        R = y.size // b.size
        flat = y.reshape(R, b.size)
        for r in range(R):
            self.L.or_bias_add(flat[r].ctypes.data_as(FP), _fp(b), b.size)
        return y

    def depthwise_conv1d(self, x, w, b):
        x, w = f32(x), f32(w)
        Cc, T = x.shape
        K = w.shape[1]
        out = np.empty_like(x)
        self.L.or_depthwise_conv1d(_fp(x), _fp(w), _fp(f32(b)) if b is not None else FP(),
                                   _fp(out), Cc, T, K)
        return out

    def relative_shift(self, bd):
        bd = f32(bd)
        Hh, T, L = bd.shape
        assert L == 2 * T - 1
        out = np.empty((Hh, T, T), np.float32)
        self.L.or_relative_shift(_fp(bd), _fp(out), Hh, T)
        return out

    def relpos_combine(self, ac, bd, scale):
        """S = (ac + relative_shift(bd)) * scale, ac [H,T,T], bd [H,T,2T-1]."""
        s = f32(ac).copy()
        bds = self.relative_shift(bd)
        self.L.or_relpos_combine(_fp(s), _fp(bds), s.size, scale)
        return s

    def qkv_split_uv(self, qkv, bqkv, u, v):
        """Bias add on each QKV row (pk_bias_add) then the head gather with u/v."""
        q = self.bias_add_rows(qkv, bqkv)
        T = q.shape[0]
        outs = [np.empty((H, T, DH), np.float32) for _ in range(4)]
        self.L.or_qkv_split_uv(_fp(q), _fp(f32(u)), _fp(f32(v)), *[_fp(o) for o in outs], T)
        return tuple(outs)

    def pos_head_split(self, P):
        P = f32(P)
        L = P.shape[0]
        out = np.empty((H, L, DH), np.float32)
        self.L.or_pos_head_split(_fp(P), _fp(out), L)
        return out

    def head_concat(self, attn_h):
        a = f32(attn_h)
        T = a.shape[1]
        out = np.empty((T, D), np.float32)
        self.L.or_head_concat(_fp(a), _fp(out), T)
        return out

    def residual(self, x, y, alpha):
        xx = f32(x).copy()
        self.L.or_residual(_fp(xx), _fp(f32(y)), alpha, xx.size)
        return xx

    def transpose(self, a):
        a = f32(a)
        r, c = a.shape
        out = np.empty((c, r), np.float32)
        self.L.or_transpose(_fp(a), _fp(out), r, c)
        return out

    def pointwise_bias(self, out, b):
        y = f32(out).copy()
        Cc, T = y.shape
        self.L.or_pointwise_bias(_fp(y), _fp(f32(b)), Cc, T)
        return y

    def glu_channel_first(self, pw1):
        p = f32(pw1)
        D2, T = p.shape
        out = np.empty((D2 // 2, T), np.float32)
        self.L.or_glu_channel_first(_fp(p), _fp(out), D2 // 2, T)
        return out

    def glu_time_first(self, x):
        p = f32(x)
        T, D2 = p.shape
        out = np.empty((T, D2 // 2), np.float32)
        self.L.or_glu_time_first(_fp(p), _fp(out), T, D2 // 2)
        return out

    def transpose_add(self, x, pw2):
        xx = f32(x).copy()
        T, Dd = xx.shape
        self.L.or_transpose_add(_fp(xx), _fp(f32(pw2)), T, Dd)
        return xx

    def batch_norm(self, y, mean, var, gamma, beta, eps=1e-5):
        yy = f32(y).copy()
        Cc, T = yy.shape
        self.L.or_batch_norm(_fp(yy), _fp(f32(mean)), _fp(f32(var)), _fp(f32(gamma)),
                             _fp(f32(beta)), eps, Cc, T)
        return yy

    def conformer_block(self, x, params: dict, standins: dict):
        """One block; returns (x_out, {capture role: GEMM input})."""
        T = x.shape[0]
        xx = f32(x).copy()
        L = 2 * T - 1
        shapes = capture_shapes(T)
        caps = {r: np.empty(shapes[r], np.float32) for r in CAPTURE_ROLES}
        p = _ptr_array([f32(params[r]) for r in PARAM_ROLES])
        s = _ptr_array([f32(standins[r]) for r in STANDIN_ROLES])
        o = _ptr_array([caps[r] for r in CAPTURE_ROLES])
        del L
        self.L.or_conformer_block(_fp(xx), T, p, s, o)
        return xx, caps

    def pre_encode(self, mel, params: dict, standins: dict):
        """Pre-encode subsampling + scaling of one utterance (mel [128, T]):
        returns (x [T', 1024], {s2d, s3d, flat}: the GEMM inputs)."""
        return _pre_call(self.L.or_pre_encode, mel, params, standins)

    def joint_add_act(self, enc, pred, act):
        enc, pred = f32(enc), f32(pred)
        B, T, J = enc.shape
        out = np.empty_like(enc)
        self.L.or_joint_add_act(_fp(enc), _fp(pred), _fp(out), B, T, J, act)
        return out

    def argmax_rows(self, logits):
        lg = f32(logits)
        R, V = lg.shape
        out = np.empty(R, np.int32)
        self.L.or_argmax_rows(_fp(lg), out.ctypes.data_as(I32P), R, V)
        return out

    def dequant_i8(self, q, scale):
        q = np.ascontiguousarray(q, np.int8)
        out = np.empty(q.shape, np.float32)
        self.L.or_dequant_i8(q.ctypes.data_as(I8P), scale, _fp(out), q.size)
        return out

    def requant_qkv_i8(self, q, k, v, sq, sk, sv):
        q, k, v = (np.ascontiguousarray(a, np.int8) for a in (q, k, v))
        K, Dd = q.shape
        fused = np.empty((K, 3 * Dd), np.int8)
        ms = self.L.or_requant_qkv_i8(q.ctypes.data_as(I8P), k.ctypes.data_as(I8P),
                                      v.ctypes.data_as(I8P), sq, sk, sv,
                                      fused.ctypes.data_as(I8P), K, Dd)
        return fused, ms

    def dequant_i4(self, packed, scales, K, N, group, axis):
        packed = np.ascontiguousarray(packed, np.uint8)
        out = np.empty((K, N), np.float32)
        self.L.or_dequant_i4(packed.ctypes.data_as(U8P), _fp(f32(scales)), _fp(out),
                             K, N, group, axis)
        return out

    def dequant_i4_qkv(self, pq, pk, pv, sq, sk, sv, K, Dd, group):
        ps = [np.ascontiguousarray(a, np.uint8) for a in (pq, pk, pv)]
        out = np.empty((K, 3 * Dd), np.float32)
        self.L.or_dequant_i4_qkv(*[a.ctypes.data_as(U8P) for a in ps],
                                 _fp(f32(sq)), _fp(f32(sk)), _fp(f32(sv)), _fp(out),
                                 K, Dd, group)
        return out


def capture_shapes(T: int) -> dict:
    L = 2 * T - 1
    return {"ln_ff1": (T, D), "h1": (T, FF), "ln_sa": (T, D), "Qu": (H, T, DH),
            "K": (H, T, DH), "Qv": (H, T, DH), "P_h": (H, L, DH), "S": (H, T, T),
            "V": (H, T, DH), "attn": (T, D), "cf": (D, T), "dw": (D, T),
            "ln_ff2": (T, D), "h2": (T, FF)}


def standin_shapes(T: int) -> dict:
    L = 2 * T - 1
    return {"ff1_h": (T, FF), "ff1_out": (T, D), "qkv": (T, 3 * D), "P": (L, D),
            "ac": (H, T, T), "bd": (H, T, L), "attn_h": (H, T, DH), "att_out": (T, D),
            "pw1": (2 * D, T), "pw2": (D, T), "ff2_h": (T, FF), "ff2_out": (T, D)}


PRE_PARAM_ROLES = ("conv0_w", "conv0_b", "conv2_w", "conv2_b", "conv3_b", "conv5_w",
                   "conv5_b", "conv6_b", "out_b")
PRE_C, PRE_MELS = 256, 128


def pre_dims(T: int) -> dict:
    """Heights and widths after each stride-2 stage for T mel frames."""
    h1 = (T + 2 - 3) // 2 + 1
    h2 = (h1 + 2 - 3) // 2 + 1
    h3 = (h2 + 2 - 3) // 2 + 1
    return {"H1": h1, "W1": 64, "H2": h2, "W2": 32, "H3": h3, "W3": 16}


def pre_param_shapes() -> dict:
    return {"conv0_w": (PRE_C, 1, 3, 3), "conv0_b": (PRE_C,), "conv2_w": (PRE_C, 1, 3, 3),
            "conv2_b": (PRE_C,), "conv3_b": (PRE_C,), "conv5_w": (PRE_C, 1, 3, 3),
            "conv5_b": (PRE_C,), "conv6_b": (PRE_C,), "out_b": (D,)}


def random_pre_inputs(rng, T: int):
    """Seeded pre-encode inputs: (params, stand-ins y2 / y3 / proj, mel [128, T])."""
    d = pre_dims(T)
    ps = {k: (0.3 * rng.standard_normal(s)).astype(np.float32) for k, s in pre_param_shapes().items()}
    si = {"y2": rng.standard_normal((PRE_C, d["H2"] * d["W2"])).astype(np.float32),
          "y3": rng.standard_normal((PRE_C, d["H3"] * d["W3"])).astype(np.float32),
          "proj": rng.standard_normal((d["H3"], D)).astype(np.float32)}
    mel = rng.standard_normal((PRE_MELS, T)).astype(np.float32)
    return ps, si, mel


def _pre_call(fn, mel, params, si):
    T = mel.shape[1]
    d = pre_dims(T)
    caps = {"s2d": np.empty((PRE_C, d["H2"] * d["W2"]), np.float32),
            "s3d": np.empty((PRE_C, d["H3"] * d["W3"]), np.float32),
            "flat": np.empty((d["H3"], PRE_C * d["W3"]), np.float32)}
    x = np.empty((d["H3"], D), np.float32)
    p = _ptr_array([f32(params[r]) for r in PRE_PARAM_ROLES])
    n = fn(_fp(f32(mel)), T, p, _fp(f32(si["y2"])), _fp(f32(si["y3"])), _fp(f32(si["proj"])),
           _fp(caps["s2d"]), _fp(caps["s3d"]), _fp(caps["flat"]), _fp(x))
    assert n == d["H3"], (n, d)
    return x, caps


def param_shapes() -> dict:
    return {"norm_ff1_w": (D,), "norm_ff1_b": (D,), "ff1_b1": (FF,), "ff1_b2": (D,),
            "norm_sa_w": (D,), "norm_sa_b": (D,), "qkv_b": (3 * D,), "pos_u": (H, DH),
            "pos_v": (H, DH), "out_b": (D,), "norm_conv_w": (D,), "norm_conv_b": (D,),
            "pw1_b": (2 * D,), "dw_w": (D, 9), "dw_b": (D,), "pw2_b": (D,),
            "norm_ff2_w": (D,), "norm_ff2_b": (D,), "ff2_b1": (FF,), "ff2_b2": (D,),
            "norm_out_w": (D,), "norm_out_b": (D,)}


def random_block_inputs(rng, T: int):
    """Seeded inputs of one block: (params, stand-in GEMM outputs, x).

    LayerNorm gammas ~ N(1, 0.1), depthwise weights ~ 0.3 N(0,1), other
    parameters ~ 0.1 N(0,1); stand-ins and x ~ N(0,1)."""
    ps = {}
    for k, s in param_shapes().items():
        if k.startswith("norm") and k.endswith("_w"):
            ps[k] = (1.0 + 0.1 * rng.standard_normal(s)).astype(np.float32)
        elif k == "dw_w":
            ps[k] = (0.3 * rng.standard_normal(s)).astype(np.float32)
        else:
            ps[k] = (0.1 * rng.standard_normal(s)).astype(np.float32)
    si = {k: rng.standard_normal(s).astype(np.float32) for k, s in standin_shapes(T).items()}
    x = rng.standard_normal((T, D)).astype(np.float32)
    return ps, si, x


# ── the reference's own compiled code (_ref/libpkref.so) ──────────────────────

class Reference:
    """Calls into the reference's compiled tensor_ops.c / encoder.c."""

    def __init__(self):
        self.L = ref_lib()

    def layer_norm_rows(self, x, g, b):
        x, g, b = f32(x), f32(g), f32(b)
        out = np.empty_like(x)
        self.L.pk_layer_norm_rows(_fp(x), _fp(g), _fp(b), _fp(out), x.shape[0], x.shape[1])
        return out

    def layer_norm_rows_inplace(self, x, g, b):
        y = f32(x).copy()
        self.L.pk_layer_norm_rows_inplace(_fp(y), _fp(f32(g)), _fp(f32(b)), y.shape[0],
                                          y.shape[1])
        return y

    def softmax_rows(self, x):
        y = f32(x).copy()
        self.L.pk_softmax_rows(_fp(y), y.shape[0], y.shape[1])
        return y

    def swish(self, x):
        y = f32(x).copy()
        self.L.pk_swish(_fp(y), y.size)
        return y

    def relu(self, x):
        y = f32(x).copy()
        self.L.pk_relu(_fp(y), y.size)
        return y

    def bias_add_rows(self, x, b):
        y = f32(x).copy()
        b = f32(b)
        flat = y.reshape(-1, b.size)
        for r in range(flat.shape[0]):
            self.L.pk_bias_add(flat[r].ctypes.data_as(FP), _fp(b), b.size)
        return y

    def depthwise_conv1d(self, x, w, b):
        x, w = f32(x), f32(w)
        Cc, T = x.shape
        out = np.empty_like(x)
        self.L.pk_depthwise_conv1d(_fp(x), _fp(w), _fp(f32(b)) if b is not None else FP(),
                                   _fp(out), Cc, T, w.shape[1])
        return out

    def relative_shift(self, bd):
        y = f32(bd).copy()
        Hh, T, L = y.shape
        assert self.L.pkref_relative_shift(_fp(y), Hh, T) == 0
        return y.reshape(-1)[: Hh * T * T].reshape(Hh, T, T).copy()

    def load_fused_qkv_i8(self, q, k, v, sq, sk, sv):
        """Writes a weights.bin / manifest holding int8 linear_{q,k,v} (and zero
        biases) for all 24 blocks (every block points at the same bytes), loads
        it with the reference's pk_load_weights and returns block 0's fused
        QKV (int8 [1024, 3072]) and (sq, sk, sv, ms) as the loader parsed them."""
        import json
        import tempfile
        q, k, v = (np.ascontiguousarray(a, np.int8) for a in (q, k, v))
        assert q.shape == (D, D) and k.shape == (D, D) and v.shape == (D, D)
        bias = np.zeros(D, np.float32)
        blob = q.tobytes() + k.tobytes() + v.tobytes() + bias.tobytes()
        man = {}
        for i in range(24):
            for j, (nm, s) in enumerate((("q", sq), ("k", sk), ("v", sv))):
                man[f"layers.{i}.self_attn.linear_{nm}.weight"] = {
                    "offset": j * D * D, "numel": D * D, "dtype": "int8",
                    "scale": float(np.float32(s))}
                man[f"layers.{i}.self_attn.linear_{nm}.bias"] = {
                    "offset": 3 * D * D, "numel": D, "dtype": "float32"}
        out = np.empty((D, 3 * D), np.int8)
        scales = np.zeros(4, np.float32)
        bits = C.c_int(0)
        with tempfile.TemporaryDirectory() as td:
            bp, jp = os.path.join(td, "weights.bin"), os.path.join(td, "weights.json")
            with open(bp, "wb") as f:
                f.write(blob)
            with open(jp, "w") as f:
                json.dump(man, f)
            rc = self.L.pkref_load_fused_qkv(bp.encode(), jp.encode(), out.ctypes.data,
                                             out.nbytes, _fp(scales), C.byref(bits))
        assert rc == 0 and bits.value == 8, (rc, bits.value)
        return out, scales

    def wmatmul(self, A, W, scale=None, alpha=1.0, beta=0.0, C_in=None):
        """A [M, K] x W [K, N] through the reference's pk_wmatmul
        (csrc/tensor_ops.c:50-61): an fp32 Weight, or with scale given an int8
        Weight (W int8 [K, N], per-tensor scale: cblas_sgemm_qb, dequantised
        while packing, csrc/blas.c:526-558, 759); C = alpha A W + beta C_in."""
        A = f32(A)
        M, K = A.shape
        N = W.shape[1]
        if scale is None:
            W = f32(W)
            w = RefWeight(W.ctypes.data, 0.0, FP(), 32)
        else:
            W = np.ascontiguousarray(W, np.int8)
            w = RefWeight(W.ctypes.data, float(scale), FP(), 8)
        out = np.zeros((M, N), np.float32) if C_in is None else f32(C_in).copy()
        self.L.pk_wmatmul(_fp(A), C.byref(w), _fp(out), M, N, K, float(alpha), float(beta))
        return out

    def pointwise_conv1d(self, x, w, b):
        """The reference's pk_pointwise_conv1d (csrc/tensor_ops.c:579-590):
        out [Cout, T] = w [Cout, Cin] x [Cin, T] (cblas_sgemm) + b[c]."""
        x, w = f32(x), f32(w)
        Cin, T = x.shape
        Cout = w.shape[0]
        out = np.empty((Cout, T), np.float32)
        self.L.pk_pointwise_conv1d(_fp(x), _fp(w), _fp(f32(b)) if b is not None else FP(), _fp(out),
                                   Cin, Cout, T)
        return out

    def ff_linear1(self, A, W, b):
        """feed_forward's first half (csrc/encoder.c:193-196): pk_wmatmul, the
        per-row pk_bias_add, pk_swish."""
        h = self.wmatmul(A, W)
        b = f32(b)
        for t in range(h.shape[0]):
            self.L.pk_bias_add(_fp(h[t]), _fp(b), h.shape[1])
        self.L.pk_swish(_fp(h), h.size)
        return h

    def linear_residual(self, x, A, W, b, scale):
        """pk_wmatmul + per-row pk_bias_add, then x + scale * out as
        feed_forward's macaron residual (scale 0.5, csrc/encoder.c:198-216: the
        AVX2 body is fma(out, 0.5, x)) or the attention residual (scale 1,
        :418-434: x + out)."""
        out = self.wmatmul(A, W)
        b = f32(b)
        for t in range(out.shape[0]):
            self.L.pk_bias_add(_fp(out[t]), _fp(b), out.shape[1])
        x = f32(x)
        if scale == 1.0:
            return (x + out).astype(np.float32)
        return (x.astype(np.float64) + np.float64(scale) * out.astype(np.float64)).astype(np.float32)

    def pre_encode(self, mel, params: dict, standins: dict):
        """The reference's own pre_encode_and_scale (csrc/encoder.c:103-175,
        578-593) with its 1x1 convolutions and projection as stand-ins."""
        return _pre_call(self.L.pkref_pre_encode, mel, params, standins)

    def manifest_scales(self, json_path, names):
        """The int8 scale the reference's manifest parser reads for each name."""
        arr = (C.c_char_p * len(names))(*[n.encode() for n in names])
        out = np.zeros(len(names), np.float32)
        n = self.L.pkref_manifest_scales(str(json_path).encode(), arr, len(names), _fp(out))
        assert n >= 0
        return out

    def load_fused_qkv_file(self, bin_path, json_path):
        """Loads a checkpoint with the reference's pk_load_weights; returns block
        0's fused QKV (int8 or fp32 [1024, 3072]), (sq, sk, sv, scale) and bits."""
        buf = np.empty(D * 3 * D * 4, np.uint8)
        scales = np.zeros(4, np.float32)
        bits = C.c_int(0)
        rc = self.L.pkref_load_fused_qkv(str(bin_path).encode(), str(json_path).encode(),
                                         buf.ctypes.data, buf.nbytes, _fp(scales), C.byref(bits))
        assert rc == 0, rc
        if bits.value == 8:
            return buf[:D * 3 * D].view(np.int8).reshape(D, 3 * D).copy(), scales, 8
        return buf.view(np.float32).reshape(D, 3 * D).copy(), scales, bits.value

    def conformer_block(self, x, params: dict, standins: dict):
        """The reference's conformer_block with GEMMs replaced by the stand-ins;
        returns (x_out, {capture role: GEMM input seen by the stand-in GEMM})."""
        T = x.shape[0]
        xx = f32(x).copy()
        shapes = capture_shapes(T)
        caps = {r: np.empty(shapes[r], np.float32) for r in CAPTURE_ROLES}
        p = _ptr_array([f32(params[r]) for r in PARAM_ROLES])
        s = _ptr_array([f32(standins[r]) for r in STANDIN_ROLES])
        o = _ptr_array([caps[r] for r in CAPTURE_ROLES])
        rc = self.L.pkref_conformer_blocks(_fp(xx), T, 1, p, s, o, 1, FP())
        assert rc == 0
        return xx, caps


# ── greedy RNN-T decode ─────────────────────────────────────────────────────

def random_dec_params(rng):
    """Seeded decoder parameters: embedding [1025, 640], LSTM biases B [5120]
    per layer, joint biases (enc, pred [640], out [1025])."""
    return {"embed": (0.5 * rng.standard_normal((DEC_V, DEC_H))).astype(np.float32),
            "B0": (0.1 * rng.standard_normal(8 * DEC_H)).astype(np.float32),
            "B1": (0.1 * rng.standard_normal(8 * DEC_H)).astype(np.float32),
            "enc_b": (0.1 * rng.standard_normal(DEC_H)).astype(np.float32),
            "pred_b": (0.1 * rng.standard_normal(DEC_H)).astype(np.float32),
            "out_b": (0.1 * rng.standard_normal(DEC_V)).astype(np.float32)}


def random_dec_products(rng, T: int, p_blank: float, max_iters: int | None = None):
    """Stand-in products for one utterance of T frames: enc [T, 640] and, per
    iteration, pred [640], out [1025] (the blank logit raised by 8 with
    probability p_blank, so that blank wins), l{0,1}_w{i,r} [2560]."""
    n = max_iters if max_iters is not None else 10 * T + 2
    out = rng.standard_normal((n, DEC_V)).astype(np.float32)
    out[rng.random(n) < p_blank, DEC_BLANK] += 8.0
    return {"enc": rng.standard_normal((max(T, 1), DEC_H)).astype(np.float32),
            "pred": rng.standard_normal((n, DEC_H)).astype(np.float32),
            "out": out,
            **{g: (0.5 * rng.standard_normal((n, 4 * DEC_H))).astype(np.float32)
               for g in ("l0_wi", "l0_wr", "l1_wi", "l1_wr")}}


class DecodeProducts:
    """Serves stand-in products to a decode (table[name][iter] -> row; enc by
    frame) and records the input each product was computed from
    (inputs[name][iter])."""

    def __init__(self, table: dict):
        self.table = {DEC_PRODUCTS.index(k): np.ascontiguousarray(v, np.float32)
                      for k, v in table.items()}
        self.inputs = {k: {} for k in DEC_PRODUCTS}
        self.fn = DEC_GEMM_FN(self._serve)

    def _serve(self, user, g, it, inp, n_in, out, n_out):
        row = self.table[g][it]
        assert row.size == n_out, (DEC_PRODUCTS[g], row.size, n_out)
        C.memmove(out, row.ctypes.data, 4 * n_out)
        if n_in:
            self.inputs[DEC_PRODUCTS[g]][it] = np.ctypeslib.as_array(inp, (n_in,)).copy()


def random_dec_weights(rng):
    """Seeded decoder weights in the reference's layouts: LSTM W_i, W_r
    [2560, 640] per layer, joint.pred [640, 640] and joint.out [640, 1025]
    as (in, out); entries N(0, 1/640)."""
    s = 1.0 / np.sqrt(DEC_H)
    m = lambda *shape: (s * rng.standard_normal(shape)).astype(np.float32)
    return {"lstm0_wi": m(4 * DEC_H, DEC_H), "lstm0_wr": m(4 * DEC_H, DEC_H),
            "lstm1_wi": m(4 * DEC_H, DEC_H), "lstm1_wr": m(4 * DEC_H, DEC_H),
            "joint_pred": m(DEC_H, DEC_H), "joint_out": m(DEC_H, DEC_V)}


class WeightProducts:
    """Serves every product of a decode computed from the decoder's weights
    (float64 accumulation, rounded once to fp32) and its input row, as the
    reference's cblas_sgemv calls would (csrc/decoder.c:20-27, 53-72); the
    encoder projection rows come from enc [T, 640] by frame. Records, per
    joint evaluation, the gap between the two largest logits (bias added)."""

    def __init__(self, weights: dict, enc, out_b):
        w = {k: np.asarray(v, np.float64) for k, v in weights.items()}
        self.mats = {DEC_PRODUCTS.index("l0_wi"): w["lstm0_wi"], DEC_PRODUCTS.index("l0_wr"): w["lstm0_wr"],
                     DEC_PRODUCTS.index("l1_wi"): w["lstm1_wi"], DEC_PRODUCTS.index("l1_wr"): w["lstm1_wr"],
                     DEC_PRODUCTS.index("pred"): w["joint_pred"].T, DEC_PRODUCTS.index("out"): w["joint_out"].T}
        self.enc = np.ascontiguousarray(enc, np.float32)
        self.out_b = np.asarray(out_b, np.float32)
        self.gaps = []
        self.fn = DEC_GEMM_FN(self._serve)

    def _serve(self, user, g, it, inp, n_in, out, n_out):
        if g == DEC_PRODUCTS.index("enc"):
            row = self.enc[it]
        else:
            x = np.ctypeslib.as_array(inp, (n_in,)).astype(np.float64)
            row = (self.mats[g] @ x).astype(np.float32)
            if g == DEC_PRODUCTS.index("out"):
                top = np.sort(row + self.out_b)[-2:]
                self.gaps.append(float(top[1] - top[0]))
        assert row.size == n_out
        row = np.ascontiguousarray(row, np.float32)
        C.memmove(out, row.ctypes.data, 4 * n_out)


def _dec_call(fn, T, params, products, extra):
    p = [f32(params[r]) for r in DEC_PARAM_ROLES]
    cap = 10 * T + 1
    tokens = np.zeros(cap, np.int32)
    n_iters = C.c_int(0)
    n = fn(T, *[_fp(a) for a in p], products.fn, None, tokens.ctypes.data_as(I32P), cap,
           *extra, C.byref(n_iters))
    assert n >= 0
    return tokens[:n].copy(), n_iters.value


def oracle_greedy_decode(T, params, products: DecodeProducts):
    """The restatement: (tokens, joint evaluations, final state [h0, h1, c0, c1])."""
    state = np.zeros(4 * DEC_H, np.float32)
    tok, it = _dec_call(oracle_lib().or_greedy_decode, T, params, products, [_fp(state)])
    return tok, it, state.reshape(4, DEC_H)


def reference_greedy_decode(T, params, products: DecodeProducts):
    """The reference's own pk_greedy_decode: (tokens, joint evaluations)."""
    return _dec_call(ref_dec_lib().pkref_greedy_decode, T, params, products, [])


def reference_greedy_decode_static(T, params, rows: dict):
    """The reference's pk_greedy_decode with fixed product rows served from C
    (rows["enc"] [T, 640], one row for each other product): the reference's own
    non-GEMM decode work with no Python in the loop. Returns (tokens, joint
    evaluations)."""
    p = [f32(params[r]) for r in DEC_PARAM_ROLES]
    rr = [f32(rows[k]) for k in DEC_PRODUCTS]
    cap = 10 * T + 1
    tokens = np.zeros(cap, np.int32)
    n_iters = C.c_int(0)
    n = ref_dec_lib().pkref_greedy_decode_static(T, *[_fp(a) for a in p], _ptr_array(rr),
                                                 tokens.ctypes.data_as(I32P), cap,
                                                 C.byref(n_iters))
    assert n >= 0
    return tokens[:n].copy(), n_iters.value


# ── the reference engine end to end (oracle/_ref/libpkref_full.so) ──────────

def ref_full_available() -> bool:
    return os.path.exists(LIB_REF_FULL)


_ref_full = None


def reference_transcribe(bin_path, json_path, mel):
    """pk_load_weights + pk_encoder + pk_greedy_decode of the reference on one
    mel spectrogram [128, T]: (encoder output [T', 1024], tokens). The
    reference's decode reads uninitialised heap memory through a beta = 0
    sgemv (pk_lstm_step): run it in a process started with
    MALLOC_PERTURB_=255 for a result that does not depend on heap history."""
    global _ref_full
    if _ref_full is None:
        _ref_full = _Lib(LIB_REF_FULL, {"pkref_transcribe": (
            C.c_int, [C.c_char_p, C.c_char_p, FP, C.c_int, FP, C.c_longlong, I32P, C.c_int,
                      I32P])}).lib
    mel = f32(mel)
    T = mel.shape[1]
    Tp = T // 8 + 4
    enc = np.zeros((Tp, D), np.float32)
    tok = np.zeros(10 * Tp + 1, np.int32)
    nt = C.c_int(0)
    got = _ref_full.pkref_transcribe(str(bin_path).encode(), str(json_path).encode(), _fp(mel), T,
                                     _fp(enc), enc.size, tok.ctypes.data_as(I32P), tok.size,
                                     C.byref(nt))
    assert got > 0, "reference failed to load the checkpoint"
    return enc[:got].copy(), tok[:nt.value].copy()


# ── fp32 operands as three bf16 parts (the library's split-operand GEMMs) ────

def bf16_rn(x):
    """float32 -> bfloat16 bits (uint16), round to nearest, ties to even (the
    conversion the split kernels use; values here are finite)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def split3_bf16(x):
    """x = x0 + x1 + x2 with x0 = bf16(x), x1 = bf16(x - x0), x2 =
    bf16(x - x0 - x1), each difference exact in fp32 (the parts as uint16
    bits, in that order)."""
    x = np.ascontiguousarray(x, np.float32)
    p0 = bf16_rn(x)
    r1 = (x - bf16_to_f32(p0)).astype(np.float32)
    p1 = bf16_rn(r1)
    r2 = (r1 - bf16_to_f32(p1)).astype(np.float32)
    return p0, p1, bf16_rn(r2)


def split_band_product(a, w):
    """A [M, K] x W [K, N] from the six part products with i + j <= 2, each
    band summed on its own and the bands added smallest first (float64
    accumulation: the arithmetic the split GEMMs approximate)."""
    pa = [bf16_to_f32(p).astype(np.float64) for p in split3_bf16(a)]
    pw = [bf16_to_f32(p).astype(np.float64) for p in split3_bf16(w)]
    band = lambda k: sum(pa[i] @ pw[k - i] for i in range(k + 1))
    return (band(2) + band(1)) + band(0)
