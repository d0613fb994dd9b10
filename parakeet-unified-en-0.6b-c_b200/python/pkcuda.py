"""ctypes binding of libpk_tensor_ops_cuda.so for Python callers (tests, bench).

The library is plain C (include/pkcuda.h); this module only marshals
arguments. Device buffers are torch CUDA tensors (torch is used for device
memory and streams only); every call goes through the C ABI and raises
PkCudaError on a non-zero status. There is no CPU fallback: if the shared
library is missing, loading fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libpk_tensor_ops_cuda.so")
CSRC_DIR = os.path.join(PKG_DIR, "csrc")

D, H, DH, FF = 1024, 8, 128, 4096
PKCU_CHANNEL_FIRST, PKCU_TIME_FIRST = 0, 1
PKCU_GROUP_ALONG_K, PKCU_GROUP_ALONG_N = 0, 1
PKCU_ACT_RELU, PKCU_ACT_TANH = 0, 1
PKCU_CHUNK_AUTO, PKCU_CHUNK_OFF, PKCU_CHUNK_ON = 0, 1, 2
PKCU_OK, PKCU_ERR_ARG, PKCU_ERR_CUDA, PKCU_ERR_NOMEM = 0, 1, 2, 3
PKCU_CHUNK_SIZE, PKCU_CHUNK_OVERLAP, PKCU_CHUNK_THRESHOLD = 400, 8, 500

# Symbols declared by include/pkcuda.h (checked by the CPU test suite).
EXPORTED = (
    "pkcu_status_string", "pkcu_last_error", "pkcu_version", "pkcu_selftest",
    "pkcu_wait_timeouts", "pkcu_selftest_wait",
    "pkcu_seq_create", "pkcu_seq_destroy", "pkcu_seq_n_items", "pkcu_seq_frames",
    "pkcu_seq_score_elems", "pkcu_seq_bd_elems", "pkcu_seq_pos_rows",
    "pk_layer_norm", "pk_layer_norm_rows", "pk_layer_norm_rows_inplace", "pk_swish", "pk_relu",
    "pk_softmax", "pk_softmax_rows", "pk_bias_add", "pk_depthwise_conv1d", "pk_cuda_status",
    "pk_softmax_rows_noalloc",
    "pkcu_layer_norm_rows", "pkcu_softmax_rows", "pkcu_swish", "pkcu_relu", "pkcu_bias_add_rows",
    "pkcu_depthwise_conv1d", "pkcu_bias_swish_rows", "pkcu_residual_add",
    "pkcu_residual_layer_norm", "pkcu_residual_layer_norm2", "pkcu_qkv_split_uv",
    "pkcu_pos_head_split", "pkcu_relative_shift", "pkcu_relpos_combine",
    "pkcu_relpos_combine_softmax", "pkcu_head_concat", "pkcu_layer_norm_transpose",
    "pkcu_residual_layer_norm_transpose", "pkcu_glu", "pkcu_dwconv_bn_swish",
    "pkcu_glu_dwconv_bn_swish",
    "pkcu_transpose_add", "pkcu_transpose_add_layer_norm", "pkcu_dequant_i8",
    "pkcu_requant_qkv_i8", "pkcu_dequant_i4", "pkcu_dequant_i4_qkv", "pkcu_joint_add_act",
    "pkcu_argmax_rows", "pkcu_encoder_nongemm", "pkcu_encoder_nongemm_launches",
    "pkcu_encoder_ws_create", "pkcu_encoder_ws_destroy", "pkcu_encoder_ws_device",
    "pkcu_encoder_ws_device_bytes", "pkcu_encoder_ws_h2d_bytes", "pkcu_encoder_ws_d2h_bytes",
    "pkcu_encoder_nongemm_host",
    "pkcu_weights_open", "pkcu_weights_upload", "pkcu_weights_destroy", "pkcu_weights_count",
    "pkcu_weights_name", "pkcu_weights_blocks", "pkcu_weights_find", "pkcu_weights_dequant",
    "pkcu_weights_fused_qkv", "pkcu_weights_block_params", "pkcu_weights_pre_params",
    "pkcu_pre_plan_create", "pkcu_pre_plan_destroy", "pkcu_pre_plan_p2", "pkcu_pre_plan_p3",
    "pkcu_pre_plan_frames", "pkcu_pre_plan_out_seq", "pkcu_pre_encode",
    "pkcu_decoder_create", "pkcu_decoder_destroy", "pkcu_decoder_buffers", "pkcu_greedy_decode",
    "pkcu_decoder_iterations", "pkcu_decoder_results",
    "pkcu_gemm_bias_swish", "pkcu_gemm_bias_residual",
    "pkcu_encoder_model_create", "pkcu_encoder_model_destroy", "pkcu_encoder_model_blocks",
    "pkcu_encoder_forward", "pkcu_asr_create", "pkcu_asr_destroy", "pkcu_asr_encoder_frames",
    "pkcu_asr_transcribe", "pkcu_asr_set_decode_mode", "pkcu_greedy_decode_graph",
    "pkcu_decoder_set_weights", "pkcu_greedy_decode_fused", "pkcu_asr_decode",
    "pkcu_should_chunk", "pkcu_chunk_bounds", "pkcu_chunk_plan_create", "pkcu_chunk_plan_destroy", "pkcu_chunk_plan_seq",
    "pkcu_chunk_plan_chunked", "pkcu_chunk_plan_items", "pkcu_chunk_plan_item", "pkcu_chunk_split",
    "pkcu_chunk_stitch", "pkcu_asr_encode", "pkcu_asr_set_chunk_mode",
    "pkcu_weight_create", "pkcu_weight_destroy", "pkcu_wmatmul_work_bytes", "pkcu_wmatmul",
    "pkcu_wmatmul_bias_swish", "pkcu_wmatmul_bias_residual", "pkcu_wmatmul_qkv",
    "pkcu_encoder_nongemm_fused", "pkcu_conv_weight_create", "pkcu_pointwise_conv1d",
    "pkcu_pointwise_conv1d_glu",
)


class PkCudaError(RuntimeError):
    pass


VP, I, LL, F = C.c_void_p, C.c_int, C.c_longlong, C.c_float

_SIGS = {
    "pkcu_status_string": (C.c_char_p, [I]),
    "pkcu_weights_open": (I, [C.c_char_p, C.c_char_p, C.POINTER(VP)]),
    "pkcu_weights_upload": (I, [VP, VP]),
    "pkcu_weights_destroy": (None, [VP]),
    "pkcu_weights_count": (I, [VP]),
    "pkcu_weights_name": (C.c_char_p, [VP, I]),
    "pkcu_weights_blocks": (I, [VP]),
    "pkcu_weights_find": (I, [VP, C.c_char_p, VP]),
    "pkcu_weights_dequant": (I, [VP, C.c_char_p, VP, VP]),
    "pkcu_weights_fused_qkv": (I, [VP, I, C.POINTER(VP), C.POINTER(I), C.POINTER(C.c_float),
                                   C.POINTER(VP)]),
    "pkcu_weights_block_params": (I, [VP, I, VP]),
    "pkcu_weights_pre_params": (I, [VP, VP]),
    "pkcu_pre_plan_create": (I, [C.POINTER(I), I, C.POINTER(VP)]),
    "pkcu_pre_plan_destroy": (None, [VP]),
    "pkcu_pre_plan_p2": (LL, [VP]),
    "pkcu_pre_plan_p3": (LL, [VP]),
    "pkcu_pre_plan_frames": (LL, [VP]),
    "pkcu_pre_plan_out_seq": (VP, [VP]),
    "pkcu_pre_encode": (I, [VP, VP, VP, VP, VP, VP, VP, VP, VP]),
    "pkcu_gemm_bias_swish": (I, [VP, VP, VP, VP, I, I, I, VP]),
    "pkcu_encoder_model_create": (I, [VP, VP, C.POINTER(VP)]),
    "pkcu_encoder_model_destroy": (None, [VP]),
    "pkcu_encoder_model_blocks": (I, [VP]),
    "pkcu_encoder_forward": (I, [VP, VP, VP, VP, VP, VP]),
    "pkcu_asr_create": (I, [VP, VP, C.POINTER(VP)]),
    "pkcu_asr_destroy": (None, [VP]),
    "pkcu_asr_encoder_frames": (I, [I]),
    "pkcu_asr_transcribe": (I, [VP, VP, C.POINTER(I), I, C.POINTER(I), C.POINTER(I), VP]),
    "pkcu_gemm_bias_residual": (I, [VP, VP, VP, VP, F, I, I, I, VP]),
    "pkcu_decoder_create": (I, [C.POINTER(I), I, C.POINTER(VP)]),
    "pkcu_decoder_destroy": (None, [VP]),
    "pkcu_decoder_buffers": (I, [VP, VP, VP]),
    "pkcu_greedy_decode": (I, [VP, VP, VP, VP, VP]),
    "pkcu_greedy_decode_graph": (I, [VP, VP, VP, VP, VP]),
    "pkcu_asr_set_decode_mode": (I, [VP, I]),
    "pkcu_asr_decode": (I, [VP, VP, C.POINTER(I), I, C.POINTER(I), C.POINTER(I), VP]),
    "pkcu_decoder_set_weights": (I, [VP, VP, VP]),
    "pkcu_greedy_decode_fused": (I, [VP, VP, VP]),
    "pkcu_decoder_iterations": (I, [VP]),
    "pkcu_decoder_results": (I, [VP, VP, VP, VP, VP]),
    "pkcu_last_error": (C.c_char_p, []),
    "pkcu_version": (C.c_char_p, []),
    "pkcu_selftest": (I, [C.POINTER(C.c_ulonglong)]),
    "pkcu_wait_timeouts": (I, [C.POINTER(C.c_uint), I]),
    "pkcu_selftest_wait": (I, [C.POINTER(C.c_int)]),
    "pkcu_seq_create": (I, [C.POINTER(I), I, C.POINTER(VP)]),
    "pkcu_seq_destroy": (None, [VP]),
    "pkcu_seq_n_items": (I, [VP]),
    "pkcu_seq_frames": (LL, [VP]),
    "pkcu_seq_score_elems": (LL, [VP]),
    "pkcu_seq_bd_elems": (LL, [VP]),
    "pkcu_seq_pos_rows": (LL, [VP]),
    "pk_layer_norm": (None, [VP, VP, VP, VP, I]),
    "pk_layer_norm_rows": (None, [VP, VP, VP, VP, I, I]),
    "pk_layer_norm_rows_inplace": (None, [VP, VP, VP, I, I]),
    "pk_swish": (None, [VP, I]),
    "pk_relu": (None, [VP, I]),
    "pk_softmax": (None, [VP, I]),
    "pk_softmax_rows": (None, [VP, I, I]),
    "pk_bias_add": (None, [VP, VP, I]),
    "pk_depthwise_conv1d": (None, [VP, VP, VP, VP, I, I, I]),
    "pk_cuda_status": (I, []),
    "pk_softmax_rows_noalloc": (I, [VP, I, I]),
    "pkcu_layer_norm_rows": (I, [VP, VP, VP, VP, I, I, VP]),
    "pkcu_softmax_rows": (I, [VP, I, I, VP]),
    "pkcu_swish": (I, [VP, LL, VP]),
    "pkcu_relu": (I, [VP, LL, VP]),
    "pkcu_bias_add_rows": (I, [VP, VP, I, I, VP]),
    "pkcu_depthwise_conv1d": (I, [VP, VP, VP, VP, I, I, I, VP]),
    "pkcu_bias_swish_rows": (I, [VP, VP, VP, I, I, VP]),
    "pkcu_residual_add": (I, [VP, VP, VP, F, I, I, VP]),
    "pkcu_residual_layer_norm": (I, [VP, VP, VP, F, VP, VP, VP, I, VP]),
    "pkcu_residual_layer_norm2": (I, [VP, VP, VP, F, VP, VP, VP, VP, VP, I, VP]),
    "pkcu_qkv_split_uv": (I, [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP]),
    "pkcu_pos_head_split": (I, [VP, VP, VP, VP]),
    "pkcu_relative_shift": (I, [VP, VP, VP, VP]),
    "pkcu_relpos_combine": (I, [VP, VP, VP, F, VP, VP]),
    "pkcu_relpos_combine_softmax": (I, [VP, VP, VP, F, VP, VP]),
    "pkcu_head_concat": (I, [VP, VP, VP, VP]),
    "pkcu_layer_norm_transpose": (I, [VP, VP, VP, VP, VP, VP]),
    "pkcu_residual_layer_norm_transpose": (I, [VP, VP, VP, F, VP, VP, VP, VP, VP]),
    "pkcu_glu": (I, [VP, VP, VP, I, I, VP, VP]),
    "pkcu_dwconv_bn_swish": (I, [VP, VP, VP, VP, F, I, VP, I, I, VP, VP]),
    "pkcu_glu_dwconv_bn_swish": (I, [VP, VP, VP, VP, VP, F, I, VP, I, I, VP, VP]),
    "pkcu_transpose_add": (I, [VP, VP, VP, VP, VP]),
    "pkcu_transpose_add_layer_norm": (I, [VP, VP, VP, VP, VP, VP, VP, VP]),
    "pkcu_dequant_i8": (I, [VP, F, VP, LL, VP]),
    "pkcu_requant_qkv_i8": (I, [VP, VP, VP, F, F, F, VP, C.POINTER(F), I, I, VP]),
    "pkcu_dequant_i4": (I, [VP, VP, VP, I, I, I, I, VP]),
    "pkcu_dequant_i4_qkv": (I, [VP, VP, VP, VP, VP, VP, VP, I, I, I, VP]),
    "pkcu_joint_add_act": (I, [VP, VP, VP, I, I, I, I, VP]),
    "pkcu_argmax_rows": (I, [VP, VP, LL, I, VP]),
    "pkcu_encoder_nongemm": (I, [VP, VP, I, VP, VP, VP, VP, VP, VP]),
    "pkcu_encoder_nongemm_fused": (I, [VP, VP, I, VP, VP, VP, VP, VP, C.c_uint, VP]),
    "pkcu_encoder_nongemm_launches": (I, [I]),
    "pkcu_encoder_ws_create": (I, [VP, I, C.POINTER(VP)]),
    "pkcu_encoder_ws_destroy": (None, [VP]),
    "pkcu_encoder_ws_device": (I, [VP, C.POINTER(VP), VP, VP]),
    "pkcu_encoder_ws_device_bytes": (LL, [VP]),
    "pkcu_encoder_ws_h2d_bytes": (LL, [VP]),
    "pkcu_encoder_ws_d2h_bytes": (LL, [VP]),
    "pkcu_encoder_nongemm_host": (I, [VP, VP, VP, VP, I, VP]),
    "pkcu_should_chunk": (I, [I, I]),
    "pkcu_chunk_bounds": (I, [I, I, I, VP, VP, VP, VP]),
    "pkcu_chunk_plan_create": (I, [C.POINTER(I), I, I, C.POINTER(VP)]),
    "pkcu_chunk_plan_destroy": (None, [VP]),
    "pkcu_chunk_plan_seq": (VP, [VP]),
    "pkcu_chunk_plan_chunked": (I, [VP]),
    "pkcu_chunk_plan_items": (I, [VP]),
    "pkcu_chunk_plan_item": (I, [VP, I, C.POINTER(I), C.POINTER(I), C.POINTER(I)]),
    "pkcu_chunk_split": (I, [VP, VP, VP, VP]),
    "pkcu_chunk_stitch": (I, [VP, VP, VP, VP]),
    "pkcu_asr_encode": (I, [VP, VP, C.POINTER(I), I, VP, VP]),
    "pkcu_asr_set_chunk_mode": (I, [VP, I]),
    "pkcu_weight_create": (I, [VP, I, F, VP, I, I, I, I, VP, C.POINTER(VP)]),
    "pkcu_weight_destroy": (None, [VP]),
    "pkcu_wmatmul_work_bytes": (LL, [I, I]),
    "pkcu_wmatmul": (I, [VP, VP, VP, I, F, F, VP, VP]),
    "pkcu_wmatmul_bias_swish": (I, [VP, VP, VP, VP, I, VP, VP]),
    "pkcu_wmatmul_bias_residual": (I, [VP, VP, VP, VP, F, I, VP, VP]),
    "pkcu_wmatmul_qkv": (I, [VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP]),
    "pkcu_conv_weight_create": (I, [VP, I, I, I, VP, C.POINTER(VP)]),
    "pkcu_pointwise_conv1d": (I, [VP, VP, VP, VP, I, VP, VP]),
    "pkcu_pointwise_conv1d_glu": (I, [VP, VP, VP, VP, I, VP, VP]),
}

_lib = None


def build(verbose: bool = False) -> str:
    """Compile the library in-tree (make in csrc/); returns the .so path."""
    out = subprocess.run(["make", "-C", CSRC_DIR, "-j8"], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("libpk_tensor_ops_cuda build failed:\n" + out.stdout + out.stderr)
    if verbose:
        print(out.stdout)
    return LIB_PATH


def lib():
    """The loaded shared library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise PkCudaError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().pkcu_last_error().decode()


def check(status: int, what: str = "") -> None:
    if status != 0:
        L = lib()
        raise PkCudaError(f"{what}: {L.pkcu_status_string(status).decode()}: "
                          f"{L.pkcu_last_error().decode()}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


# ── torch plumbing ────────────────────────────────────────────────────────────

def ptr(t) -> int | None:
    """Device address of a torch tensor (None for None)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class Seq:
    """A pkcu_seq batch descriptor (items of T_b frames)."""

    def __init__(self, lengths):
        self.lengths = [int(t) for t in lengths]
        arr = (I * len(self.lengths))(*self.lengths)
        h = VP()
        check(lib().pkcu_seq_create(arr, len(self.lengths), C.byref(h)), "pkcu_seq_create")
        self.handle = h

    @property
    def frames(self) -> int:
        return lib().pkcu_seq_frames(self.handle)

    @property
    def score_elems(self) -> int:
        return lib().pkcu_seq_score_elems(self.handle)

    @property
    def bd_elems(self) -> int:
        return lib().pkcu_seq_bd_elems(self.handle)

    @property
    def pos_rows(self) -> int:
        return lib().pkcu_seq_pos_rows(self.handle)

    def close(self):
        if self.handle:
            lib().pkcu_seq_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ── sequence driver structs ───────────────────────────────────────────────────

BLOCK_PARAM_FIELDS = ("norm_ff1_w", "norm_ff1_b", "ff1_b1", "ff1_b2", "norm_sa_w", "norm_sa_b",
                      "qkv_b", "pos_u", "pos_v", "out_b", "norm_conv_w", "norm_conv_b", "pw1_b",
                      "dw_w", "dw_b", "pw2_b", "norm_ff2_w", "norm_ff2_b", "ff2_b1", "ff2_b2",
                      "norm_out_w", "norm_out_b")
GEMM_OUT_FIELDS = ("ff1_h", "ff1_out", "qkv", "P", "ac", "bd", "attn_h", "att_out", "pw1", "pw2",
                   "ff2_h", "ff2_out")
GEMM_IN_FIELDS = ("ln_ff1", "h1", "ln_sa", "Qu", "K", "Qv", "P_h", "S", "V", "attn", "cf", "dw",
                  "ln_ff2", "h2", "gated")


class Weight:
    """pkcu_weight: a GEMM weight prepared for the tcgen05 weight products
    (bits 32: fp32 [K, N]; 8: int8 [K, N] with scale; 4: packed int4 [K, N/2]
    with group scales)."""

    def __init__(self, data, bits, K, N, scale=0.0, scales=None, group=32, axis=PKCU_GROUP_ALONG_N,
                 stream=None):
        h = VP()
        call("pkcu_weight_create", data if isinstance(data, int) else ptr(data), int(bits), float(scale),
             None if scales is None else (scales if isinstance(scales, int) else ptr(scales)), int(group),
             int(axis), int(K), int(N), stream_handle(stream), C.byref(h))
        self.handle, self.K, self.N = h, K, N

    def close(self):
        if self.handle:
            lib().pkcu_weight_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ConvWeight(Weight):
    """pkcu_weight of a pointwise convolution: fp32 W [Cout, Cin] as stored,
    glu=True for pkcu_pointwise_conv1d_glu."""

    def __init__(self, data, Cout, Cin, glu=False, stream=None):
        h = VP()
        call("pkcu_conv_weight_create", data if isinstance(data, int) else ptr(data), int(Cout), int(Cin),
             int(bool(glu)), stream_handle(stream), C.byref(h))
        self.handle, self.K, self.N = h, Cin, Cout


class ChunkPlan:
    """pkcu_chunk_plan: the chunk batch of the reference's chunked encoder."""

    def __init__(self, frames, mode=PKCU_CHUNK_AUTO):
        n = len(frames)
        arr = (I * n)(*[int(t) for t in frames])
        h = VP()
        check(lib().pkcu_chunk_plan_create(arr, n, int(mode), C.byref(h)), "pkcu_chunk_plan_create")
        self.handle = h
        L = lib()
        self.n_items = L.pkcu_chunk_plan_items(h)
        self.chunked = L.pkcu_chunk_plan_chunked(h)
        self.items = []
        for i in range(self.n_items):
            u, f0, nf = I(), I(), I()
            check(L.pkcu_chunk_plan_item(h, i, C.byref(u), C.byref(f0), C.byref(nf)), "pkcu_chunk_plan_item")
            self.items.append((u.value, f0.value, nf.value))
        self.seq_handle = L.pkcu_chunk_plan_seq(h)

    @property
    def lengths(self):
        return [nf for _, _, nf in self.items]

    def split(self, x, xc, stream=None):
        call("pkcu_chunk_split", self.handle, x if isinstance(x, int) else ptr(x),
             xc if isinstance(xc, int) else ptr(xc), stream_handle(stream))

    def stitch(self, xc, x, stream=None):
        call("pkcu_chunk_stitch", self.handle, xc if isinstance(xc, int) else ptr(xc),
             x if isinstance(x, int) else ptr(x), stream_handle(stream))

    def close(self):
        if self.handle:
            lib().pkcu_chunk_plan_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BlockParams(C.Structure):
    _fields_ = [(f, VP) for f in BLOCK_PARAM_FIELDS]


class GemmOutputs(C.Structure):
    _fields_ = [(f, VP) for f in GEMM_OUT_FIELDS]


class GemmInputs(C.Structure):
    _fields_ = [(f, VP) for f in GEMM_IN_FIELDS]


PKCU_DTYPE_F32, PKCU_DTYPE_I8, PKCU_DTYPE_I4 = 0, 1, 2


class Tensor(C.Structure):
    """pkcu_tensor: one manifest entry (include/pkcuda.h)."""
    _fields_ = [("dtype", I), ("ndim", I), ("shape", C.c_longlong * 4), ("numel", C.c_longlong),
                ("scale", C.c_float), ("n_scales", C.c_longlong), ("host", VP),
                ("host_scales", VP), ("dev", VP), ("dev_scales", VP)]

    @property
    def dims(self):
        return tuple(self.shape[d] for d in range(self.ndim))


class Weights:
    """A weights.bin / weights.json checkpoint (the reference's format):
    parsed on the host when opened, copied to the current device by upload()."""

    def __init__(self, bin_path, json_path):
        h = VP()
        check(lib().pkcu_weights_open(str(bin_path).encode(), str(json_path).encode(), C.byref(h)),
              "pkcu_weights_open")
        self.h = h

    def upload(self, stream=None):
        call("pkcu_weights_upload", self.h, stream)

    def names(self):
        L = lib()
        return [L.pkcu_weights_name(self.h, i).decode() for i in range(L.pkcu_weights_count(self.h))]

    def blocks(self) -> int:
        return lib().pkcu_weights_blocks(self.h)

    def find(self, name) -> Tensor:
        t = Tensor()
        call("pkcu_weights_find", self.h, name.encode(), C.byref(t))
        return t

    def dequant(self, name, out_ptr, stream=None):
        call("pkcu_weights_dequant", self.h, name.encode(), out_ptr, stream)

    def fused_qkv(self, block):
        w, b = VP(), VP()
        bits, scale = I(), C.c_float()
        call("pkcu_weights_fused_qkv", self.h, block, C.byref(w), C.byref(bits), C.byref(scale),
             C.byref(b))
        return w.value, bits.value, scale.value, b.value

    def block_params(self, block) -> "BlockParams":
        p = BlockParams()
        call("pkcu_weights_block_params", self.h, block, C.byref(p))
        return p

    def close(self):
        if self.h:
            lib().pkcu_weights_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def block_params_array(blocks):
    """blocks: list of {field: tensor} -> ctypes array of pkcu_block_params."""
    arr = (BlockParams * len(blocks))()
    for i, b in enumerate(blocks):
        for f in BLOCK_PARAM_FIELDS:
            setattr(arr[i], f, ptr(b[f]))
    return arr


def gemm_outputs(d) -> GemmOutputs:
    g = GemmOutputs()
    for f in GEMM_OUT_FIELDS:
        setattr(g, f, ptr(d[f]))
    return g


def gemm_inputs(d) -> GemmInputs:
    g = GemmInputs()
    for f in GEMM_IN_FIELDS:
        setattr(g, f, ptr(d[f]))
    return g


class EncoderWorkspace:
    """pkcu_encoder_ws: device buffers of one batch shape, n_groups pipeline groups."""

    def __init__(self, seq: Seq, n_groups: int):
        h = VP()
        check(lib().pkcu_encoder_ws_create(seq.handle, n_groups, C.byref(h)),
              "pkcu_encoder_ws_create")
        self.handle = h
        self.seq = seq

    def device(self):
        """(x address, GemmOutputs, GemmInputs) of the device buffers."""
        x = VP()
        go, gi = GemmOutputs(), GemmInputs()
        check(lib().pkcu_encoder_ws_device(self.handle, C.byref(x), C.byref(go), C.byref(gi)),
              "pkcu_encoder_ws_device")
        return x.value, go, gi

    @property
    def device_bytes(self) -> int:
        return lib().pkcu_encoder_ws_device_bytes(self.handle)

    @property
    def h2d_bytes(self) -> int:
        return lib().pkcu_encoder_ws_h2d_bytes(self.handle)

    @property
    def d2h_bytes(self) -> int:
        return lib().pkcu_encoder_ws_d2h_bytes(self.handle)

    def run_host(self, x_host_addr: int, gout_host: GemmOutputs, blocks_arr, n_blocks: int,
                 stream=None) -> None:
        call("pkcu_encoder_nongemm_host", self.handle, x_host_addr, C.cast(C.pointer(gout_host), VP),
             C.cast(blocks_arr, VP), n_blocks, stream_handle(stream))

    def close(self):
        if self.handle:
            lib().pkcu_encoder_ws_destroy(self.handle)
            self.handle = VP()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def encoder_nongemm(x, blocks_arr, n_blocks, gout: GemmOutputs, gin: GemmInputs, seq: Seq,
                    stream=None, hook=None) -> None:
    """hook: a GEMM_HOOK (called at every GEMM point of every block) or None."""
    call("pkcu_encoder_nongemm", x if isinstance(x, int) else ptr(x), C.cast(blocks_arr, VP), n_blocks,
         C.cast(C.pointer(gout), VP), C.cast(C.pointer(gin), VP), seq.handle,
         C.cast(hook, VP) if hook is not None else None, None, stream_handle(stream))


# ── pre-encode subsampling (pkcu_pre_encode) ────────────────────────────────
PRE_PARAM_FIELDS = ("conv0_w", "conv0_b", "conv2_w", "conv2_b", "conv3_b", "conv5_w", "conv5_b",
                    "conv6_b", "out_b")
PRE_GEMM_OUT_FIELDS = ("pw1", "pw2", "proj")
PRE_GEMM_IN_FIELDS = ("s2d", "s3d", "flat")
PKCU_GEMM_PRE_PW1, PKCU_GEMM_PRE_PW2, PKCU_GEMM_PRE_OUT = 16, 17, 18
GEMM_HOOK = C.CFUNCTYPE(I, VP, I, I, VP)


class PreParams(C.Structure):
    _fields_ = [(f, VP) for f in PRE_PARAM_FIELDS]


class PreGemmOutputs(C.Structure):
    _fields_ = [(f, VP) for f in PRE_GEMM_OUT_FIELDS]


class PreGemmInputs(C.Structure):
    _fields_ = [(f, VP) for f in PRE_GEMM_IN_FIELDS]


def _struct(cls, fields, d):
    s = cls()
    for f in fields:
        setattr(s, f, d[f] if isinstance(d[f], int) else ptr(d[f]))
    return s


class PrePlan:
    """pkcu_pre_plan: a batch of utterances of T_b mel frames each."""

    def __init__(self, mel_lengths):
        self.mel_lengths = [int(t) for t in mel_lengths]
        arr = (I * len(self.mel_lengths))(*self.mel_lengths)
        h = VP()
        check(lib().pkcu_pre_plan_create(arr, len(self.mel_lengths), C.byref(h)),
              "pkcu_pre_plan_create")
        self.handle = h

    @property
    def p2(self) -> int:
        return lib().pkcu_pre_plan_p2(self.handle)

    @property
    def p3(self) -> int:
        return lib().pkcu_pre_plan_p3(self.handle)

    @property
    def frames(self) -> int:
        return lib().pkcu_pre_plan_frames(self.handle)

    @property
    def out_seq(self) -> int:
        """Address of the plan's pkcu_seq of output frames (owned by the plan)."""
        return lib().pkcu_pre_plan_out_seq(self.handle)

    def close(self):
        if self.handle:
            lib().pkcu_pre_plan_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def pre_encode(mel, params, gout, gin, x, plan: PrePlan, hook=None, stream=None) -> None:
    """params / gout / gin: {field: tensor or address}; hook: a GEMM_HOOK or None."""
    p = _struct(PreParams, PRE_PARAM_FIELDS, params)
    go = _struct(PreGemmOutputs, PRE_GEMM_OUT_FIELDS, gout)
    gi = _struct(PreGemmInputs, PRE_GEMM_IN_FIELDS, gin)
    call("pkcu_pre_encode", mel if isinstance(mel, int) else ptr(mel), C.byref(p), C.byref(go),
         C.byref(gi), x if isinstance(x, int) else ptr(x), plan.handle,
         C.cast(hook, VP) if hook is not None else None, None, stream_handle(stream))


# ── batched greedy RNN-T decode (pkcu_greedy_decode) ────────────────────────
DEC_PARAM_FIELDS = ("embed", "lstm0_b", "lstm1_b", "joint_enc_b", "joint_pred_b", "joint_out_b")
DEC_OUT_FIELDS = ("enc", "pred", "out", "g0i", "g0r", "g1i", "g1r")
DEC_IN_FIELDS = ("x0", "h0", "h1", "hidden")
(PKCU_GEMM_DEC_ENC, PKCU_GEMM_DEC_L0_WI, PKCU_GEMM_DEC_L0_WR, PKCU_GEMM_DEC_L1_WI,
 PKCU_GEMM_DEC_L1_WR, PKCU_GEMM_DEC_PRED, PKCU_GEMM_DEC_OUT) = range(32, 39)


class DecParams(C.Structure):
    _fields_ = [(f, VP) for f in DEC_PARAM_FIELDS]


DEC_WEIGHT_FIELDS = ("lstm0_wi", "lstm0_wr", "lstm1_wi", "lstm1_wr", "joint_pred", "joint_out")


class DecWeights(C.Structure):
    _fields_ = [(f, VP) for f in DEC_WEIGHT_FIELDS]


class DecGemmOutputs(C.Structure):
    _fields_ = [(f, VP) for f in DEC_OUT_FIELDS]


class DecGemmInputs(C.Structure):
    _fields_ = [(f, VP) for f in DEC_IN_FIELDS]


class Decoder:
    """pkcu_decoder: device state for a batch of utterances of frames[b] frames."""

    def __init__(self, frames):
        self.frames = [int(t) for t in frames]
        arr = (I * len(self.frames))(*self.frames)
        h = VP()
        check(lib().pkcu_decoder_create(arr, len(self.frames), C.byref(h)), "pkcu_decoder_create")
        self.handle = h
        go, gi = DecGemmOutputs(), DecGemmInputs()
        call("pkcu_decoder_buffers", self.handle, C.byref(go), C.byref(gi))
        self.gemm_out = {f: getattr(go, f) for f in DEC_OUT_FIELDS}
        self.gemm_in = {f: getattr(gi, f) for f in DEC_IN_FIELDS}

    def decode(self, params, hook=None, stream=None, graph=False) -> None:
        """params: {field: tensor or address}; hook: a GEMM_HOOK or None;
        graph=True: pkcu_greedy_decode_graph (the hook must be capture-safe)."""
        p = _struct(DecParams, DEC_PARAM_FIELDS, params)
        call("pkcu_greedy_decode_graph" if graph else "pkcu_greedy_decode", self.handle,
             C.byref(p), C.cast(hook, VP) if hook is not None else None, None,
             stream_handle(stream))

    def set_weights(self, weights, stream=None) -> None:
        """weights: {field: tensor or address} over DEC_WEIGHT_FIELDS."""
        w = _struct(DecWeights, DEC_WEIGHT_FIELDS, weights)
        call("pkcu_decoder_set_weights", self.handle, C.byref(w), stream_handle(stream))

    def decode_fused(self, params, stream=None) -> None:
        p = _struct(DecParams, DEC_PARAM_FIELDS, params)
        call("pkcu_greedy_decode_fused", self.handle, C.byref(p), stream_handle(stream))

    @property
    def iterations(self) -> int:
        return lib().pkcu_decoder_iterations(self.handle)

    def results(self):
        """(n_tokens [B], evals [B], tokens per utterance as lists)."""
        import numpy as np
        B, F = len(self.frames), sum(self.frames)
        n = np.zeros(B, np.int32)
        ev = np.zeros(B, np.int32)
        tok = np.zeros(10 * F, np.int32)
        call("pkcu_decoder_results", self.handle, n.ctypes.data, ev.ctypes.data, tok.ctypes.data,
             None)
        off = np.concatenate([[0], np.cumsum(self.frames)]) * 10
        return n, ev, [tok[off[b]:off[b] + n[b]].copy() for b in range(B)]

    def close(self):
        if self.handle:
            lib().pkcu_decoder_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class EncoderModel:
    """pkcu_encoder_model: every block's GEMM weights of an uploaded checkpoint
    as fp32 device copies; forward() runs all blocks, GEMMs included."""

    def __init__(self, weights: "Weights", stream=None):
        h = VP()
        check(lib().pkcu_encoder_model_create(weights.h, stream_handle(stream), C.byref(h)),
              "pkcu_encoder_model_create")
        self.handle = h

    @property
    def blocks(self) -> int:
        return lib().pkcu_encoder_model_blocks(self.handle)

    def forward(self, x_addr: int, gout: GemmOutputs, gin: GemmInputs, seq: Seq, stream=None):
        call("pkcu_encoder_forward", self.handle, x_addr, C.byref(gout), C.byref(gin), seq.handle,
             stream_handle(stream))

    def close(self):
        if self.handle:
            lib().pkcu_encoder_model_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ASR:
    """pkcu_asr: mel spectrograms to tokens with the library's own GEMMs."""

    def __init__(self, weights: "Weights", stream=None):
        h = VP()
        check(lib().pkcu_asr_create(weights.h, stream_handle(stream), C.byref(h)), "pkcu_asr_create")
        self.handle = h

    DECODE_FUSED, DECODE_GRAPH, DECODE_EAGER, DECODE_TC = 0, 1, 2, 3

    def set_decode_mode(self, mode: int) -> None:
        call("pkcu_asr_set_decode_mode", self.handle, int(mode))

    def set_chunk_mode(self, mode: int) -> None:
        call("pkcu_asr_set_chunk_mode", self.handle, int(mode))

    def encode(self, mel, mel_frames, out, stream=None) -> None:
        """pk_encoder for a batch: out (device) receives the encoder outputs
        [sum encoder frames, 1024], utterance after utterance."""
        n = len(mel_frames)
        mf = (I * n)(*[int(t) for t in mel_frames])
        call("pkcu_asr_encode", self.handle, mel if isinstance(mel, int) else ptr(mel), mf, n,
             out if isinstance(out, int) else ptr(out), stream_handle(stream))

    def transcribe(self, mel, mel_frames, stream=None):
        """mel: device tensor of the spectrograms [128, T_b] one after another;
        returns one token array per utterance."""
        import numpy as np
        n = len(mel_frames)
        mf = (I * n)(*[int(t) for t in mel_frames])
        enc = [lib().pkcu_asr_encoder_frames(int(t)) for t in mel_frames]
        cap = 10 * sum(enc)
        tok = (I * cap)()
        cnt = (I * n)()
        call("pkcu_asr_transcribe", self.handle, mel if isinstance(mel, int) else ptr(mel), mf, n,
             tok, cnt, stream_handle(stream))
        t = np.frombuffer(tok, dtype=np.int32)
        off = np.concatenate([[0], np.cumsum(enc)]) * 10
        return [t[off[b]:off[b] + cnt[b]].copy() for b in range(n)]

    def decode(self, enc, enc_frames, stream=None):
        """enc: device tensor of the encoder outputs [T_b, 1024] one after
        another; returns one token array per utterance."""
        import numpy as np
        n = len(enc_frames)
        ef = (I * n)(*[int(t) for t in enc_frames])
        cap = 10 * sum(int(t) for t in enc_frames)
        tok = (I * cap)()
        cnt = (I * n)()
        call("pkcu_asr_decode", self.handle, enc if isinstance(enc, int) else ptr(enc), ef, n,
             tok, cnt, stream_handle(stream))
        t = np.frombuffer(tok, dtype=np.int32)
        off = np.concatenate([[0], np.cumsum([int(x) for x in enc_frames])]) * 10
        return [t[off[b]:off[b] + cnt[b]].copy() for b in range(n)]

    def close(self):
        if self.handle:
            lib().pkcu_asr_destroy(self.handle)
            self.handle = VP()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
