"""CPU: the C ABI of libpk_tensor_ops_cuda.so (no kernel launches).

Checks that the built library loads, exports every function include/pkcuda.h
declares, and rejects bad arguments with PKCU_ERR_ARG before touching a GPU.
"""
import ctypes as C
import os
import re
import subprocess

import pytest

import pkcuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pkcuda.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(pk(?:cu)?_\w+)\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if not n.endswith("_t")))


@pytest.fixture(scope="module")
def L():
    if not os.path.exists(pkcuda.LIB_PATH):
        pkcuda.build()
    return pkcuda.lib()


def test_header_declares_expected_surface():
    names = header_functions()
    assert set(names) == set(pkcuda.EXPORTED), set(names) ^ set(pkcuda.EXPORTED)


def test_library_exports_every_header_symbol(L):
    out = subprocess.run(["nm", "-D", "--defined-only", pkcuda.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in header_functions() if n not in exported]
    assert not missing, missing


def test_dropin_prototypes_match_reference_header():
    """The drop-in block repeats csrc/parakeet.h:231-262 prototype for prototype."""
    src = open(HEADER).read()
    for proto in (
        "void pk_layer_norm(const float *x, const float *gamma, const float *beta_, float *out, int len);",
        "void pk_swish(float *x, int len);",
        "void pk_relu(float *x, int len);",
        "void pk_softmax(float *x, int len);",
        "void pk_softmax_rows(float *x, int n_rows, int len);",
        "void pk_bias_add(float *x, const float *b, int len);",
    ):
        assert proto in src, proto


def test_status_strings(L):
    assert L.pkcu_status_string(0) == b"ok"
    assert L.pkcu_status_string(1) == b"invalid argument"
    assert L.pkcu_status_string(2) == b"CUDA error"
    assert L.pkcu_version().decode().count(".") == 2
    assert L.pkcu_encoder_nongemm_launches(24) == 1 + 11 * 24


def test_argument_validation_without_gpu(L):
    ERR_ARG = 1
    assert L.pkcu_layer_norm_rows(None, None, None, None, 4, 1024, None) == ERR_ARG
    assert b"pkcu_layer_norm_rows" in L.pkcu_last_error()
    assert L.pkcu_softmax_rows(None, 1, 5, None) == ERR_ARG
    assert L.pkcu_swish(None, 5, None) == ERR_ARG
    assert L.pkcu_relu(None, 5, None) == ERR_ARG
    assert L.pkcu_depthwise_conv1d(None, None, None, None, 4, 4, 9, None) == ERR_ARG
    assert L.pkcu_dequant_i4(None, None, None, 4, 7, 32, 1, None) == ERR_ARG  # odd N
    assert L.pkcu_argmax_rows(None, None, 3, 1025, None) == ERR_ARG
    assert L.pkcu_joint_add_act(None, None, None, 1, 1, 640, 7, None) == ERR_ARG
    # misaligned pointer where 16-byte alignment is required
    assert L.pkcu_residual_layer_norm(3, 16, None, C.c_float(1.0), 16, 16, 16, 4, None) == ERR_ARG
    assert b"aligned" in L.pkcu_last_error()
    # NULL batch descriptor
    assert L.pkcu_qkv_split_uv(16, None, 16, 16, 16, 16, 16, 16, None, None) == ERR_ARG
    assert L.pkcu_encoder_nongemm(None, None, 1, None, None, None, None, None, None) == ERR_ARG


def test_requant_rejects_bad_scales(L):
    ms = C.c_float()
    assert L.pkcu_requant_qkv_i8(16, 16, 16, 0.0, 1.0, 1.0, 16, C.byref(ms), 4, 16, None) == 1


def test_seq_rejects_bad_lengths(L):
    h = C.c_void_p()
    arr = (C.c_int * 3)(5, 0, 7)
    assert L.pkcu_seq_create(arr, 3, C.byref(h)) == 1
    assert not h.value
    assert L.pkcu_seq_create(arr, 0, C.byref(h)) == 1


def test_uniform_seq_needs_no_device(L):
    """A uniform batch keeps no device arrays: its offsets are arithmetic."""
    h = C.c_void_p()
    arr = (C.c_int * 4)(375, 375, 375, 375)
    assert L.pkcu_seq_create(arr, 4, C.byref(h)) == 0
    assert L.pkcu_seq_frames(h) == 1500
    assert L.pkcu_seq_score_elems(h) == 4 * 8 * 375 * 375
    assert L.pkcu_seq_bd_elems(h) == 4 * 8 * 375 * 749
    assert L.pkcu_seq_pos_rows(h) == 4 * 749
    L.pkcu_seq_destroy(h)


def test_pre_plan_sizes_and_validation(L):
    """pkcu_pre_plan: output frames ceil(ceil(ceil(T/2)/2)/2) per utterance
    (csrc/encoder.c:116-152); a uniform batch keeps no device arrays."""
    h = C.c_void_p()
    arr = (C.c_int * 4)(3000, 3000, 3000, 3000)
    assert L.pkcu_pre_plan_create(arr, 4, C.byref(h)) == 0
    assert L.pkcu_pre_plan_frames(h) == 4 * 375
    assert L.pkcu_pre_plan_p2(h) == 4 * 32 * 750
    assert L.pkcu_pre_plan_p3(h) == 4 * 16 * 375
    assert L.pkcu_pre_plan_out_seq(h)
    L.pkcu_pre_plan_destroy(h)
    bad = (C.c_int * 2)(11, 0)
    h2 = C.c_void_p()
    assert L.pkcu_pre_plan_create(bad, 2, C.byref(h2)) == 1 and not h2.value
    assert L.pkcu_pre_plan_create(arr, 0, C.byref(h2)) == 1
    assert L.pkcu_pre_encode(None, None, None, None, None, None, None, None, None) == 1
    assert b"pkcu_pre_encode" in L.pkcu_last_error()


def test_decoder_validation(L):
    """pkcu_decoder_create / pkcu_greedy_decode reject bad arguments before any
    CUDA call (utterances need at least one frame)."""
    h = C.c_void_p()
    bad = (C.c_int * 3)(4, 0, 9)
    assert L.pkcu_decoder_create(bad, 3, C.byref(h)) == 1 and not h.value
    assert b"utterance 1" in L.pkcu_last_error()
    assert L.pkcu_decoder_create(bad, 0, C.byref(h)) == 1
    assert L.pkcu_greedy_decode(None, None, None, None, None) == 1
    assert L.pkcu_decoder_iterations(None) == -1


def test_gemm_validation(L):
    """The fused GEMMs reject NULL operands, N or K not a multiple of 4 and
    misaligned pointers before any CUDA call."""
    assert L.pkcu_gemm_bias_swish(None, 16, 16, 16, 4, 8, 8, None) == 1
    assert L.pkcu_gemm_bias_swish(16, 16, 16, 16, 4, 6, 8, None) == 1
    assert b"multiples of 4" in L.pkcu_last_error()
    assert L.pkcu_gemm_bias_residual(16, 16, 16, 20, C.c_float(0.5), 4, 8, 8, None) == 1
    assert b"aligned" in L.pkcu_last_error()


def test_fused_decode_argument_checks():
    """The fused-decode and ASR-decode entry points reject NULL handles before
    any CUDA call."""
    import ctypes as C
    import pkcuda
    ERR_ARG = 1   # PKCU_ERR_ARG
    L = pkcuda.lib()
    w = pkcuda.DecWeights()
    p = pkcuda.DecParams()
    assert L.pkcu_decoder_set_weights(None, C.byref(w), None) == ERR_ARG
    assert L.pkcu_greedy_decode_fused(None, C.byref(p), None) == ERR_ARG
    assert L.pkcu_greedy_decode_graph(None, C.byref(p), None, None, None) == ERR_ARG
    assert L.pkcu_asr_set_decode_mode(None, 0) == ERR_ARG
    frames = (C.c_int * 1)(8)
    tok = (C.c_int * 80)()
    cnt = (C.c_int * 1)()
    assert L.pkcu_asr_decode(None, None, frames, 1, tok, cnt, None) == ERR_ARG


def test_asr_encoder_frames_follow_the_pre_encode_convolutions():
    """pkcu_asr_encoder_frames (host arithmetic, no GPU) gives the frame count of
    the restatement's three stride-2 convolutions (kernel 3, padding 1) for
    every length up to 5000 mel frames."""
    import pkcuda
    import pyoracle as po
    L = pkcuda.lib()
    for T in range(1, 5001):
        assert L.pkcu_asr_encoder_frames(T) == po.pre_dims(T)["H3"], T
