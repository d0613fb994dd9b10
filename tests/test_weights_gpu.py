"""GPU: the checkpoint loader's device side (pkcu_weights_upload and its
views) on files in the reference's format.

  * every tensor dequantised on the device equals the file's values through
    the reference's formulas: float32 copied, int8 (float)q * scale with the
    scale the reference's parser reads, int4 (float)nibble * scale[k, col/32];
  * the fused QKV weight and bias of a block equal the reference loader's
    (pk_load_weights, csrc/weights.c:403-487) for int8 and float32 q/k/v, and
    the restatement of its int4 branch (:488-544) for int4 q/k/v;
  * the block parameters the loader hands out drive pkcu_encoder_nongemm to
    the same result as the restatement given the file's parameters."""
import ctypes as C

import numpy as np
import pytest

import pyoracle as po
import weights_fixture as wf
from conftest import assert_bitexact, assert_close
from gpuhelp import D, Layout, dev, empty, from_device, host

pytestmark = pytest.mark.gpu


def _ckpt(tmp_path_factory, tag, attn, ff, n_blocks, alias, seed):
    d = tmp_path_factory.mktemp(tag)
    tensors = wf.make_tensors(np.random.default_rng(seed), n_blocks, attn=attn, ff=ff)
    bp, jp, man = wf.write_checkpoint(str(d), tensors, alias_blocks=alias)
    return tensors, bp, jp, man


@pytest.fixture(scope="module")
def ckpt_i8(tmp_path_factory):
    return _ckpt(tmp_path_factory, "w_i8", "int8", "int4", 2, 24, 81)


def test_upload_dequantises_every_tensor(cuda, oracle, reference, ckpt_i8):
    tensors, bp, jp, man = ckpt_i8
    int8 = [n for n, e in man.items() if e["dtype"] == "int8"]
    parsed = dict(zip(int8, reference.manifest_scales(jp, int8)))
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        for name, e in man.items():
            if not name.startswith(("layers.0.", "layers.1.")):
                continue                             # aliases of block 0
            t = w.find(name)
            assert t.dev is not None and t.dev % 256 == 0, name
            src = tensors[name]["data"]
            if e["dtype"] == "int4":
                K, N = src.shape[0], 2 * src.shape[1]
                want = oracle.dequant_i4(src, tensors[name]["scales"], K, N, 32, 1)
            elif e["dtype"] == "int8":
                want = oracle.dequant_i8(src.reshape(-1), float(parsed[name])).reshape(src.shape)
            else:
                want = src
            out = empty(want.size)
            w.dequant(name, out.data_ptr(), cuda.stream_handle())
            assert_bitexact(host(out).reshape(want.shape), want, name)


def test_fused_qkv_int8_matches_reference_loader(cuda, reference, ckpt_i8):
    tensors, bp, jp, man = ckpt_i8
    ref_w, ref_s, ref_bits = reference.load_fused_qkv_file(bp, jp)
    assert ref_bits == 8
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        assert w.blocks() == 24
        for b in (0, 1, 23):                           # 23 aliases block 0's q, k, v
            wp, bits, scale, bias = w.fused_qkv(b)
            assert bits == 8
            got = from_device(wp, D * 3 * D, np.int8).reshape(D, 3 * D)
            src = b if b < 2 else 0
            if src == 0:
                assert_bitexact(got, ref_w, f"fused int8 block {b}")
                assert np.float32(scale) == ref_s[3]
            want_b = np.concatenate([tensors[f"layers.{src}.self_attn.linear_{m}.bias"]["data"]
                                     for m in wf.QKV])
            got_b = from_device(bias, 3 * D, np.float32)
            assert_bitexact(got_b, want_b, f"fused bias block {b}")


def test_fused_qkv_float32_matches_reference_loader(cuda, reference, tmp_path_factory):
    tensors, bp, jp, man = _ckpt(tmp_path_factory, "w_f32", "float32", "int8", 1, 24, 82)
    ref_w, ref_s, ref_bits = reference.load_fused_qkv_file(bp, jp)
    assert ref_bits == 32
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        wp, bits, scale, bias = w.fused_qkv(0)
        assert bits == 32 and scale == 0.0
        got = from_device(wp, D * 3 * D, np.float32).reshape(D, 3 * D)
        assert_bitexact(got, ref_w, "fused fp32")


def test_fused_qkv_int4_follows_the_int4_branch(cuda, oracle, tmp_path_factory):
    """The reference never reaches its int4 fused branch (int4 entries have
    scale 0, which its float32 test takes first), so the check is the
    restatement of that branch."""
    tensors, bp, jp, man = _ckpt(tmp_path_factory, "w_i4", "int4", "int4", 1, 0, 83)
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        wp, bits, scale, bias = w.fused_qkv(0)
        assert bits == 32
        got = from_device(wp, D * 3 * D, np.float32).reshape(D, 3 * D)
        p = [tensors[f"layers.0.self_attn.linear_{m}.weight"] for m in wf.QKV]
        want = oracle.dequant_i4_qkv(*[x["data"] for x in p], *[x["scales"] for x in p], D, D, 32)
        assert_bitexact(got, want, "fused int4")


def test_block_params_drive_the_encoder_sequence(cuda, oracle, ckpt_i8):
    """Block 1's parameters from the loader, one item of 41 frames through
    pkcu_encoder_nongemm, against the restatement given the file's values."""
    from test_encoder_gpu import batch_standins, gpu_inputs
    tensors, bp, jp, man = ckpt_i8
    T = 41
    _, si, x = po.random_block_inputs(np.random.default_rng(41), T)
    L = Layout([T])
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        arr = (cuda.BlockParams * 1)(w.block_params(1))
        gout = {k: dev(v) for k, v in batch_standins(L, [(si, x)]).items()}
        gin = gpu_inputs(L)
        xd = dev(x)
        with cuda.Seq([T]) as seq:
            cuda.encoder_nongemm(xd, arr, 1, cuda.gemm_outputs(gout), cuda.gemm_inputs(gin), seq)
            got = host(xd)
    want, _ = oracle.conformer_block(x, wf.block_params(tensors, 1), si)
    assert_close(got, want, "x after block 1")


def test_pre_params_drive_the_pre_encode_stage(cuda, oracle, ckpt_i8):
    """pkcu_weights_pre_params: the pre-encode parameters from the loader drive
    pkcu_pre_encode to the restatement's result given the file's values."""
    from test_preencode_gpu import make_items, run_gpu
    tensors = ckpt_i8[0]
    params = wf.pre_params(tensors)
    lengths = [37, 8]
    _, items = make_items(lengths, seed=12)
    with cuda.Weights(ckpt_i8[1], ckpt_i8[2]) as w:
        w.upload(cuda.stream_handle())
        pp = cuda.PreParams()
        cuda.call("pkcu_weights_pre_params", w.h, C.byref(pp))
        dev_params = {f: getattr(pp, f) for f in cuda.PRE_PARAM_FIELDS}
        L, got = run_gpu(cuda, lengths, dev_params, items, params_on_device=True)
    for i, (si, mel) in enumerate(items):
        xo, caps = oracle.pre_encode(mel, params, si)
        assert_bitexact(L.rows(got["x"], i, D), xo, f"x item {i}")
        assert_bitexact(L.plane(got["s2d"], i, 2), caps["s2d"], f"s2d item {i}")
