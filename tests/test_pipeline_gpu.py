"""End to end on the GPU against the reference engine: a complete checkpoint
in the reference's weights.bin / weights.json format (int8 projections, fp32
everything else; block 0's tensors aliased by blocks 1..23) and one mel
spectrogram of 200 frames.

Reference: oracle/_ref/libpkref_full.so, the whole reference engine with
nothing redirected -- pk_load_weights, pk_encoder (pre-encode, 24 conformer
blocks, its own int8 / fp32 GEMMs), pk_greedy_decode.

GPU: this library end to end -- pkcu_weights_open / _upload (fused int8 QKV
requantised on the device), pkcu_pre_encode, pkcu_encoder_nongemm over the 24
blocks, pkcu_greedy_decode -- with every GEMM of the model (1x1 convolutions
and projection of the pre-encode; FF, QKV, positional, score, context, output
and pointwise-conv products of each block; LSTM and joint products of the
decoder) done by torch in fp32 (TF32 off) at the library's GEMM hooks, on
weights the library dequantised.

Checked: the encoder output within 5e-5 absolute (24 blocks of fp32 GEMMs
summed in a different order than the reference's BLAS; every block ends in a
LayerNorm, so the difference does not grow with depth) and the decoded tokens
exactly.
"""
import contextlib
import ctypes as C
import subprocess
import sys

import numpy as np
import pytest

import pyoracle as po
import weights_fixture as wf
from gpuhelp import D, DH, FF, H, Layout, dev, empty, host

pytestmark = pytest.mark.gpu

MEL_T = 200


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    d = tmp_path_factory.mktemp("full_ckpt")
    tensors, bp, jp = wf.write_full_checkpoint(str(d), np.random.default_rng(5), enc_gain=1.0,
                                               blank_bias=0.0)
    mel = np.random.default_rng(6).standard_normal((128, MEL_T)).astype(np.float32)
    return tensors, bp, jp, mel


def reference_run(bp, jp, mel, tmp):
    """The reference engine in a fresh process (its loader keeps file-scope
    state between loads): (encoder output, tokens).

    Run with glibc's MALLOC_PERTURB_=255, which makes every allocation start
    zeroed: the reference's pk_lstm_step fills a freshly malloc'd gates buffer
    through cblas_sgemv with beta = 0, and that sgemv computes
    alpha * acc + beta * y (csrc/tensor_ops.c:601-606, csrc/blas.c:67), so NaN
    or Inf bytes left in the allocation poison the LSTM state and the tokens
    then depend on the process's heap history. Zeroed allocations give the
    result the code intends (beta = 0 overwrites)."""
    np.save(tmp / "mel.npy", mel)
    code = ("import sys, numpy as np; sys.path[:0] = sys.argv[1:3]; import pyoracle as po; "
            "e, t = po.reference_transcribe(sys.argv[3], sys.argv[4], np.load(sys.argv[5])); "
            "np.save(sys.argv[6], e); np.save(sys.argv[7], t)")
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    subprocess.run([sys.executable, "-c", code, os.path.join(root, "oracle"),
                    os.path.join(root, "tests"), bp, jp, str(tmp / "mel.npy"),
                    str(tmp / "enc.npy"), str(tmp / "tok.npy")], check=True,
                   capture_output=True, env={**os.environ, "MALLOC_PERTURB_": "255"})
    return np.load(tmp / "enc.npy"), np.load(tmp / "tok.npy")


class Engine:
    """GEMMs for every hook of the library, done with torch on the hook's
    stream from the library's own (dequantised) copies of the weights."""

    def __init__(self, cuda, w):
        import torch
        self.torch, self.cuda, self.w = torch, cuda, w
        self.cache = {}

    def weight(self, name, shape=None):
        """fp32 device copy of a checkpoint tensor (int8 dequantised)."""
        if name not in self.cache:
            t = self.w.find(name)
            out = self.torch.empty(t.numel, dtype=self.torch.float32, device="cuda")
            self.w.dequant(name, out.data_ptr())
            self.cache[name] = out.view(*(shape or t.dims))
        return self.cache[name]

    def fused_qkv(self, b):
        key = f"qkv{b}"
        if key not in self.cache:
            wp, bits, scale, _ = self.w.fused_qkv(b)
            assert bits == 8
            out = self.torch.empty(D * 3 * D, dtype=self.torch.float32, device="cuda")
            self.cuda.call("pkcu_dequant_i8", wp, C.c_float(scale), out.data_ptr(), D * 3 * D, None)
            self.cache[key] = out.view(D, 3 * D)
        return self.cache[key]

    def stream(self, s):
        t = self.torch
        return t.cuda.stream(t.cuda.ExternalStream(s)) if s else contextlib.nullcontext()


def view(ptr, *shape):
    import torch
    from gpuhelp import _DeviceView
    n = int(np.prod(shape))
    return torch.as_tensor(_DeviceView(ptr, n, np.float32), device="cuda").view(*shape)


def gpu_run(cuda, bp, jp, mel):
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return _gpu_run(cuda, bp, jp, mel)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def pre_encode_gpu(cuda, w, eng, mel):
    """pkcu_pre_encode with its three GEMMs done by torch: (x [T', 1024], T')."""
    plan = cuda.PrePlan([MEL_T])
    P2, P3, T = plan.p2, plan.p3, plan.frames
    pp = cuda.PreParams()
    cuda.call("pkcu_weights_pre_params", w.h, C.byref(pp))
    pre_out = {"pw1": empty(256 * P2), "pw2": empty(256 * P3), "proj": empty(T * D)}
    pre_in = {"s2d": empty(256 * P2), "s3d": empty(256 * P3), "flat": empty(T * 4096)}
    x = empty(T * D)

    def pre_hook(user, block, gemm, s):
        with eng.stream(s):
            if gemm == 16:
                view(pre_out["pw1"].data_ptr(), 256, P2).copy_(
                    eng.weight("pre_encode.conv.3.weight", (256, 256)) @ pre_in["s2d"].view(256, P2))
            elif gemm == 17:
                view(pre_out["pw2"].data_ptr(), 256, P3).copy_(
                    eng.weight("pre_encode.conv.6.weight", (256, 256)) @ pre_in["s3d"].view(256, P3))
            else:
                pre_out["proj"].view(T, D).copy_(
                    pre_in["flat"].view(T, 4096) @ eng.weight("pre_encode.out.weight"))
        return 0

    ph = cuda.GEMM_HOOK(pre_hook)
    cuda.pre_encode(dev(mel.reshape(-1)), {f: getattr(pp, f) for f in cuda.PRE_PARAM_FIELDS},
                    pre_out, pre_in, x, plan, hook=ph)
    plan.close()
    return x, T


def _gpu_run(cuda, bp, jp, mel):
    import torch
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        eng = Engine(cuda, w)
        x, T = pre_encode_gpu(cuda, w, eng, mel)
        # ── 24 conformer blocks ──
        L = Layout([T])
        shapes = po.standin_shapes(T)
        gout = {k: empty(int(np.prod(shapes[k]))) for k in po.STANDIN_ROLES}
        gin = {"ln_ff1": empty(T * D), "h1": empty(T * FF), "ln_sa": empty(T * D),
               "Qu": empty(T * D), "K": empty(T * D), "Qv": empty(T * D), "V": empty(T * D),
               "P_h": empty((2 * T - 1) * D), "S": empty(H * T * T), "attn": empty(T * D),
               "cf": empty(T * D), "dw": empty(T * D), "ln_ff2": empty(T * D),
               "h2": empty(T * FF), "gated": empty(T * D)}
        pe = eng.weight("pos_encoding.pe_table")[4999 - T + 1:4999 + T]

        def blk_hook(user, b, gemm, s):
            n = f"layers.{b}."
            with eng.stream(s):
                if gemm == 0:
                    gout["ff1_h"].view(T, FF).copy_(gin["ln_ff1"].view(T, D) @ eng.weight(n + "feed_forward1.linear1.weight"))
                elif gemm == 1:
                    gout["ff1_out"].view(T, D).copy_(gin["h1"].view(T, FF) @ eng.weight(n + "feed_forward1.linear2.weight"))
                elif gemm == 2:
                    gout["qkv"].view(T, 3 * D).copy_(gin["ln_sa"].view(T, D) @ eng.fused_qkv(b))
                elif gemm == 3:
                    gout["P"].view(2 * T - 1, D).copy_(pe @ eng.weight(n + "self_attn.linear_pos.weight"))
                elif gemm == 4:
                    gout["ac"].view(H, T, T).copy_(torch.bmm(gin["Qu"].view(H, T, DH),
                                                             gin["K"].view(H, T, DH).transpose(1, 2)))
                elif gemm == 5:
                    gout["bd"].view(H, T, 2 * T - 1).copy_(torch.bmm(
                        gin["Qv"].view(H, T, DH), gin["P_h"].view(H, 2 * T - 1, DH).transpose(1, 2)))
                elif gemm == 6:
                    gout["attn_h"].view(H, T, DH).copy_(torch.bmm(gin["S"].view(H, T, T),
                                                                  gin["V"].view(H, T, DH)))
                elif gemm == 7:
                    gout["att_out"].view(T, D).copy_(gin["attn"].view(T, D) @ eng.weight(n + "self_attn.linear_out.weight"))
                elif gemm == 8:
                    gout["pw1"].view(2 * D, T).copy_(eng.weight(n + "conv.pointwise_conv1.weight", (2 * D, D)) @ gin["cf"].view(D, T))
                elif gemm == 9:
                    gout["pw2"].view(D, T).copy_(eng.weight(n + "conv.pointwise_conv2.weight", (D, D)) @ gin["dw"].view(D, T))
                elif gemm == 10:
                    gout["ff2_h"].view(T, FF).copy_(gin["ln_ff2"].view(T, D) @ eng.weight(n + "feed_forward2.linear1.weight"))
                elif gemm == 11:
                    gout["ff2_out"].view(T, D).copy_(gin["h2"].view(T, FF) @ eng.weight(n + "feed_forward2.linear2.weight"))
            return 0

        bh = cuda.GEMM_HOOK(blk_hook)
        arr = (cuda.BlockParams * 24)(*[w.block_params(b) for b in range(24)])
        with cuda.Seq([T]) as seq:
            cuda.call("pkcu_encoder_nongemm", x.data_ptr(), C.cast(arr, cuda.VP), 24,
                      C.byref(cuda.gemm_outputs(gout)), C.byref(cuda.gemm_inputs(gin)), seq.handle,
                      C.cast(bh, cuda.VP), None, cuda.stream_handle())
        enc = host(x).reshape(T, D).copy()
        # ── greedy decode ──
        with cuda.Decoder([T]) as dec:
            go, gi = dec.gemm_out, dec.gemm_in
            Hd = 640

            def dec_hook(user, block, gemm, s):
                with eng.stream(s):
                    if gemm == 32:
                        view(go["enc"], T, Hd).copy_(x.view(T, D) @ eng.weight("joint.enc.weight"))
                    elif gemm in (33, 34, 35, 36):
                        l, kind = (0 if gemm < 35 else 1), ("W_i" if gemm in (33, 35) else "W_r")
                        src = gi["x0"] if gemm == 33 else (gi["h0"] if gemm in (34, 35) else gi["h1"])
                        dst = {33: "g0i", 34: "g0r", 35: "g1i", 36: "g1r"}[gemm]
                        Wm = eng.weight(f"decoder.lstm.{l}.{kind}", (4 * Hd, Hd))
                        view(go[dst], 1, 4 * Hd).copy_(view(src, 1, Hd) @ Wm.t())
                    elif gemm == 37:
                        view(go["pred"], 1, Hd).copy_(view(gi["h1"], 1, Hd) @ eng.weight("joint.pred.weight"))
                    else:
                        view(go["out"], 1, 1025).copy_(view(gi["hidden"], 1, Hd) @ eng.weight("joint.out.weight"))
                return 0

            dh = cuda.GEMM_HOOK(dec_hook)
            dp = {"embed": w.find("decoder.prediction.embed.weight").dev,
                  "lstm0_b": w.find("decoder.lstm.0.B").dev, "lstm1_b": w.find("decoder.lstm.1.B").dev,
                  "joint_enc_b": w.find("joint.enc.bias").dev, "joint_pred_b": w.find("joint.pred.bias").dev,
                  "joint_out_b": w.find("joint.joint_net.2.bias").dev}
            dec.decode(dp, hook=dh)
            n_tok, _, toks = dec.results()
    return enc, toks[0]


def test_pipeline_matches_reference_engine(cuda, model, tmp_path):
    if not po.ref_full_available():
        pytest.skip("oracle/_ref/libpkref_full.so not built (reference tree absent)")
    tensors, bp, jp, mel = model
    enc_ref, tok_ref = reference_run(bp, jp, mel, tmp_path)
    enc, tok = gpu_run(cuda, bp, jp, mel)
    assert enc.shape == enc_ref.shape
    err = np.abs(enc.astype(np.float64) - enc_ref).max()
    print(f"encoder output max |gpu - reference| = {err:.3e} (max |reference| "
          f"{np.abs(enc_ref).max():.3f}); {len(tok_ref)} tokens")
    assert err <= 5e-5, f"encoder output differs by {err:.3e}"
    assert len(tok) == len(tok_ref) and (tok == tok_ref).all(), (len(tok), len(tok_ref))


def _forward(cuda, bp, jp, mel):
    """pre-encode (torch GEMMs at the hooks) then pkcu_encoder_forward."""
    import torch
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with cuda.Weights(bp, jp) as w:
            w.upload(cuda.stream_handle())
            x, T = pre_encode_gpu(cuda, w, Engine(cuda, w), mel)
            with cuda.EncoderModel(w) as em, cuda.Seq([T]) as seq:
                assert em.blocks == 24
                ws = cuda.EncoderWorkspace(seq, 1)
                xa, gout, gin = ws.device()
                view(xa, T, D).copy_(x.view(T, D))
                em.forward(xa, gout, gin, seq)
                enc = host(view(xa, T, D)).copy()
                ws.close()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return enc


def test_encoder_forward_matches_reference_engine(cuda, model, tmp_path):
    """The encoder stack through pkcu_encoder_forward -- the library's own
    fp32-accurate GEMMs on the weights pkcu_encoder_model_create prepared from
    the uploaded checkpoint -- after pkcu_pre_encode, against the reference's
    pk_encoder on the same checkpoint and spectrogram. Twice: with the
    projections stored int8 (used as stored, q exact in bf16) and stored as
    float32 with the same values (split into three bf16 parts); the reference
    dequantises both to the same fp32 weights."""
    if not po.ref_full_available():
        pytest.skip("oracle/_ref/libpkref_full.so not built (reference tree absent)")
    tensors, bp, jp, mel = model
    enc_ref, _ = reference_run(bp, jp, mel, tmp_path)
    d = tmp_path / "fp32_ckpt"
    d.mkdir()
    _, bp32, jp32 = wf.write_full_checkpoint(str(d), np.random.default_rng(5), enc_gain=1.0,
                                             blank_bias=0.0, fp32_matrices=True)
    for what, (b, j) in (("int8 projections", (bp, jp)), ("fp32 projections", (bp32, jp32))):
        enc = _forward(cuda, b, j, mel)
        err = np.abs(enc.astype(np.float64) - enc_ref).max()
        print(f"pkcu_encoder_forward ({what}): max |gpu - reference| = {err:.3e}")
        assert err <= 5e-5, f"encoder output ({what}) differs by {err:.3e}"


def test_asr_transcribe_matches_reference_engine(cuda, model, tmp_path):
    """pkcu_asr_transcribe -- mel to tokens with every GEMM done by the library --
    on a ragged batch of two spectrograms (200 and 136 mel frames) against the
    reference engine run on each alone."""
    if not po.ref_full_available():
        pytest.skip("oracle/_ref/libpkref_full.so not built (reference tree absent)")
    tensors, bp, jp, mel = model
    mel2 = np.random.default_rng(8).standard_normal((128, 136)).astype(np.float32)
    want, enc = [], []
    for i, m in enumerate((mel, mel2)):
        d = tmp_path / f"u{i}"
        d.mkdir()
        e, t = reference_run(bp, jp, m, d)
        enc.append(e)
        want.append(t)
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        with cuda.ASR(w) as asr:
            mels = dev(np.concatenate([mel.reshape(-1), mel2.reshape(-1)]))
            frames = [mel.shape[1], mel2.shape[1]]
            got = []
            ref_enc = dev(np.concatenate([e.reshape(-1) for e in enc]))
            for mode in (asr.DECODE_FUSED, asr.DECODE_TC, asr.DECODE_GRAPH, asr.DECODE_EAGER):
                asr.set_decode_mode(mode)
                got.append(asr.transcribe(mels, frames))
                # the decode alone, on the reference's own encoder outputs
                got.append(asr.decode(ref_enc, [e.shape[0] for e in enc]))
            # other lengths replace the kept buffers and decoder, the first lengths again
            # rebuild them
            alone = asr.transcribe(dev(mel.reshape(-1)), [mel.shape[1]])
            again = asr.transcribe(mels, frames)
    assert len(alone) == 1 and (alone[0] == want[0]).all()
    got.append(again)
    for b in range(2):
        for g in got:
            assert len(g[b]) == len(want[b]) and (g[b] == want[b]).all(), \
                (b, len(g[b]), len(want[b]))


@pytest.mark.parametrize("frames", [[3000, 3000], [3000, 1999]], ids=["uniform", "ragged"])
def test_asr_encode_at_bench_length(cuda, model, tmp_path, frames):
    """pkcu_asr_encode at the bench's utterance length (3000 mel frames = 375
    encoder frames; all 24 blocks, every product on the library's tcgen05
    GEMM: the per-head products as one batched launch for a uniform batch, one
    per utterance for a ragged one) against the reference engine's pk_encoder
    on the first spectrogram."""
    if not po.ref_full_available():
        pytest.skip("oracle/_ref/libpkref_full.so not built (reference tree absent)")
    tensors, bp, jp, _ = model
    rng = np.random.default_rng(33)
    mels = [rng.standard_normal((128, f)).astype(np.float32) for f in frames]
    if frames[0] == frames[1]:
        mels[1] = mels[0]
    enc_ref, _ = reference_run(bp, jp, mels[0], tmp_path)
    ef = [cuda.lib().pkcu_asr_encoder_frames(f) for f in frames]
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        with cuda.ASR(w) as asr:
            out = empty(sum(ef) * D)
            asr.encode(dev(np.concatenate([m.reshape(-1) for m in mels])), frames, out)
            enc = host(out).reshape(-1, D)
    err = np.abs(enc[:ef[0]].astype(np.float64) - enc_ref).max()
    print(f"{frames}: max |gpu - reference| = {err:.3e} over {ef[0]} frames")
    assert err <= 5e-5, err
    if frames[0] == frames[1]:
        assert np.array_equal(enc[:ef[0]], enc[ef[0]:])
