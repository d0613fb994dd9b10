"""GPU: long audio through the chunked encoder (csrc/encoder.c:514-575,
597-633).

* The chunk plan's split and stitch (pkcu_chunk_split / pkcu_chunk_stitch)
  against the chunk bounds: every chunk item holds its utterance's input
  frames, and stitch takes each frame from the chunk that owns it.
* pkcu_asr_encode and pkcu_asr_transcribe on a ragged batch of a long
  spectrogram (4,104 mel frames -> 513 encoder frames, above the 500-frame
  threshold: chunks of 408 and 121 input frames) and a short one, against the
  reference engine's own pk_encoder + pk_greedy_decode run on each alone
  (oracle/_ref/libpkref_full.so): encoder output within the end-to-end bound
  and identical tokens."""
import numpy as np
import pytest

import pyoracle as po
import weights_fixture as wf
from conftest import assert_bitexact
from gpuhelp import D, dev, empty, host
from test_pipeline_gpu import reference_run

pytestmark = pytest.mark.gpu


def test_split_stitch_follow_the_chunk_bounds(cuda, monkeypatch):
    monkeypatch.delenv("PK_CHUNK", raising=False)
    frames = [1201, 375, 900, 501, 500]
    x = np.random.default_rng(3).standard_normal((sum(frames), D)).astype(np.float32)
    with cuda.ChunkPlan(frames) as plan:
        assert plan.chunked == 3        # 1201, 900 and 501 frames exceed 500
        assert plan.lengths == [408, 416, 409, 9, 375, 408, 416, 108, 408, 109, 500]
        xd = dev(x)
        xc = empty(sum(plan.lengths) * D)
        plan.split(xd, xc)
        got = host(xc).reshape(-1, D)
        base = np.concatenate([[0], np.cumsum(frames)])
        row = 0
        for u, f0, nf in plan.items:
            assert_bitexact(got[row:row + nf], x[base[u] + f0:base[u] + f0 + nf], f"chunk at row {row}")
            row += nf
        # stitch: the owned centre of each chunk; mark every chunk row with its item
        mark = np.concatenate([np.full((nf, D), i, np.float32) for i, (_, _, nf) in enumerate(plan.items)])
        back = empty(sum(frames) * D)
        plan.stitch(dev(mark), back)
        owner = host(back).reshape(-1, D)[:, 0]
        for u, T in enumerate(frames):
            items = [i for i, it in enumerate(plan.items) if it[0] == u]
            want = np.concatenate([np.full(min(400, T - 400 * k), i) for k, i in enumerate(items)]) \
                if len(items) > 1 else np.full(T, items[0])
            assert (owner[base[u]:base[u + 1]] == want).all(), u
        # round trip of the real data
        plan.stitch(xc, back)
        assert_bitexact(host(back).reshape(-1, D), x, "split then stitch")


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    d = tmp_path_factory.mktemp("chunk_ckpt")
    _, bp, jp = wf.write_full_checkpoint(str(d), np.random.default_rng(5), enc_gain=1.0, blank_bias=0.0)
    return bp, jp


def test_long_audio_matches_reference_engine(cuda, checkpoint, tmp_path, monkeypatch):
    if not po.ref_full_available():
        pytest.skip("oracle/_ref/libpkref_full.so not built (reference tree absent)")
    monkeypatch.delenv("PK_CHUNK", raising=False)
    bp, jp = checkpoint
    rng = np.random.default_rng(41)
    mels = [rng.standard_normal((128, 4104)).astype(np.float32),
            rng.standard_normal((128, 200)).astype(np.float32)]
    want_enc, want_tok = [], []
    for i, m in enumerate(mels):
        d = tmp_path / f"u{i}"
        d.mkdir()
        e, t = reference_run(bp, jp, m, d)
        want_enc.append(e)
        want_tok.append(t)
    frames = [m.shape[1] for m in mels]
    enc_frames = [cuda.lib().pkcu_asr_encoder_frames(f) for f in frames]
    assert enc_frames == [513, 25] and [e.shape[0] for e in want_enc] == enc_frames
    mel_d = dev(np.concatenate([m.reshape(-1) for m in mels]))
    with cuda.Weights(bp, jp) as w:
        w.upload(cuda.stream_handle())
        with cuda.ASR(w) as asr:
            out = empty(sum(enc_frames) * D)
            asr.encode(mel_d, frames, out)
            enc = host(out).reshape(-1, D).copy()
            toks = asr.transcribe(mel_d, frames)
            asr.set_chunk_mode(cuda.PKCU_CHUNK_OFF)        # the whole 513 frames at once
            asr.encode(mel_d, frames, out)
            enc_off = host(out).reshape(-1, D).copy()
    base = np.concatenate([[0], np.cumsum(enc_frames)])
    for u in range(2):
        e = enc[base[u]:base[u + 1]]
        err = np.abs(e.astype(np.float64) - want_enc[u]).max()
        print(f"utterance {u}: {enc_frames[u]} encoder frames, max |gpu - reference| = {err:.3e}, "
              f"{len(want_tok[u])} tokens")
        assert err <= 5e-5, (u, err)
        assert len(toks[u]) == len(want_tok[u]) and (toks[u] == want_tok[u]).all(), \
            (u, len(toks[u]), len(want_tok[u]))
    # chunking changed the long utterance (attention over 408 + 121 frames,
    # not 513) and left the short one alone
    assert np.abs(enc_off[:513] - enc[:513]).max() > 1e-3
    assert_bitexact(enc_off[513:], enc[513:], "short utterance unchanged by the chunk mode")
