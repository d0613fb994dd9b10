"""GPU parity at model depth, teacher-forced: the fused 24-block sequence
(pkcu_encoder_nongemm, one call over all 24 blocks) on the benchmarked
configurations, with every block checked against the restatement of
csrc/encoder.c:482-491 fed that block's own GPU input.

A GEMM hook captures, inside the one 24-block call, each block's input x (at
the block's first GEMM point, before any residual touches x) and all fourteen
GEMM inputs the block produces (at its last GEMM point, where every one of
them is still in place). The oracle then runs each block on the GPU's input
for that block, so rounding differences cannot compound from block to block
and the north-star tolerance (|a - b| <= max(2e-6, 1e-5 |b|); bit-exact for
the data-movement outputs) holds at every depth:

  * BASELINE config 4, the bench's workload: utterances of T = 375 frames;
  * 3200 frames as 8 chunks of 400 frames with 8-frame
    overlaps, edge chunks 408 frames and interior ones 416
    (csrc/encoder.c:531-543), one ragged batch.

The free-running drift (GPU chain against the restatement's own chain, no
teacher forcing) is measured in the same run beside the drift of the
reference's own build against the same restatement over the same blocks
(test_free_running_drift_tracks_reference_build): every block ends in a
LayerNorm, so neither grows with depth (both stay near 1e-6 over 24 blocks)."""
import numpy as np
import pytest

import pyoracle as po
from conftest import assert_bitexact, assert_close
from gpuhelp import Layout, dev
from test_encoder_gpu import EXACT, batch_standins, gpu_inputs, item_view, make_batch

pytestmark = pytest.mark.gpu

PKCU_GEMM_FF1_1, PKCU_GEMM_FF2_2 = 0, 11


def run_gpu_captured(cuda, lengths, blocks, items):
    """One pkcu_encoder_nongemm call over all blocks; returns the layout, the
    per-block inputs x_b (host), the final x and, per block, the GEMM inputs
    (host arrays)."""
    import torch
    L = Layout(lengths)
    cat = batch_standins(L, items)
    x = np.concatenate([xi for _, xi in items])
    dev_blocks = [{k: dev(v) for k, v in p.items()} for p in blocks]
    arr = cuda.block_params_array(dev_blocks)
    gout_t = {k: dev(v) for k, v in cat.items()}
    gin_t = gpu_inputs(L)
    xd = dev(x)
    x_in = [None] * len(blocks)
    caps = [None] * len(blocks)
    errors = []

    def on_gemm(user, block, gemm, s):
        # copies enqueued on the sequence's own stream (None: the legacy default stream)
        try:
            stream = torch.cuda.ExternalStream(s) if s else torch.cuda.default_stream()
            with torch.cuda.stream(stream):
                if gemm == PKCU_GEMM_FF1_1:
                    x_in[block] = xd.clone()
                elif gemm == PKCU_GEMM_FF2_2:
                    caps[block] = {r: gin_t[r].clone() for r in po.CAPTURE_ROLES}
        except Exception as e:   # a ctypes callback cannot raise: report it as a failing hook
            errors.append(e)
            return 1
        return 0

    hook = cuda.GEMM_HOOK(on_gemm)
    with cuda.Seq(lengths) as seq:
        try:
            cuda.encoder_nongemm(xd, arr, len(blocks), cuda.gemm_outputs(gout_t),
                                 cuda.gemm_inputs(gin_t), seq, hook=hook)
        except cuda.PkCudaError:
            if errors:
                raise errors[0]
            raise
        torch.cuda.synchronize()
    assert not errors, errors
    assert all(c is not None for c in caps) and all(v is not None for v in x_in)
    x_host = [t.cpu().numpy() for t in x_in]
    return L, x_host, xd.cpu().numpy(), caps


def check_teacher_forced(oracle, L, items, blocks, x_in, x_out, caps):
    """Every block of every item against the restatement run on the GPU's own
    block input; returns the largest |diff| of x per block."""
    worst = []
    for b, p in enumerate(blocks):
        got = {r: caps[b][r].cpu().numpy() for r in po.CAPTURE_ROLES}
        nxt = x_in[b + 1] if b + 1 < len(blocks) else x_out
        w = 0.0
        for i, (si, _) in enumerate(items):
            xo, ref = oracle.conformer_block(L.frames_of(x_in[b], i), p, si)
            g = L.frames_of(nxt, i)
            assert_close(g, xo, f"x after block {b} item {i}")
            w = max(w, float(np.abs(g.astype(np.float64) - xo).max()))
            for role in po.CAPTURE_ROLES:
                gv = item_view(L, role, got[role], i)
                if role in EXACT:
                    assert_bitexact(gv, ref[role], f"{role} block {b} item {i}")
                else:
                    assert_close(gv, ref[role], f"{role} block {b} item {i}")
        caps[b] = None   # release the block's device copies
        worst.append(w)
    return worst


@pytest.mark.parametrize("lengths", [[375] * 4, [408] + [416] * 6 + [408]],
                         ids=["config4_T375x4", "config3_chunks408_416"])
def test_24_blocks_teacher_forced(cuda, oracle, lengths):
    blocks, items = make_batch(lengths, 24, seed=24 + sum(lengths))
    L, x_in, x_out, caps = run_gpu_captured(cuda, lengths, blocks, items)
    # block 0's input is the batch's x as given
    assert_bitexact(x_in[0], np.concatenate([x for _, x in items]), "block 0 input")
    worst = check_teacher_forced(oracle, L, items, blocks, x_in, x_out, caps)
    assert len(worst) == 24 and max(worst) < 1e-4


def _chain(fn, x, blocks, si):
    out = []
    for p in blocks:
        x, _ = fn(x, p, si)
        out.append(x)
    return out


def test_free_running_drift_tracks_reference_build(cuda, oracle, reference):
    """Free-running 24 blocks on one utterance of T = 375: the GPU's chain and
    the reference build's own chain (csrc/encoder.c:482 compiled with the
    reference flags) both drift from the IEEE restatement's chain; the GPU's
    drift stays within a small multiple of the reference's own."""
    blocks, items = make_batch([375], 24, seed=375)
    L, x_in, x_out, _ = run_gpu_captured(cuda, [375], blocks, items)
    si, x0 = items[0]
    ora = _chain(oracle.conformer_block, x0, blocks, si)
    ref = _chain(reference.conformer_block, x0, blocks, si)
    gpu = [g.reshape(x0.shape) for g in x_in[1:] + [x_out]]
    d_gpu = [float(np.abs(g.astype(np.float64) - o).max()) for g, o in zip(gpu, ora)]
    d_ref = [float(np.abs(r.astype(np.float64) - o).max()) for r, o in zip(ref, ora)]
    print("block  |gpu - restatement|  |reference build - restatement|")
    for b, (a, c) in enumerate(zip(d_gpu, d_ref)):
        print(f"{b:5d}  {a:.3e}  {c:.3e}")
    # within the north-star tolerance, like the reference build's own drift
    assert max(d_gpu) <= max(2 * max(d_ref), 2e-6), (d_gpu, d_ref)
    assert np.isfinite(x_out).all()
