"""GPU parity of the fused per-block sequence (pkcu_encoder_nongemm) against
the restatement of csrc/encoder.c:482-491 run block by block, item by item
(and, for one block, against the reference's own conformer_block).

Every GEMM input the sequence produces (the 4 LayerNorm outputs, both Swish
outputs, Q+u, Q+v, K, V, P heads, softmax scores, head concat, channel-first
LN, depthwise-conv output) and the residual stream x are compared."""
import numpy as np
import pytest

import pyoracle as po
from conftest import assert_bitexact, assert_close
from gpuhelp import D, DH, FF, H, Layout, dev, empty, host

pytestmark = pytest.mark.gpu

EXACT = ("Qu", "K", "Qv", "V", "P_h", "attn")


def make_batch(lengths, n_blocks, seed):
    r = np.random.default_rng(seed)
    blocks = [po.random_block_inputs(r, 1)[0] for _ in range(n_blocks)]
    items = []
    for T in lengths:
        _, si, x = po.random_block_inputs(r, T)
        items.append((si, x))
    return blocks, items


def batch_standins(L, items):
    cat = {}
    for role in po.STANDIN_ROLES:
        cat[role] = np.concatenate([si[role].reshape(-1) for si, _ in items])
    return cat


def gpu_inputs(L):
    F = L.frames
    return {"ln_ff1": empty(F * D), "h1": empty(F * FF), "ln_sa": empty(F * D),
            "Qu": empty(F * D), "K": empty(F * D), "Qv": empty(F * D), "V": empty(F * D),
            "P_h": empty(int(L.pos[-1]) * D), "S": empty(int(L.score[-1])), "attn": empty(F * D),
            "cf": empty(F * D), "dw": empty(F * D), "ln_ff2": empty(F * D), "h2": empty(F * FF),
            "gated": empty(F * D)}


def item_view(L, role, flat, i):
    T = L.T[i]
    if role in ("ln_ff1", "ln_sa", "attn", "ln_ff2"):
        return L.frames_of(flat, i)
    if role in ("h1", "h2"):
        return L.frames_of(flat, i, FF)
    if role in ("Qu", "K", "Qv", "V"):
        return L.chunk(flat, i, D, (H, T, DH))
    if role == "P_h":
        return flat[L.pos[i] * D:L.pos[i + 1] * D].reshape(H, 2 * T - 1, DH)
    if role == "S":
        return L.scores(flat, i)
    if role in ("cf", "dw"):
        return L.chunk(flat, i, D, (D, T))
    raise KeyError(role)


def run_gpu(cuda, lengths, blocks, items):
    L = Layout(lengths)
    cat = batch_standins(L, items)
    x = np.concatenate([xi for _, xi in items])
    dev_blocks = [{k: dev(v) for k, v in p.items()} for p in blocks]
    arr = cuda.block_params_array(dev_blocks)
    gout_t = {k: dev(v) for k, v in cat.items()}
    gin_t = gpu_inputs(L)
    xd = dev(x)
    with cuda.Seq(lengths) as seq:
        cuda.encoder_nongemm(xd, arr, len(blocks), cuda.gemm_outputs(gout_t),
                             cuda.gemm_inputs(gin_t), seq)
        got = {k: host(v) for k, v in gin_t.items()}
        gx = host(xd)
    return L, gx, got


@pytest.mark.parametrize("lengths,n_blocks", [([9], 1), ([1, 7, 32], 1), ([408, 416, 408], 1),
                                              ([37, 5], 2), ([375], 2)])
def test_encoder_nongemm_vs_oracle(cuda, oracle, lengths, n_blocks):
    blocks, items = make_batch(lengths, n_blocks, seed=sum(lengths) + n_blocks)
    L, gx, got = run_gpu(cuda, lengths, blocks, items)
    for i, (si, x) in enumerate(items):
        xi = x
        for p in blocks:
            xi, caps = oracle.conformer_block(xi, p, si)
        assert_close(L.frames_of(gx, i), xi, f"x item {i}")
        for role in po.CAPTURE_ROLES:
            g = item_view(L, role, got[role], i)
            if role in EXACT:
                assert_bitexact(g, caps[role], f"{role} item {i}")
            else:
                assert_close(g, caps[role], f"{role} item {i}")


@pytest.mark.parametrize("lengths,n_groups", [([9, 5, 7], 2), ([408, 416, 416, 408], 3),
                                              ([33], 1)])
def test_encoder_nongemm_host_buffers(cuda, oracle, lengths, n_groups):
    """pkcu_encoder_nongemm_host: host x and GEMM outputs in, host x out, the
    batch pipelined over n_groups; same result as the device-resident call."""
    import torch
    blocks, items = make_batch(lengths, 2, seed=9 + sum(lengths))
    L, gx_dev, _ = run_gpu(cuda, lengths, blocks, items)
    cat = batch_standins(L, items)
    host_out = {k: torch.from_numpy(v).pin_memory() for k, v in cat.items()}
    x_host = torch.from_numpy(np.concatenate([xi for _, xi in items])).pin_memory()
    dev_blocks = [{k: dev(v) for k, v in p.items()} for p in blocks]
    arr = cuda.block_params_array(dev_blocks)
    with cuda.Seq(lengths) as seq:
        ws = cuda.EncoderWorkspace(seq, n_groups)
        assert ws.d2h_bytes == L.frames * D * 4
        assert ws.h2d_bytes == ws.d2h_bytes + sum(v.numel() * 4 for v in host_out.values())
        ws.run_host(x_host.data_ptr(), cuda.gemm_outputs(host_out), arr, len(blocks))
        ws.close()
    got = x_host.numpy()
    assert_bitexact(got, gx_dev, "host path == device path")
    for i, (si, x) in enumerate(items):
        for p in blocks:
            x, _ = oracle.conformer_block(x, p, si)
        assert_close(L.frames_of(got, i), x, f"x item {i}")


@pytest.mark.parametrize("T", [41, 375])
def test_encoder_nongemm_vs_reference_block(cuda, reference, T):
    """One block against the reference's own conformer_block (csrc/encoder.c:482),
    also at the bench's T = 375."""
    blocks, items = make_batch([T], 1, seed=4100 + T)
    L, gx, got = run_gpu(cuda, [T], blocks, items)
    si, x = items[0]
    xr, caps = reference.conformer_block(x, blocks[0], si)
    assert_close(gx, xr, "x")
    for role in po.CAPTURE_ROLES:
        assert_close(item_view(L, role, got[role], 0), caps[role], role)


def test_chunked_long_audio_24_blocks(cuda, oracle):
    """3200 frames in 8 chunks of 400 + 8-frame overlaps, the
    edge chunks 408 frames and the interior ones 416 (csrc/encoder.c:531-543),
    as one ragged batch through all 24 blocks; every chunk against the
    restatement run chunk by chunk, block by block."""
    lengths = [408] + [416] * 6 + [408]
    blocks, items = make_batch(lengths, 24, seed=3200)
    L, gx, got = run_gpu(cuda, lengths, blocks, items)
    for i, (si, x) in enumerate(items):
        for p in blocks:
            x, caps = oracle.conformer_block(x, p, si)
        # 24 free-running blocks: every block ends in a LayerNorm, so rounding
        # differences do not compound (measured drift about 1.4e-6, as for the
        # reference's own build against the restatement: test_depth_gpu.py)
        assert_close(L.frames_of(gx, i), x, f"x chunk {i}")
        for role in ("S", "dw", "h2", "ln_ff2"):
            assert_close(item_view(L, role, got[role], i), caps[role], f"{role} chunk {i}")
    assert np.isfinite(gx).all()


def test_encoder_nongemm_24_blocks_stays_bounded(cuda, oracle):
    """24 blocks (the model depth): residual stream within tolerance of the
    restatement after every LN_out renormalisation."""
    blocks, items = make_batch([33], 24, seed=2424)
    L, gx, got = run_gpu(cuda, [33], blocks, items)
    si, x = items[0]
    for p in blocks:
        x, caps = oracle.conformer_block(x, p, si)
    assert_close(gx, x, "x after 24 blocks")
    assert np.isfinite(gx).all()


def test_sequence_launch_count(cuda):
    """pkcu_encoder_nongemm_launches (the bench's gpu_launches claim) equals
    the number of kernels one call launches, counted by the CUDA profiler."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    lengths, n_blocks = [37, 5, 40], 2
    blocks, items = make_batch(lengths, n_blocks, seed=77)
    run_gpu(cuda, lengths, blocks, items)   # warm-up: first-call attribute setup
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run_gpu(cuda, lengths, blocks, items)
        torch.cuda.synchronize()
    seq_kernels = ("ln1024_kernel", "row_vec_kernel", "qkv_split_kernel", "pos_split_kernel",
                   "relpos_scores", "head_concat_kernel", "ln_transpose_kernel",
                   "dwconv_al_kernel", "dwconv_row_kernel", "transpose_add_kernel")
    n = sum(1 for e in prof.events()
            if e.device_type == torch.autograd.DeviceType.CUDA and any(k in e.name for k in seq_kernels))
    assert n == cuda.lib().pkcu_encoder_nongemm_launches(n_blocks), n
