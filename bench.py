#!/usr/bin/env python3
"""Encoder non-GEMM throughput on B200: frames/s and achieved HBM GB/s.

Workload (the one the metric is quoted on at 1/2/4/8 GPUs):
per GPU, a batch of 256 independent utterances of T = 375 frames run through
the 24-block non-GEMM op sequence of the FastConformer encoder
(pkcu_encoder_nongemm: LayerNorms, bias+Swish, residuals, QKV head split with
pos_bias_u/v, positional head split, rel-shift + score combine + softmax, head
concat, GLU, depthwise conv + Swish, conv transpose-add). GEMM outputs are
seeded N(0,1) stand-ins resident in HBM (the GEMMs are outside this path);
block parameters are random (LN gamma ~ N(1,0.1), others ~ 0.1 N(0,1)).
Each step reads > 10 GB per GPU, far above the 126 MB L2.

Multi-GPU: one process per GPU (torchrun), every rank runs its own batch, no
collective on the data path (weak scaling); time = max over ranks of the
device time (CUDA events), value = all ranks' frames / that time.

  python bench.py [--gpus N] [--steps K] [--warmup W]          # this library
  python bench.py --impl reference [--steps K] [--warmup W]    # reference CPU code

Output: one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime as dt
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "parakeet-unified-en-0.6b-c_b200")
sys.path.insert(0, os.path.join(PKG, "python"))

METRIC = "encoder non-GEMM frames/s and achieved HBM GB/s (% of peak) at 1/2/4/8 B200"
D, H, DH, FF = 1024, 8, 128, 4096
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--utts", type=int, default=256, help="utterances per GPU")
    ap.add_argument("--T", type=int, default=375, help="frames per utterance")
    ap.add_argument("--blocks", type=int, default=24)
    ap.add_argument("--groups", type=int, default=8, help="pipeline groups of the host-buffer run")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of a CUDA graph")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-aux", action="store_true", help="skip the standalone-kernel table")
    ap.add_argument("--extras", action="store_true",
                    help="also time the steps beyond the non-GEMM path (fused GEMMs, encoder "
                         "with GEMMs, decode, mel-to-tokens) and print them as one JSON line "
                         "before the bench line")
    ap.add_argument("--aux-only", action="store_true",
                    help="time only the standalone kernels (one JSON object), e.g. for ncu")
    ap.add_argument("--pre-only", action="store_true",
                    help="with --aux-only: time only the pre-encode stage")
    ap.add_argument("--gemm-only", action="store_true",
                    help="with --aux-only: time only the weight products (tcgen05 GEMMs with fused epilogues)")
    ap.add_argument("--gemm-rows", type=int, default=24000,
                    help="rows M of the fused-GEMM timing")
    ap.add_argument("--forward-only", action="store_true",
                    help="with --aux-only: time only the encoder stack with its GEMMs")
    ap.add_argument("--decode-fused-only", action="store_true",
                    help="with --aux-only: time only pkcu_greedy_decode_fused (--dec-utts, --dec-frames, --dec-shift)")
    ap.add_argument("--dec-utts", type=int, default=256)
    ap.add_argument("--dec-frames", type=int, default=40)
    ap.add_argument("--dec-shift", type=float, default=0.0)
    ap.add_argument("--asr-decode-only", action="store_true",
                    help="with --aux-only: time only pkcu_asr_decode")
    ap.add_argument("--asr-only", action="store_true",
                    help="with --aux-only: time only mel-to-tokens transcription")
    ap.add_argument("--decode-only", action="store_true",
                    help="with --aux-only: time only the batched greedy decode")
    ap.add_argument("--pre-utts", type=int, default=64,
                    help="utterances of 3000 mel frames in the pre-encode timing")
    ap.add_argument("--aux-reps", type=int, default=5,
                    help="timed launches per standalone kernel (0: one untimed launch each)")
    return ap.parse_args()


# ── algorithmic bytes (read each input once, write each output once) ─────────

def kernel_table(F, T, n_items):
    """(name, bytes per launch over the batch, launches per block)."""
    L = 2 * T - 1
    S = n_items * H * T * T
    return [
        ("bias_swish_rows", 8 * F * FF, 2),
        ("residual_layer_norm", 16 * F * D, 1),
        ("qkv_split_uv", 28 * F * D, 1),
        ("pos_head_split", 8 * n_items * L * D, 1),
        ("relpos_combine_softmax", 12 * S, 1),
        ("head_concat", 8 * F * D, 1),
        ("residual_layer_norm_transpose", 16 * F * D, 1),
        ("glu_dwconv_bn_swish", 12 * F * D, 1),
        ("transpose_add_layer_norm", 16 * F * D, 1),
        ("residual_layer_norm2", 16 * F * D, 1),
    ]


def step_bytes(F, T, n_items, n_blocks):
    per_block = sum(b * n for _, b, n in kernel_table(F, T, n_items))
    # + the first block's LN_ff1 (8FD); the last block's residual_layer_norm2 writes no LN_next
    return n_blocks * per_block + 8 * F * D - 4 * F * D


# ── multi-GPU plumbing (one process per GPU, no data-path collective) ────────

def shard(rank: int, world: int, per_rank: int) -> range:
    """Global indices of the utterances one rank processes. Weak scaling: each
    rank owns its own per_rank independent utterances; nothing is exchanged."""
    assert 0 <= rank < world and per_rank > 0
    return range(rank * per_rank, (rank + 1) * per_rank)


def max_over_ranks(x: float, world: int, device=None) -> float:
    """Max of a per-rank timing over all ranks (the slowest rank sets the pace)."""
    import torch
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ── clocks during the timed region ───────────────────────────────────────────

class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, local_index):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        ident = str(local_index)
        if vis:
            parts = [p.strip() for p in vis.split(",") if p.strip()]
            if local_index < len(parts):
                ident = parts[local_index]
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", ident], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except OSError:
            self.proc = None

    def stop(self, t0, t1):
        if self.proc is None:
            return {"unavailable": "nvidia-smi not found"}
        self.proc.terminate()
        try:
            out = self.proc.communicate(timeout=10)[0]
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out = ""
        rows = []
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                ts = dt.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[1]), float(f[2]), f[3], f[4:8]))
            except ValueError:
                continue
        inside = [r for r in rows if t0 <= r[0] <= t1] or rows
        if not inside:
            return {"unavailable": "no samples"}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v == "Active"})
        sm = sorted(r[1] for r in inside)
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(r[2] for r in inside),
                "samples": len(inside), "reasons": reasons}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel)
    except (OSError, ValueError):
        return None


# ── CPU reference path (the reference's own compiled code) ────────────────────

class RefRunner:
    """The reference's conformer_block (csrc/encoder.c:482-491) from
    oracle/_ref/libpkref.so, GEMM calls replaced by no-ops, so that only the
    reference's non-GEMM code runs; one utterance of T frames per call, rows
    spread over PK_THREADS pool threads as in the reference."""

    def __init__(self, T, n_blocks, threads=None):
        import numpy as np
        cores = os.cpu_count() or 1
        self.threads_req = threads or min(cores, 16)   # the reference clamps to 16 (csrc/threadpool.c:10)
        os.environ["PK_THREADS"] = str(self.threads_req)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import pyoracle as po
        self.po = po
        self.ref = po.Reference()
        rng = np.random.default_rng(4)
        blocks = [po.random_block_inputs(rng, 1)[0] for _ in range(min(n_blocks, 4))]
        self.flat = (po.FP * (22 * n_blocks))()
        self.keep = []
        for b in range(n_blocks):
            p = blocks[b % len(blocks)]
            for j, role in enumerate(po.PARAM_ROLES):
                a = po.f32(p[role])
                self.keep.append(a)
                self.flat[22 * b + j] = a.ctypes.data_as(po.FP)
        self.ws = rng.standard_normal(self.ref.L.pkref_ws_floats(T)).astype(np.float32)
        self.x = rng.standard_normal((T, D)).astype(np.float32)
        self.T, self.n_blocks = T, n_blocks
        self.run_one()   # warm-up; creates the thread pool
        self.threads = self.ref.L.pkref_pool_threads()

    def run_one(self):
        po = self.po
        rc = self.ref.L.pkref_conformer_blocks(self.x.ctypes.data_as(po.FP), self.T, self.n_blocks,
                                               self.flat, None, None, 0, self.ws.ctypes.data_as(po.FP))
        assert rc == 0

    def sample(self, seconds, min_utts=1, max_utts=64):
        n, t0 = 0, time.perf_counter()
        while n < min_utts or (time.perf_counter() - t0 < seconds and n < max_utts):
            self.run_one()
            n += 1
        secs = time.perf_counter() - t0
        return n * self.T / secs, n, secs


def reference_arm(args, rank, world):
    """--impl reference: rank 0 times the reference CPU implementation."""
    if rank != 0:
        return
    r = RefRunner(args.T, args.blocks)
    for _ in range(args.warmup):
        r.run_one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r.run_one()
    secs = time.perf_counter() - t0
    threads = r.threads
    frames = args.steps * args.T
    value = frames / secs
    sample = (f"{args.steps} steps x 1 utterance x T={args.T} x {args.blocks} blocks through the "
              f"reference's conformer_block with GEMMs as no-ops, PK_THREADS={threads}")
    config = config_dict(args, world)
    config["workload"] = (f"config 4 sampled: each step 1 utterance x T={args.T} through the "
                          f"{args.blocks}-block non-GEMM op sequence (utterances are independent, "
                          f"so frames/s does not depend on how many run), fp32")
    config["utterances_per_step"] = 1
    line = {
        "metric": METRIC, "value": value, "unit": "frames/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * secs / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": value, "unit": "frames/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args, world):
    return {"workload": f"config 4: {args.utts} utterances x T={args.T} per GPU, "
                        f"{args.blocks}-block non-GEMM op sequence (fused kernels), fp32",
            "model": "parakeet-unified-en-0.6b FastConformer (D=1024, 8x128 heads, FF=4096, conv k=9)",
            "utterances_per_gpu": args.utts, "global_batch": args.utts * world, "seq_len": args.T,
            "blocks": args.blocks, "parallelism": f"dp{world} (utterances sharded, no collectives)",
            "l2": "inputs larger than L2 (GEMM stand-ins > 10 GB per GPU per step)"}


# ── this library ──────────────────────────────────────────────────────────────

def setup_device(args, rank, world):
    import torch
    import pkcuda
    mine = shard(rank, world, args.utts)
    seq = pkcuda.Seq([args.T] * len(mine))
    ws = pkcuda.EncoderWorkspace(seq, args.groups)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234 + mine.start)   # this rank's own utterances
    x_addr, gout, gin = fill_workspace(ws, seq, gen)
    blocks = random_block_params(args.blocks, gen)
    arr = pkcuda.block_params_array(blocks)
    return seq, ws, x_addr, gout, gin, blocks, arr


def random_block_params(n_blocks, gen):
    """Device block parameters: LN gamma ~ N(1, 0.1), depthwise taps 0.3 N(0,1),
    the rest 0.1 N(0,1)."""
    import torch
    import pkcuda
    blocks = []
    for _ in range(n_blocks):
        p = {}
        for f in pkcuda.BLOCK_PARAM_FIELDS:
            n = {"ff1_b1": FF, "ff2_b1": FF, "qkv_b": 3 * D, "pw1_b": 2 * D, "dw_w": 9 * D,
                 "pos_u": D, "pos_v": D}.get(f, D)
            t = torch.randn(n, device="cuda", generator=gen)
            if f.startswith("norm") and f.endswith("_w"):
                t = 1.0 + 0.1 * t
            elif f == "dw_w":
                t = 0.3 * t
            else:
                t = 0.1 * t
            p[f] = t.contiguous()
        blocks.append(p)
    return blocks


def fill_workspace(ws, seq, gen):
    """N(0,1) in x and every stand-in GEMM output of a workspace."""
    import pkcuda
    x_addr, gout, gin = ws.device()
    F = seq.frames
    ext = {"ff1_h": F * FF, "ff1_out": F * D, "qkv": 3 * F * D, "P": seq.pos_rows * D,
           "ac": seq.score_elems, "bd": seq.bd_elems, "attn_h": F * D, "att_out": F * D,
           "pw1": 2 * F * D, "pw2": F * D, "ff2_h": F * FF, "ff2_out": F * D}
    tensor_at(x_addr, F * D).normal_(generator=gen)
    for f in pkcuda.GEMM_OUT_FIELDS:
        tensor_at(getattr(gout, f), ext[f]).normal_(generator=gen)
    return x_addr, gout, gin


CONFIG3_LENGTHS = [408] + [416] * 6 + [408]


def ragged_step_bytes(lengths, n_blocks):
    """Algorithmic bytes of the sequence over a ragged batch: every term of
    step_bytes is a sum over items, so the batch total is the items' sum."""
    return sum(step_bytes(T, T, 1, n_blocks) for T in lengths)


def time_config3(args, stream, reps=10):
    """BASELINE config 3 as configured: 3200 frames of long audio as 8 chunks
    of 400 frames plus 8-frame overlaps (edge chunks 408 frames, interior ones
    416, csrc/encoder.c:531-543), one ragged batch through the 24-block
    sequence; GEMM outputs are N(0,1) stand-ins (about 375 MB, above the L2).
    CUDA-graph replays timed with CUDA events on the bench stream."""
    import torch
    import pkcuda
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3200)
    seq = pkcuda.Seq(CONFIG3_LENGTHS)
    ws = pkcuda.EncoderWorkspace(seq, 1)
    try:
        x_addr, gout, gin = fill_workspace(ws, seq, gen)
        blocks = random_block_params(args.blocks, gen)
        arr = pkcuda.block_params_array(blocks)

        def step():
            pkcuda.call("pkcu_encoder_nongemm", x_addr, C.cast(arr, pkcuda.VP), args.blocks,
                        C.byref(gout), C.byref(gin), seq.handle, None, None, stream.cuda_stream)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        del graph
    finally:
        ws.close()
        seq.close()
    frames = sum(CONFIG3_LENGTHS)
    nb = ragged_step_bytes(CONFIG3_LENGTHS, args.blocks)
    return {"chunks": "408,416x6,408", "frames": frames, "ms": round(ms, 4),
            "frames_per_s": round(frames / (ms * 1e-3)), "gbs": round(nb / (ms * 1e-3) / 1e9, 1)}


def time_config5(stream, reps=20):
    """BASELINE config 5 as configured, each op timed launch by launch with an
    L2 flush (a 512 MB device write) between launches, since these sizes fit
    in the 126 MB L2: GPTQ int4 dequant of FF1 [1024, 4096] and FF2
    [4096, 1024] with G = 128 along K; int8 dequant of the fused QKV
    [1024, 3072] and out-proj [1024, 1024] weights; the RNN-T joint add + tanh
    at B = 32 x T = 416 x J = 640 and the argmax over [13312, 1025] logits.
    Algorithmic bytes as in kernel_table's notes (each input read once, each
    output written once)."""
    import torch
    import pkcuda
    sh = stream.cuda_stream
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    f32 = dict(device=dev, dtype=torch.float32)
    flush = torch.empty(128 << 20, **f32)
    out = {}

    def timed(name, nbytes, fn):
        fn()
        total = 0.0
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        ms = total / reps
        out[name] = {"us": round(1000 * ms, 2), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}

    G = 128
    for tag, K, N in (("dequant_i4_ff1_g128_k", 1024, 4096), ("dequant_i4_ff2_g128_k", 4096, 1024)):
        pk = torch.randint(0, 256, (K * N // 2,), generator=g, device=dev, dtype=torch.uint8)
        sc = 1e-3 + 1.9e-2 * torch.rand(K * N // G, generator=g, **f32)
        o = torch.empty(K * N, **f32)
        timed(tag, K * N // 2 + 4 * K * N // G + 4 * K * N,
              lambda: pkcuda.call("pkcu_dequant_i4", pk.data_ptr(), sc.data_ptr(), o.data_ptr(), K, N, G,
                                  pkcuda.PKCU_GROUP_ALONG_K, sh))
    for tag, n in (("dequant_i8_qkv", 1024 * 3072), ("dequant_i8_out", 1024 * 1024)):
        q = torch.randint(-127, 128, (n,), generator=g, device=dev, dtype=torch.int8)
        o = torch.empty(n, **f32)
        timed(tag, 5 * n, lambda: pkcuda.call("pkcu_dequant_i8", q.data_ptr(), 5e-3, o.data_ptr(), n, sh))
    B, T, J, V = 32, 416, 640, 1025
    enc = torch.randn(B * T * J, generator=g, **f32)
    pred = torch.randn(B * J, generator=g, **f32)
    jo = torch.empty_like(enc)
    timed("joint_add_tanh", 8 * B * T * J + 4 * B * J,
          lambda: pkcuda.call("pkcu_joint_add_act", enc.data_ptr(), pred.data_ptr(), jo.data_ptr(),
                              B, T, J, pkcuda.PKCU_ACT_TANH, sh))
    logits = torch.randn(B * T * V, generator=g, **f32)
    am = torch.empty(B * T, device=dev, dtype=torch.int32)
    timed("argmax_rows", 4 * B * T * V + 4 * B * T,
          lambda: pkcuda.call("pkcu_argmax_rows", logits.data_ptr(), am.data_ptr(), B * T, V, sh))
    torch.cuda.synchronize()
    return out


def tensor_at(addr, n):
    """A float32 torch view of n elements of device memory owned by the C library."""
    import torch

    class _Holder:
        pass

    h = _Holder()
    h.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (addr, False),
                                  "version": 3, "strides": None}
    return torch.as_tensor(h, device="cuda")


def time_kernels(args, seq, x_addr, gout, gin, blocks, stream, reps=10):
    """Device time of each kernel of the sequence, launched alone on the bench
    stream over the full batch (CUDA events on that stream): the median of
    three runs of `reps` back-to-back launches, averaged per launch."""
    import torch
    import pkcuda
    F, T, n = seq.frames, args.T, args.utts
    p = blocks[0]
    sh = stream.cuda_stream
    P = lambda k: pkcuda.ptr(p[k])
    scale = 1.0 / (128.0 ** 0.5)
    calls = {
        "bias_swish_rows": lambda: pkcuda.call("pkcu_bias_swish_rows", gout.ff1_h, P("ff1_b1"), gin.h1, F, FF, sh),
        "residual_layer_norm": lambda: pkcuda.call("pkcu_residual_layer_norm", x_addr, gout.ff1_out, P("ff1_b2"), 0.5,
                                                   P("norm_sa_w"), P("norm_sa_b"), gin.ln_sa, F, sh),
        "qkv_split_uv": lambda: pkcuda.call("pkcu_qkv_split_uv", gout.qkv, P("qkv_b"), P("pos_u"), P("pos_v"),
                                            gin.Qu, gin.Qv, gin.K, gin.V, seq.handle, sh),
        "pos_head_split": lambda: pkcuda.call("pkcu_pos_head_split", gout.P, gin.P_h, seq.handle, sh),
        "relpos_combine_softmax": lambda: pkcuda.call("pkcu_relpos_combine_softmax", gout.ac, gout.bd, gin.S,
                                                      scale, seq.handle, sh),
        "head_concat": lambda: pkcuda.call("pkcu_head_concat", gout.attn_h, gin.attn, seq.handle, sh),
        "residual_layer_norm_transpose": lambda: pkcuda.call(
            "pkcu_residual_layer_norm_transpose", x_addr, gout.att_out, P("out_b"), 1.0, P("norm_conv_w"),
            P("norm_conv_b"), gin.cf, seq.handle, sh),
        "glu_dwconv_bn_swish": lambda: pkcuda.call("pkcu_glu_dwconv_bn_swish", gout.pw1, P("pw1_b"), P("dw_w"),
                                                   P("dw_b"), None, 0.0, 1, gin.dw, D, 9, seq.handle, sh),
        "transpose_add_layer_norm": lambda: pkcuda.call(
            "pkcu_transpose_add_layer_norm", x_addr, gout.pw2, P("pw2_b"), P("norm_ff2_w"), P("norm_ff2_b"),
            gin.ln_ff2, seq.handle, sh),
        "residual_layer_norm2": lambda: pkcuda.call(
            "pkcu_residual_layer_norm2", x_addr, gout.ff2_out, P("ff2_b2"), 0.5, P("norm_out_w"), P("norm_out_b"),
            P("norm_ff1_w"), P("norm_ff1_b"), gin.ln_ff1, F, sh),
    }
    table = {}
    for name, nbytes, per_block in kernel_table(F, T, n):
        fn = calls[name]
        fn()
        # median of three runs of `reps` back-to-back launches
        runs = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            e1.synchronize()
            runs.append(e0.elapsed_time(e1) / reps)
        ms = sorted(runs)[1]
        table[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9,
                       "launches_per_step": per_block * args.blocks}
    return table


def time_aux_kernels(stream, reps=5, pre_utts=64, pre_only=False):
    """The tensor_ops entry points that are not part of the encoder block
    sequence, each timed alone (CUDA events on the bench stream, one warm-up
    launch) at a size above the 126 MB L2, with algorithmic bytes (each input
    read once, each output written once): plain LayerNorm [R, 1024]; row softmax over the
    score rows of 256 utterances (in place); Swish / ReLU (in place); int8
    dequant of 24 blocks' QKV + out weights; int4 dequant of 24 blocks' FF1 +
    FF2 weights with the reference's G = 32 scales along N and with G = 128
    along K; the RNN-T joint add + ReLU / tanh and the greedy argmax at 256
    utterances x 416 frames (J = 640, V = 1025). A device fill of the int4
    output size is timed beside them as the write-only reference point."""
    import torch
    import pkcuda
    if pre_only:
        return time_pre_encode(stream, reps, pre_utts)
    sh = stream.cuda_stream
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(8)
    out = {}

    def timed(name, shape, nbytes, fn):
        fn()
        torch.cuda.synchronize()
        if reps == 0:
            out[name] = {"shape": shape, "ms": None, "bytes": nbytes, "gbs": None}
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        out[name] = {"shape": shape, "ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}

    f32 = dict(device=dev, dtype=torch.float32)
    R, Dm = 96000, D
    x = torch.randn(R * Dm, generator=g, **f32)
    gam = 1 + 0.1 * torch.randn(Dm, generator=g, **f32)
    bet = 0.1 * torch.randn(Dm, generator=g, **f32)
    y = torch.empty_like(x)
    timed("layer_norm_rows", [R, Dm], 8 * R * Dm + 8 * Dm,
          lambda: pkcuda.call("pkcu_layer_norm_rows", x.data_ptr(), gam.data_ptr(), bet.data_ptr(),
                              y.data_ptr(), R, Dm, sh))
    del x, y
    rows, n = 256 * H * 375, 375
    sc = 4 * torch.randn(rows * n, generator=g, **f32)
    timed("softmax_rows", [rows, n], 8 * rows * n,
          lambda: pkcuda.call("pkcu_softmax_rows", sc.data_ptr(), rows, n, sh))
    del sc
    nv = 64 << 20
    v = 4 * torch.randn(nv, generator=g, **f32)
    timed("swish", [nv], 8 * nv, lambda: pkcuda.call("pkcu_swish", v.data_ptr(), nv, sh))
    timed("relu", [nv], 8 * nv, lambda: pkcuda.call("pkcu_relu", v.data_ptr(), nv, sh))
    del v
    n8 = 24 * (1024 * 3072 + 1024 * 1024)
    q8 = torch.randint(-127, 128, (n8,), generator=g, device=dev, dtype=torch.int8)
    o8 = torch.empty(n8, **f32)
    timed("dequant_i8", [n8], 5 * n8,
          lambda: pkcuda.call("pkcu_dequant_i8", q8.data_ptr(), 3e-3, o8.data_ptr(), n8, sh))
    del q8, o8
    K4, N4 = 24 * 2 * 1024, 4096     # 24 blocks of FF1 [1024, 4096] + FF2 (same count)
    p4 = torch.randint(0, 256, (K4 * N4 // 2,), generator=g, device=dev, dtype=torch.uint8)
    o4 = torch.empty(K4 * N4, **f32)
    for G, axis, tag in ((32, pkcuda.PKCU_GROUP_ALONG_N, "dequant_i4_g32_n"),
                         (128, pkcuda.PKCU_GROUP_ALONG_K, "dequant_i4_g128_k")):
        s4 = 1e-3 + 2e-2 * torch.rand(K4 * N4 // G, generator=g, **f32)
        timed(tag, [K4, N4], K4 * N4 // 2 + 4 * K4 * N4 // G + 4 * K4 * N4,
              lambda: pkcuda.call("pkcu_dequant_i4", p4.data_ptr(), s4.data_ptr(), o4.data_ptr(),
                                  K4, N4, G, axis, sh))
        del s4
    # reference point for write-dominated kernels: torch's fill of the same
    # 805 MB (a library kernel, write-only traffic)
    timed("fill_reference_write_only", [K4, N4], 4 * K4 * N4, lambda: o4.fill_(1.0))
    del p4, o4
    B, T, J, V = 256, 416, 640, 1025
    enc = torch.randn(B * T * J, generator=g, **f32)
    pred = torch.randn(B * J, generator=g, **f32)
    jo = torch.empty_like(enc)
    for act, tag in ((pkcuda.PKCU_ACT_RELU, "joint_add_relu"), (pkcuda.PKCU_ACT_TANH, "joint_add_tanh")):
        timed(tag, [B, T, J], 8 * B * T * J + 4 * B * J,
              lambda: pkcuda.call("pkcu_joint_add_act", enc.data_ptr(), pred.data_ptr(), jo.data_ptr(),
                                  B, T, J, act, sh))
    del enc, pred, jo
    logits = torch.randn(B * T * V, generator=g, **f32)
    am = torch.empty(B * T, device=dev, dtype=torch.int32)
    timed("argmax_rows", [B * T, V], 4 * B * T * V + 4 * B * T,
          lambda: pkcuda.call("pkcu_argmax_rows", logits.data_ptr(), am.data_ptr(), B * T, V, sh))
    del logits, am
    out.update(time_pre_encode(stream, reps, pre_utts))
    torch.cuda.synchronize()
    return out


GEMM_ROWS = 24000   # 64 utterances x 375 frames


def time_fused_gemms(stream, reps, M=GEMM_ROWS):
    """The GEMMs with fused epilogues at the feed-forward shapes, M = 24000
    rows: FF linear1 [M, 1024] x [1024, 4096] + bias + Swish, FF linear2
    [M, 4096] x [4096, 1024] + bias + 0.5 residual. Beside each, the unfused
    path it replaces: torch's fp32 GEMM (cuBLAS, TF32 off) followed by this
    library's separate bias + Swish / residual kernel. Reported: ms, fp32
    TFLOP/s (2 M N K / t) and, for the fused form, the bf16 tensor-core rate
    it runs at (nine bf16 MMAs per fp32 product) against the measured bf16 peak."""
    import torch
    import pkcuda
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    f32 = dict(device=dev, dtype=torch.float32)
    sh = stream.cuda_stream
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16_peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        bf16_peak = 1590.0

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(max(reps, 1)):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / max(reps, 1)

    res = {}
    for name, N, K in (("ff1_gemm_bias_swish", 4096, 1024), ("ff2_gemm_bias_residual", 1024, 4096)):
        A = torch.randn(M, K, generator=g, **f32)
        W = torch.randn(K, N, generator=g, **f32) / K ** 0.5
        b = 0.1 * torch.randn(N, generator=g, **f32)
        X = torch.randn(M, N, generator=g, **f32)
        if name.startswith("ff1"):
            fused = lambda: pkcuda.call("pkcu_gemm_bias_swish", A.data_ptr(), W.data_ptr(),
                                        b.data_ptr(), X.data_ptr(), M, N, K, sh)

            def unfused():
                H = torch.mm(A, W)
                pkcuda.call("pkcu_bias_swish_rows", H.data_ptr(), b.data_ptr(), H.data_ptr(), M, N, sh)
        else:
            fused = lambda: pkcuda.call("pkcu_gemm_bias_residual", A.data_ptr(), W.data_ptr(),
                                        b.data_ptr(), X.data_ptr(), 0.5, M, N, K, sh)

            def unfused():
                H = torch.mm(A, W)
                pkcuda.call("pkcu_residual_add", X.data_ptr(), H.data_ptr(), b.data_ptr(),
                            C.c_float(0.5), M, N, sh)
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            ms_f, ms_u = timed(fused), timed(unfused)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        flop = 2.0 * M * N * K
        res[name] = {"M": M, "N": N, "K": K, "ms": round(ms_f, 4),
                     "tflops_fp32": round(flop / ms_f / 1e9, 1),
                     "tensor_bf16_tflops": round(9 * flop / ms_f / 1e9, 1),
                     "tensor_frac": round(9 * flop / ms_f / 1e9 / bf16_peak, 3),
                     "unfused_cublas_fp32_ms": round(ms_u, 4),
                     "speedup_vs_unfused": round(ms_u / ms_f, 2)}
        del A, W, b, X
    torch.cuda.synchronize()
    return res


def time_tc_gemms(stream, reps, M=GEMM_ROWS):
    """The weight products on the library's tcgen05 GEMM (pkcu_wmatmul*) at
    the block's shapes, M = 24000 rows (64 utterances x 375 frames): FF
    linear1 + bias + Swish and linear2 + bias + 0.5 residual, the fused QKV
    with its head split, and the first pointwise convolution with its GLU, for
    the reference's weight storages (int8 per-tensor as its checkpoints store
    the projections, fp32, GPTQ int4 with G = 32 along N). Each call includes
    the activation's three-part split. Reported: ms (CUDA events), fp32
    TFLOP/s (2 M N K / t) and the bf16 tensor rate it runs at (three MMAs per
    product for an int8 weight, six for fp32 / int4) as a fraction of the
    measured sustained bf16 peak (the GEMMs run inside long steps)."""
    import torch
    import pkcuda
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(13)
    f32 = dict(device=dev, dtype=torch.float32)
    sh = stream.cuda_stream
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops_sustained"])
    except (OSError, KeyError, ValueError):
        peak = 1400.0
    L = pkcuda.lib()

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(max(reps, 1)):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / max(reps, 1)

    def weight(bits, K, N):
        if bits == 8:
            q = torch.randint(-127, 128, (K * N,), generator=g, device=dev, dtype=torch.int8)
            return pkcuda.Weight(q, 8, K, N, scale=0.004, stream=stream), [q]
        if bits == 4:
            pk = torch.randint(0, 256, (K * N // 2,), generator=g, device=dev, dtype=torch.uint8)
            sc = 1e-3 + 1.9e-2 * torch.rand(K * N // 32, generator=g, **f32)
            return pkcuda.Weight(pk, 4, K, N, scales=sc, stream=stream), [pk, sc]
        W = torch.randn(K * N, generator=g, **f32) / K ** 0.5
        return pkcuda.Weight(W, 32, K, N, stream=stream), [W]

    res = {}
    cases = (("ff1_bias_swish_int8", 8, 4096, 1024), ("ff2_bias_residual_int8", 8, 1024, 4096),
             ("qkv_head_split_int8", 8, 3072, 1024), ("ff1_bias_swish_fp32", 32, 4096, 1024),
             ("ff1_bias_swish_int4_g32", 4, 4096, 1024), ("pw1_glu_fp32", 32, 2048, 1024))
    for name, bits, N, K in cases:
        A = torch.randn(M * K, generator=g, **f32)
        b = 0.1 * torch.randn(N, generator=g, **f32)
        work = torch.empty(int(L.pkcu_wmatmul_work_bytes(M, K)) // 4 + 64, **f32)
        if name.startswith("pw1"):
            Wc = torch.randn(N * K, generator=g, **f32) / K ** 0.5
            w, keep = pkcuda.ConvWeight(Wc, N, K, glu=True, stream=stream), [Wc]
            X = torch.randn(K * M, generator=g, **f32)   # one item of M frames, channel-first
            out = torch.empty(N // 2 * M, **f32)
            fn = lambda: pkcuda.call("pkcu_pointwise_conv1d_glu", X.data_ptr(), w.handle, b.data_ptr(),
                                     out.data_ptr(), M, work.data_ptr(), sh)
        else:
            w, keep = weight(bits, K, N)
            out = torch.randn(M * N, generator=g, **f32)
            if "swish" in name:
                fn = lambda: pkcuda.call("pkcu_wmatmul_bias_swish", A.data_ptr(), w.handle, b.data_ptr(),
                                         out.data_ptr(), M, work.data_ptr(), sh)
            elif "residual" in name:
                fn = lambda: pkcuda.call("pkcu_wmatmul_bias_residual", A.data_ptr(), w.handle, b.data_ptr(),
                                         out.data_ptr(), C.c_float(0.5), M, work.data_ptr(), sh)
            else:
                seq = pkcuda.Seq([375] * (M // 375))
                u = 0.1 * torch.randn(D, generator=g, **f32)
                v = 0.1 * torch.randn(D, generator=g, **f32)
                heads = [torch.empty(M * D, **f32) for _ in range(4)]
                fn = lambda: pkcuda.call("pkcu_wmatmul_qkv", A.data_ptr(), w.handle, b.data_ptr(), u.data_ptr(),
                                         v.data_ptr(), *[t.data_ptr() for t in heads], seq.handle,
                                         work.data_ptr(), sh)
        ms = timed(fn)
        flop = 2.0 * M * N * K
        prods = 3 if bits == 8 else 6
        res[name] = {"M": M, "N": N, "K": K, "ms": round(ms, 4), "tflops_fp32": round(flop / ms / 1e9, 1),
                     "tensor_bf16_tflops": round(prods * flop / ms / 1e9, 1),
                     "tensor_frac_sustained": round(prods * flop / ms / 1e9 / peak, 3)}
        w.close()
        del A, b, work, out, keep
    torch.cuda.synchronize()
    res["peak_bf16_tflops_sustained"] = peak
    return res


FWD_UTTS = 32


def encoder_gemm_flops(T):
    """GEMM FLOPs of one conformer block per utterance of T frames (FF 2 x
    (1024x4096 + 4096x1024), QKV, output, positional on 2T-1 rows, the per-head
    score / positional-score / context products, the two pointwise convs)."""
    L = 2 * T - 1
    return 2 * (T * (2 * 2 * D * FF + D * 3 * D + D * D + 2 * D * D + D * D) + L * D * D
                + H * (T * T * DH + T * L * DH + T * T * DH))


def _synthetic_checkpoint(blank_bias=0.0):
    import tempfile
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import weights_fixture as wf
    d = tempfile.mkdtemp(prefix="pk_bench_ckpt_")
    _, bp, jp = wf.write_full_checkpoint(d, np.random.default_rng(5), blank_bias=blank_bias)
    return d, bp, jp


DEC_PROFILES = {"about_1_token_per_frame": 3.5, "10_tokens_every_frame": 0.0}


def decode_fmas(pending_rows, active_rows):
    """Multiply-adds of one fused decode iteration: per pending row both LSTM
    layers' gate products (2 x 2 x 2560 x 640), per active row the pred
    (640 x 640) and out (640 x 1025) products."""
    return pending_rows * 2 * 2 * 2560 * 640 + active_rows * (640 * 640 + 640 * 1025)


def time_decode_fused(stream, reps, n_utts=256, T=40, blank_shift=0.0):
    """pkcu_greedy_decode_fused on device-resident inputs: seeded random
    decoder weights and encoder projections; blank_shift raises the blank
    logit's bias (0: every frame emits the 10-symbol cap, every row pending
    every iteration; 3.5: a decoder step on a few rows per iteration).
    CUDA-event time of whole decodes divided by their iterations."""
    import numpy as np
    import torch
    import pkcuda
    rng = np.random.default_rng(5)
    Hd, V = 640, 1025
    g = lambda *shape, sd=1.0: torch.from_numpy((sd * rng.standard_normal(shape)).astype(np.float32)).cuda()
    # decoder parameters and weights in the reference's layouts (embedding
    # [1025, 640], LSTM biases [5120], joint biases; W_i / W_r [2560, 640],
    # joint.pred [640, 640], joint.out [640, 1025] as (in, out))
    dp = {"embed": g(V, Hd, sd=0.5), "lstm0_b": g(8 * Hd, sd=0.1), "lstm1_b": g(8 * Hd, sd=0.1),
          "joint_enc_b": g(Hd, sd=0.1), "joint_pred_b": g(Hd, sd=0.1), "joint_out_b": g(V, sd=0.1)}
    dp["joint_out_b"][V - 1] += blank_shift   # the blank token's bias
    s = 1.0 / np.sqrt(Hd)
    w = {"lstm0_wi": g(4 * Hd, Hd, sd=s), "lstm0_wr": g(4 * Hd, Hd, sd=s), "lstm1_wi": g(4 * Hd, Hd, sd=s),
         "lstm1_wr": g(4 * Hd, Hd, sd=s), "joint_pred": g(Hd, Hd, sd=s), "joint_out": g(Hd, V, sd=s)}
    with pkcuda.Decoder([T] * n_utts) as dec:
        enc = torch.as_tensor(_DevView(dec.gemm_out["enc"], n_utts * T * 640), device="cuda")
        enc.copy_(torch.randn(n_utts * T * 640, generator=torch.Generator(device="cuda").manual_seed(7),
                              device="cuda"))
        dec.set_weights(w, stream)
        dec.decode_fused(dp, stream)
        torch.cuda.synchronize()
        best = None
        for _ in range(max(reps, 1)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            dec.decode_fused(dp, stream)
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        n_tok, evals, _ = dec.results()
        iters = dec.iterations
    n_ev = int(evals.sum())
    # every evaluation is one active row of an iteration; the decoder steps are
    # the tokens plus the first step of each utterance
    fma = decode_fmas(int(n_tok.sum()) + n_utts, n_ev)
    return {"utterances": n_utts, "frames": T, "blank_shift": blank_shift, "iterations": iters,
            "us_per_iteration": round(best * 1000 / iters, 2), "joint_evals_per_s": round(n_ev / best * 1000),
            "tokens": int(n_tok.sum()), "fp32_tflops": round(2 * fma / best / 1e9, 2)}


def time_asr_decode(stream, reps, n_utts=256, T=375, cpu=True):
    """pkcu_asr_decode (the decode alone, a batched pk_greedy_decode with the
    model's own product kernels) on n_utts x T encoder frames of N(0, 1),
    through the public API (host tokens out), for two emission profiles set by
    the checkpoint's blank bias; beside each, the reference's own
    pk_greedy_decode on one such utterance (its sgemv products, host cores)."""
    import shutil
    import numpy as np
    import torch
    import pkcuda
    out = {}
    for name, bb in DEC_PROFILES.items():
        d, bp, jp = _synthetic_checkpoint(blank_bias=bb)
        try:
            enc = np.random.default_rng(21).standard_normal((n_utts * T, D)).astype(np.float32)
            modes = {}
            with pkcuda.Weights(bp, jp) as w:
                w.upload(stream)
                with pkcuda.ASR(w, stream) as asr:
                    x = torch.from_numpy(enc).cuda()
                    for mname, mode in (("fused_cuda_cores", asr.DECODE_FUSED), ("tcgen05", asr.DECODE_TC)):
                        asr.set_decode_mode(mode)
                        toks = asr.decode(x, [T] * n_utts, stream)
                        torch.cuda.synchronize()
                        t0 = time.perf_counter()
                        for _ in range(max(reps, 1)):
                            toks = asr.decode(x, [T] * n_utts, stream)
                        modes[mname] = ((time.perf_counter() - t0) / max(reps, 1), toks)
            dt, toks = min(modes.values(), key=lambda v: v[0])
            same = all(len(a) == len(b) and (a == b).all() for a, b in zip(modes["fused_cuda_cores"][1],
                                                                          modes["tcgen05"][1]))
            ntok = int(sum(len(t) for t in toks))
            r = {"utterances": n_utts, "frames": T, "blank_bias": bb, "seconds_per_call": round(dt, 4),
                 "frames_per_s": round(n_utts * T / dt), "tokens_per_frame": round(ntok / (n_utts * T), 3),
                 "seconds_per_call_by_mode": {k: round(v[0], 4) for k, v in modes.items()},
                 "modes_agree": bool(same)}
            if cpu:
                r["cpu_baseline"] = _cpu_ref_decode(bp, jp, enc[:T], T)
            out[name] = r
        finally:
            shutil.rmtree(d, ignore_errors=True)
    out["note"] = ("host wall clock of the synchronous call after a first call with the same lengths "
                   "(which creates the decoder and captures its graph): the encoder projection, the "
                   "decode graph, tokens copied to the host")
    return out


def _cpu_ref_decode(bp, jp, enc, T):
    """The reference's pk_greedy_decode on one utterance's encoder rows."""
    cores = os.cpu_count() or 1
    os.environ.setdefault("PK_THREADS", str(min(cores, 16)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import tempfile
    import numpy as np
    import pyoracle as po
    if not po.ref_full_available():
        return {"unavailable": "oracle/_ref/libpkref_full.so not built"}
    with tempfile.TemporaryDirectory() as td:
        ep = os.path.join(td, "enc.npy")
        np.save(ep, np.ascontiguousarray(enc, np.float32))
        code = ("import ctypes as C, sys, time, numpy as np; L = C.CDLL(sys.argv[1]); "
                "L.pkref_model_load.argtypes = [C.c_char_p, C.c_char_p]; "
                "L.pkref_model_decode.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]; "
                "assert L.pkref_model_load(sys.argv[2].encode(), sys.argv[3].encode()) == 0; "
                "e = np.load(sys.argv[4]); tok = np.zeros(10 * e.shape[0], np.int32); "
                "t0 = time.perf_counter(); n = L.pkref_model_decode(e.ctypes.data, e.shape[0], tok.ctypes.data, tok.size); "
                "print(time.perf_counter() - t0, n)")
        o = subprocess.run([sys.executable, "-c", code, po.LIB_REF_FULL, bp, jp, ep], capture_output=True,
                           text=True, check=True, env={**os.environ, "MALLOC_PERTURB_": "255"}).stdout.split()
    dt, n = float(o[-2]), int(o[-1])
    return {"value": round(T / dt, 1), "unit": "frames/s", "cores": int(os.environ["PK_THREADS"]),
            "kind": "reference", "sample": f"1 utterance of {T} encoder frames through the reference's "
                                           f"pk_greedy_decode, {dt:.2f} s, {n} tokens"}


def time_encoder_forward(stream, reps, n_utts=FWD_UTTS, T=375):
    """pkcu_encoder_forward: all 24 blocks, GEMMs included (the tcgen05
    FastFP32 GEMM for the row-major projections, cuBLAS fp32 for the rest, on
    fp32 weights), over n_utts x T frames of a synthetic checkpoint in the
    reference's format (int8 projections dequantised once)."""
    import shutil
    import torch
    import pkcuda
    d, bp, jp = _synthetic_checkpoint()
    try:
        with pkcuda.Weights(bp, jp) as w:
            w.upload(stream)
            with pkcuda.EncoderModel(w, stream) as em, pkcuda.Seq([T] * n_utts) as seq:
                ws = pkcuda.EncoderWorkspace(seq, 1)
                xa, gout, gin = ws.device()
                x = torch.as_tensor(_DevView(xa, n_utts * T * D), device="cuda")
                x.copy_(torch.randn(n_utts * T * D, device="cuda"))
                em.forward(xa, gout, gin, seq, stream)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(max(reps, 1)):
                    em.forward(xa, gout, gin, seq, stream)
                e1.record(stream)
                e1.synchronize()
                ms = e0.elapsed_time(e1) / max(reps, 1)
                ws.close()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    flop = 24 * n_utts * encoder_gemm_flops(T)
    return {"utterances": n_utts, "frames": T, "blocks": 24, "ms": round(ms, 3),
            "frames_per_s": round(n_utts * T / (ms * 1e-3)),
            "gemm_tflops_fp32": round(flop / (ms * 1e-3) / 1e12, 1)}


def cpu_encoder_baseline(T=375):
    """The reference's own pk_encoder (oracle/_ref/libpkref_full.so, its GEMMs
    included, PK_THREADS = min(cores, 16)) on one utterance of T frames of the
    same synthetic checkpoint; the load is outside the timed call."""
    import shutil
    import numpy as np
    cores = os.cpu_count() or 1
    os.environ.setdefault("PK_THREADS", str(min(cores, 16)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    if not po.ref_full_available():
        return {"unavailable": "oracle/_ref/libpkref_full.so not built"}
    d, bp, jp = _synthetic_checkpoint()
    try:
        lib = C.CDLL(po.LIB_REF_FULL)
        lib.pkref_model_load.argtypes = [C.c_char_p, C.c_char_p]
        lib.pkref_model_encode.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_longlong]
        if lib.pkref_model_load(bp.encode(), jp.encode()) != 0:
            return {"unavailable": "reference failed to load the synthetic checkpoint"}
        mel = np.random.default_rng(7).standard_normal((128, 8 * T)).astype(np.float32)
        t0 = time.perf_counter()
        tp = lib.pkref_model_encode(mel.ctypes.data, 8 * T, None, 0)
        dt = time.perf_counter() - t0
        lib.pkref_model_free()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return {"value": round(tp / dt, 1), "unit": "frames/s", "cores": int(os.environ["PK_THREADS"]),
            "kind": "reference", "sample": f"1 utterance of {8 * T} mel frames ({tp} encoder frames) "
                                           f"through the reference's pk_encoder, {dt:.2f} s"}


ASR_UTTS, ASR_MEL = 32, 3000


def time_asr(stream, reps, n_utts=ASR_UTTS, mel_frames=ASR_MEL, blank_bias=0.0):
    """pkcu_asr_transcribe: n_utts spectrograms of 3000 mel frames (30 s each)
    to tokens -- pre-encode, 24 blocks, greedy decode, every GEMM done by the
    library -- on a synthetic checkpoint in the reference's format (blank bias
    0: its random weights emit the 10-symbol cap on every frame, the decode's
    worst case)."""
    import shutil
    import torch
    import pkcuda
    d, bp, jp = _synthetic_checkpoint(blank_bias=blank_bias)
    try:
        with pkcuda.Weights(bp, jp) as w:
            w.upload(stream)
            with pkcuda.ASR(w, stream) as asr:
                g = torch.Generator(device="cuda")
                g.manual_seed(13)
                mel = torch.randn(n_utts * 128 * mel_frames, generator=g, device="cuda")
                frames = [mel_frames] * n_utts
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                out = asr.transcribe(mel, frames, stream)
                first = time.perf_counter() - t0
                t0 = time.perf_counter()
                for _ in range(max(reps, 1)):
                    out = asr.transcribe(mel, frames, stream)
                dt = (time.perf_counter() - t0) / max(reps, 1)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    enc = n_utts * (((mel_frames + 1) // 2 + 1) // 2 + 1) // 2
    ntok = int(sum(len(o) for o in out))
    return {"utterances": n_utts, "mel_frames": mel_frames, "blank_bias": blank_bias,
            "seconds_per_call": round(dt, 4),
            "utterances_per_s": round(n_utts / dt, 2), "encoder_frames_per_s": round(enc / dt),
            "audio_seconds_per_s": round(n_utts * mel_frames / 100.0 / dt, 1),
            "tokens": ntok, "tokens_per_frame": round(ntok / enc, 3),
            "first_call_s": round(first, 4),
            "note": "host wall clock of the synchronous call with spectrograms on the device; after the "
                    "first call (which allocates the working buffers and captures the decode graph) "
                    "the same lengths reuse them"}


def cpu_asr_baseline(mel_frames=ASR_MEL):
    """The reference's own pk_encoder + pk_greedy_decode on one 30 s
    utterance of the same synthetic checkpoint (load outside the timed call;
    run with allocations zeroed, see tests/test_pipeline_gpu.py)."""
    import shutil
    cores = os.cpu_count() or 1
    os.environ.setdefault("PK_THREADS", str(min(cores, 16)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    if not po.ref_full_available():
        return {"unavailable": "oracle/_ref/libpkref_full.so not built"}
    d, bp, jp = _synthetic_checkpoint()
    code = ("import ctypes as C, sys, time, numpy as np; L = C.CDLL(sys.argv[1]); "
            "L.pkref_model_load.argtypes = [C.c_char_p, C.c_char_p]; "
            "L.pkref_model_transcribe.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int]; "
            "assert L.pkref_model_load(sys.argv[2].encode(), sys.argv[3].encode()) == 0; "
            "T = int(sys.argv[4]); mel = np.random.default_rng(7).standard_normal((128, T)).astype(np.float32); "
            "tok = np.zeros(10 * T, np.int32); t0 = time.perf_counter(); "
            "n = L.pkref_model_transcribe(mel.ctypes.data, T, tok.ctypes.data, tok.size); "
            "print(time.perf_counter() - t0, n)")
    try:
        out = subprocess.run([sys.executable, "-c", code, po.LIB_REF_FULL, bp, jp, str(mel_frames)],
                             capture_output=True, text=True, check=True,
                             env={**os.environ, "MALLOC_PERTURB_": "255"}).stdout.split()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    dt, n = float(out[-2]), int(out[-1])
    return {"value": round(1.0 / dt, 4), "unit": "utterances/s", "cores": int(os.environ["PK_THREADS"]),
            "kind": "reference", "sample": f"1 utterance of {mel_frames} mel frames through the "
                                           f"reference's pk_encoder + pk_greedy_decode, {dt:.2f} s, "
                                           f"{n} tokens"}


DEC_UTTS, DEC_T = 256, 375


def time_decode(stream, reps):
    """pkcu_greedy_decode over 256 utterances x 375 encoder frames with the
    products resident as seeded stand-ins (no hook: the products are GEMMs
    outside the path). Static products make every utterance either always
    advance (blank wins: 375 iterations, joint + argmax only) or always emit
    (the 10-symbol cap on every frame: 3750 iterations, both LSTM layers on
    every row). Reported per case: device time per decode, per iteration, and
    joint evaluations per second."""
    import torch
    import pkcuda
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(10)
    f32 = dict(device=dev, dtype=torch.float32)
    B, T = DEC_UTTS, DEC_T
    params = {"embed": 0.5 * torch.randn(1025 * 640, generator=g, **f32),
              "lstm0_b": 0.1 * torch.randn(5120, generator=g, **f32),
              "lstm1_b": 0.1 * torch.randn(5120, generator=g, **f32),
              "joint_enc_b": 0.1 * torch.randn(640, generator=g, **f32),
              "joint_pred_b": 0.1 * torch.randn(640, generator=g, **f32),
              "joint_out_b": 0.1 * torch.randn(1025, generator=g, **f32)}
    res = {}
    with pkcuda.Decoder([T] * B) as dec:
        sizes = {"enc": B * T * 640, "pred": B * 640, "out": B * 1025, "g0i": B * 2560,
                 "g0r": B * 2560, "g1i": B * 2560, "g1r": B * 2560}
        views = {k: torch.as_tensor(_DevView(dec.gemm_out[k], n), device=dev) for k, n in sizes.items()}
        for k, v in views.items():
            v.copy_(torch.randn(v.numel(), generator=g, **f32))
        out = views["out"].view(B, 1025)
        for case, blank in (("decode_all_blank", 100.0), ("decode_always_emit", -100.0)):
            out[:, 1024] = blank
            dec.decode(params, stream=stream)          # warm-up
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(max(reps, 1)):
                dec.decode(params, stream=stream)
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / max(reps, 1)
            it = dec.iterations
            n_tok, evals, _ = dec.results()
            res[case] = {"utterances": B, "frames": T, "ms": round(ms, 4), "iterations": it,
                         "us_per_iteration": round(1e3 * ms / it, 3),
                         "joint_evals_per_s": round(int(evals.sum()) / (ms * 1e-3)),
                         "tokens": int(n_tok.sum()), "frames_per_s": round(B * T / (ms * 1e-3))}
    return res


def cpu_decode_baseline(T=DEC_T, seconds=1.0):
    """The reference's own pk_greedy_decode (oracle/_ref/libpkref_dec.so) on
    the host, one core, with the same static-product cases as time_decode:
    joint evaluations per second per case over a bounded sample of utterances."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    if not po.ref_dec_available():
        return {"unavailable": "oracle/_ref/libpkref_dec.so not built"}
    rng = np.random.default_rng(11)
    params = po.random_dec_params(rng)
    t = po.random_dec_products(rng, T, 0.0, max_iters=1)
    rows = {k: (t[k] if k == "enc" else t[k][0].copy()) for k in po.DEC_PRODUCTS}
    out = {"cores": 1, "kind": "reference", "unit": "joint evaluations/s"}
    for case, blank in (("decode_all_blank", 100.0), ("decode_always_emit", -100.0)):
        rows["out"][po.DEC_BLANK] = blank
        n_utts, evals, t0 = 0, 0, time.perf_counter()
        while n_utts < 1 or time.perf_counter() - t0 < seconds / 2:
            evals += po.reference_greedy_decode_static(T, params, rows)[1]
            n_utts += 1
        dt = time.perf_counter() - t0
        out[case] = {"joint_evals_per_s": round(evals / dt), "utterances": n_utts, "seconds": round(dt, 3)}
    out["sample"] = (f"utterances of T={T} decoded one after another through the reference's "
                     f"pk_greedy_decode, products served from fixed rows in C")
    return out


class _DevView:
    """A device address seen as a 1-D float32 array (the CUDA array interface)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (int(ptr), False),
                                         "version": 3}


PRE_UTTS, PRE_MEL_T = 64, 3000


def pre_encode_bytes(n, T):
    """Algorithmic bytes of the pre-encode kernels for n utterances of T mel
    frames (each input read once, each output written once; weights ignored)."""
    h1 = (T + 1) // 2
    h2 = (h1 + 1) // 2
    h3 = (h2 + 1) // 2
    s2, s3 = 4 * 256 * 32 * h2, 4 * 256 * 16 * h3
    return {"pre_conv0_dw2": n * (4 * 128 * T + s2), "pre_dw5": n * (s2 + s3),
            "pre_flatten": n * (s3 + 4 * 4096 * h3), "pre_out_scale": n * 8 * 1024 * h3}


def time_pre_encode(stream, reps, n_utts=PRE_UTTS):
    """pkcu_pre_encode over 64 utterances x 3000 mel frames (30 s each ->
    375 frames), GEMM products as seeded stand-ins. A GEMM hook records a CUDA
    event at each GEMM point, which splits the stage into its four kernels."""
    import torch
    import pkcuda
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    f32 = dict(device=dev, dtype=torch.float32)
    n, T = n_utts, PRE_MEL_T
    plan = pkcuda.PrePlan([T] * n)
    P2, P3, F = plan.p2, plan.p3, plan.frames
    mel = torch.randn(n * 128 * T, generator=g, **f32)
    params = {k: 0.3 * torch.randn(1024 if k == "out_b" else 256 * (9 if k.endswith("_w") else 1),
                                   generator=g, **f32) for k in pkcuda.PRE_PARAM_FIELDS}
    gout = {"pw1": torch.randn(256 * P2, generator=g, **f32),
            "pw2": torch.randn(256 * P3, generator=g, **f32),
            "proj": torch.randn(F * 1024, generator=g, **f32)}
    gin = {"s2d": torch.empty(256 * P2, **f32), "s3d": torch.empty(256 * P3, **f32),
           "flat": torch.empty(F * 4096, **f32)}
    x = torch.empty(F * 1024, **f32)
    marks = []

    def on_gemm(user, block, gemm, s):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        marks.append(ev)
        return 0

    hook = pkcuda.GEMM_HOOK(on_gemm)

    def once():
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        marks.append(ev)
        pkcuda.pre_encode(mel, params, gout, gin, x, plan, hook=hook, stream=stream)
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        marks.append(ev)

    once()
    torch.cuda.synchronize()
    names = ("pre_conv0_dw2", "pre_dw5", "pre_flatten", "pre_out_scale")
    ms = dict.fromkeys(names, 0.0)
    for _ in range(max(reps, 1)):
        marks.clear()
        once()
        marks[-1].synchronize()
        for i, k in enumerate(names):
            ms[k] += marks[i].elapsed_time(marks[i + 1]) / max(reps, 1)
    nb = pre_encode_bytes(n, T)
    res = {k: {"shape": [n, 128, T], "ms": ms[k], "bytes": nb[k],
               "gbs": nb[k] / (ms[k] * 1e-3) / 1e9} for k in names}
    tot_ms, tot_b = sum(ms.values()), sum(nb.values())
    res["pre_encode_stage"] = {"shape": [n, 128, T], "ms": tot_ms, "bytes": tot_b,
                               "gbs": tot_b / (tot_ms * 1e-3) / 1e9,
                               "frames_per_s": n * ((((T + 1) // 2 + 1) // 2 + 1) // 2) / (tot_ms * 1e-3)}
    plan.close()
    return res


def aux_only(args, local_rank):
    import torch
    import pkcuda
    torch.cuda.set_device(local_rank)
    pkcuda.lib()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        if args.decode_fused_only:
            print(json.dumps({"decode_fused": time_decode_fused(stream, args.aux_reps, args.dec_utts,
                                                                args.dec_frames, args.dec_shift)}), flush=True)
            return
        if args.asr_decode_only:
            print(json.dumps({"asr_decode": time_asr_decode(stream, args.aux_reps,
                                                            cpu=not args.no_cpu_baseline)}), flush=True)
            return
        if args.asr_only:
            asr = time_asr(stream, args.aux_reps)
            asr["every_frame_blank"] = time_asr(stream, args.aux_reps, blank_bias=6.0)
            if not args.no_cpu_baseline:
                asr["cpu_baseline"] = cpu_asr_baseline()
            print(json.dumps({"asr": asr}), flush=True)
            return
        if args.forward_only:
            fwd = time_encoder_forward(stream, args.aux_reps)
            if not args.no_cpu_baseline:
                fwd["cpu_baseline"] = cpu_encoder_baseline()
            print(json.dumps({"encoder_forward": fwd}), flush=True)
            return
        if args.gemm_only:
            print(json.dumps({"tc_gemms": time_tc_gemms(stream, args.aux_reps, args.gemm_rows),
                              "fused_gemms_fastfp32": time_fused_gemms(stream, args.aux_reps, args.gemm_rows)}),
                  flush=True)
            return
        if args.decode_only:
            dec = time_decode(stream, args.aux_reps)
            if not args.no_cpu_baseline:
                dec["cpu_baseline"] = cpu_decode_baseline()
            print(json.dumps({"decode": dec}), flush=True)
            return
        aux = time_aux_kernels(stream, reps=args.aux_reps, pre_utts=args.pre_utts,
                               pre_only=args.pre_only)
    peak, peak_kind = measured_peak()
    print(json.dumps({"kernels_aux": {k: {**v, "frac": v["gbs"] / peak if v["gbs"] else None}
                                      for k, v in aux.items()},
                      "peak_gbs": peak, "peak_kind": peak_kind}), flush=True)


def ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import pkcuda

    torch.cuda.set_device(local_rank)
    pkcuda.lib()
    stream = torch.cuda.Stream()        # graphs cannot be captured on the legacy stream
    with torch.cuda.stream(stream):
        _ours(args, rank, world, local_rank, stream)


def _ours(args, rank, world, local_rank, stream):
    import torch
    import torch.distributed as dist
    import pkcuda
    seq, ws, x_addr, gout, gin, blocks, arr = setup_device(args, rank, world)
    F = seq.frames

    def step():
        pkcuda.call("pkcu_encoder_nongemm", x_addr, C.cast(arr, pkcuda.VP), args.blocks,
                    C.byref(gout), C.byref(gin), seq.handle, None, None, stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        graph.replay()
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        run()
    e1.record(stream)
    e1.synchronize()
    t1 = time.time()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(t0, t1)
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, world, device="cuda")
    frames_all = F * args.steps * world
    value = frames_all / (ms_max / 1e3)
    bytes_step = step_bytes(F, args.T, args.utts, args.blocks)
    hbm_gbs = bytes_step * args.steps / (ms / 1e3) / 1e9

    # Per-kernel device times (each kernel alone over the full batch).
    table = time_kernels(args, seq, x_addr, gout, gin, blocks, stream)

    # End to end through the host-buffer C entry point (pinned host memory).
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, ws, arr, gout, x_addr, stream, world)

    used_graph = graph is not None
    del graph
    aux = cfg3 = cfg5 = None
    if rank == 0 and not args.no_aux:
        aux = time_aux_kernels(stream)
        cfg3 = time_config3(args, stream)
        cfg5 = time_config5(stream)
    if rank == 0 and args.extras:
        print(json.dumps({"extras": run_extras(args, stream, world)}), flush=True)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = RefRunner(args.T, args.blocks)
        fps, n_utts, secs = r.sample(args.cpu_seconds)
        cpu = {"value": fps, "unit": "frames/s", "cores": r.threads, "kind": "reference",
               "sample": f"{n_utts} utterance(s) x T={args.T} x {args.blocks} blocks through the "
                         f"reference's own conformer_block (GEMMs as no-ops), "
                         f"PK_THREADS={r.threads}, {secs:.1f} s"}
    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    dom = max(table, key=lambda k: table[k]["ms"] * table[k]["launches_per_step"])
    d = table[dom]
    traffic = ncu_traffic(dom)
    fr = lambda gbs: round(gbs / peak, 3)
    line = {
        "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) GEMM outputs and inputs, random block parameters)",
        "config": config_dict(args, world),
        "gpu_launches": pkcuda.lib().pkcu_encoder_nongemm_launches(args.blocks) * args.steps,
        "graph": used_graph,
        "clocks": clocks,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "hbm": {"bytes_per_step": bytes_step, "gbs": round(hbm_gbs, 1), "frac": round(hbm_gbs / peak, 3)},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": d["gbs"], "peak": peak,
                     "unit": "GB/s", "frac": d["gbs"] / peak, "traffic": traffic,
                     "peak_kind": peak_kind},
    }
    if cfg3 is not None:
        line["config3"] = {**cfg3, "frac": fr(cfg3["gbs"])}
    if cfg5 is not None:
        line["config5_frac"] = {k: fr(v["gbs"]) for k, v in cfg5.items()}
        line["config5_us"] = {k: v["us"] for k, v in cfg5.items()}
    if aux is not None:
        # standalone entry points at sizes above the L2: fraction of the measured copy peak
        line["kernels_aux_frac"] = {k: fr(v["gbs"]) for k, v in aux.items() if v.get("gbs")}
    # the sequence's kernels, each alone over the full batch: [ms, GB/s, fraction]
    line["kernels"] = {k: [round(v["ms"], 3), round(v["gbs"]), fr(v["gbs"])] for k, v in table.items()}
    print(json.dumps(line), flush=True)


def run_extras(args, stream, world):
    """The steps beyond the non-GEMM path, on rank 0 after the timed region:
    batched greedy decode, fused-epilogue GEMMs, the encoder with its GEMMs,
    mel-to-tokens and the decode alone, each beside the reference's own code
    on the host where one exists."""
    cpu = world == 1 and not args.no_cpu_baseline
    ex = {"decode": time_decode(stream, 3), "tc_gemms": time_tc_gemms(stream, 3),
          "fused_gemms_fastfp32": time_fused_gemms(stream, 3),
          "encoder_forward": time_encoder_forward(stream, 2)}
    asr = time_asr(stream, 1)
    asr["every_frame_blank"] = {k: v for k, v in time_asr(stream, 1, blank_bias=6.0).items()
                                if k in ("blank_bias", "seconds_per_call", "utterances_per_s",
                                         "audio_seconds_per_s", "tokens_per_frame")}
    ex["asr"] = asr
    ex["asr_decode"] = time_asr_decode(stream, 2, cpu=cpu)
    ex["decode_fused"] = {"10_tokens_every_frame": time_decode_fused(stream, 2, 256, 40, 0.0),
                          "sparse_decoder_steps": time_decode_fused(stream, 2, 256, 200, 3.5)}
    if cpu:
        ex["encoder_forward"]["cpu_baseline"] = cpu_encoder_baseline()
        ex["asr"]["cpu_baseline"] = cpu_asr_baseline()
        ex["decode"]["cpu_baseline"] = cpu_decode_baseline()
    return ex


def run_e2e(args, ws, arr, gout, x_addr, stream, world):
    """frames/s through pkcu_encoder_nongemm_host: every step copies x and the
    GEMM outputs from pinned host memory and x back (max over ranks)."""
    import torch
    import torch.distributed as dist
    import pkcuda
    seq = ws.seq
    F = seq.frames
    # Pinned host copies of x and the GEMM outputs: skip the run (and say so)
    # unless every local rank's copy fits well inside the host's free memory.
    need = (ws.h2d_bytes + ws.d2h_bytes) * int(os.environ.get("LOCAL_WORLD_SIZE", world))
    avail = 0
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    if need > 0.4 * avail:
        return {"unavailable": f"pinned host buffers need {need / 1e9:.1f} GB, "
                               f"host has {avail / 1e9:.1f} GB available"}
    host = {}
    for f in pkcuda.GEMM_OUT_FIELDS:
        addr = getattr(gout, f)
        n = {"ff1_h": F * FF, "ff2_h": F * FF, "qkv": 3 * F * D, "P": seq.pos_rows * D,
             "ac": seq.score_elems, "bd": seq.bd_elems, "pw1": 2 * F * D}.get(f, F * D)
        h = torch.empty(n, dtype=torch.float32, pin_memory=True)
        h.copy_(tensor_at(addr, n))
        host[f] = h
    xh = torch.empty(F * D, dtype=torch.float32, pin_memory=True)
    xh.copy_(tensor_at(x_addr, F * D))
    gh = pkcuda.gemm_outputs(host)
    steps = max(2, min(args.steps, 5))
    ws.run_host(xh.data_ptr(), gh, arr, args.blocks, stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        ws.run_host(xh.data_ptr(), gh, arr, args.blocks, stream)
    secs = max_over_ranks(time.perf_counter() - t0, world, device="cuda")
    # The host-link ceiling this path meets: the same page-locked buffers
    # copied to the same device buffers with nothing else running, every rank
    # at once (barrier, then max over ranks), H2D and D2H as in one step.
    dst = [(tensor_at(getattr(gout, f), host[f].numel()), host[f]) for f in pkcuda.GEMM_OUT_FIELDS]
    dst.append((tensor_at(x_addr, F * D), xh))

    def copies():
        with torch.cuda.stream(stream):
            for d, h in dst:
                d.copy_(h, non_blocking=True)
            xh.copy_(tensor_at(x_addr, F * D), non_blocking=True)
        stream.synchronize()

    copies()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        copies()
    csecs = max_over_ranks(time.perf_counter() - t0, world, device="cuda")
    ceiling = (ws.h2d_bytes + ws.d2h_bytes) * steps / csecs / 1e9
    achieved = (ws.h2d_bytes + ws.d2h_bytes) * steps / secs / 1e9
    return {"value": F * steps * world / secs, "unit": "frames/s", "steps": steps,
            "h2d_bytes_per_step": ws.h2d_bytes, "d2h_bytes_per_step": ws.d2h_bytes,
            "pipeline_groups": args.groups,
            "host_link_gbs_per_rank": round(achieved, 1),
            "copy_only_ceiling_gbs_per_rank": round(ceiling, 1),
            "frac_of_copy_ceiling": round(achieved / ceiling, 3),
            "note": "pkcu_encoder_nongemm_host, host clock, max over ranks"}


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.aux_only:
        if rank == 0:
            aux_only(args, local_rank)
        return
    if args.impl == "reference":
        if world > 1 and rank != 0:
            return
        reference_arm(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=dt.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
