"""GPU parity of the pre-encode stage (pkcu_pre_encode) against the
restatement of csrc/encoder.c:103-175, 578-593 (pinned bit for bit to the
reference's own pre_encode_and_scale on the CPU).

A batch of utterances runs in one call; every GEMM input the stage produces
(s2d, s3d: the inputs of the two 1x1 convolutions; flat: the input of the
projection) and the blocks' input x are compared bit for bit, item by item.
"""
import contextlib

import numpy as np
import pytest

import pyoracle as po
from conftest import assert_bitexact
from gpuhelp import D, dev, empty, host

pytestmark = pytest.mark.gpu

C = po.PRE_C


class PreLayout:
    """Batch layout of the stage: [256, *] tensors are channel-major across the
    batch (row c = each item's plane in turn), time-first tensors are frames of
    every item in turn."""

    def __init__(self, lengths):
        self.T = list(lengths)
        self.dims = [po.pre_dims(t) for t in self.T]
        self.h2 = np.concatenate([[0], np.cumsum([d["H2"] for d in self.dims])]).astype(np.int64)
        self.h3 = np.concatenate([[0], np.cumsum([d["H3"] for d in self.dims])]).astype(np.int64)

    @property
    def P2(self):
        return int(self.h2[-1]) * 32

    @property
    def P3(self):
        return int(self.h3[-1]) * 16

    @property
    def frames(self):
        return int(self.h3[-1])

    def plane(self, a, i, stage):
        """Item i's [256, H*W] plane of a [256, P] batch tensor."""
        off, w = (self.h2, 32) if stage == 2 else (self.h3, 16)
        return a.reshape(C, -1)[:, off[i] * w:off[i + 1] * w]

    def rows(self, a, i, width):
        return a.reshape(-1, width)[self.h3[i]:self.h3[i + 1]]


def make_items(lengths, seed):
    r = np.random.default_rng(seed)
    params = None
    items = []
    for T in lengths:
        ps, si, mel = po.random_pre_inputs(r, T)
        params = params or ps
        items.append((si, mel))
    return params, items


def run_gpu(cuda, lengths, params, items, hook=None, params_on_device=False):
    """params: host arrays, or device addresses with params_on_device."""
    L = PreLayout(lengths)
    mel = dev(np.concatenate([m.reshape(-1) for _, m in items]))
    pd = dict(params) if params_on_device else {k: dev(v) for k, v in params.items()}
    gout = {"pw1": dev(np.concatenate([si["y2"] for si, _ in items], axis=1)),
            "pw2": dev(np.concatenate([si["y3"] for si, _ in items], axis=1)),
            "proj": dev(np.concatenate([si["proj"] for si, _ in items]))}
    gin = {"s2d": empty(C * L.P2), "s3d": empty(C * L.P3), "flat": empty(L.frames * 4096)}
    x = empty(L.frames * D)
    with cuda.PrePlan(lengths) as plan:
        assert (plan.p2, plan.p3, plan.frames) == (L.P2, L.P3, L.frames)
        if hook is not None:
            hook.bind(pd, gout, gin)
        cuda.pre_encode(mel, pd, gout, gin, x, plan, hook=hook.fn if hook else None)
        got = {k: host(v) for k, v in gin.items()}
        got["x"] = host(x)
        got.update({k: host(v) for k, v in gout.items()})
    return L, got


def check_items(oracle, L, got, params, items):
    for i, (si, mel) in enumerate(items):
        xo, caps = oracle.pre_encode(mel, params, si)
        assert_bitexact(L.plane(got["s2d"], i, 2), caps["s2d"], f"s2d item {i} (T={L.T[i]})")
        assert_bitexact(L.plane(got["s3d"], i, 3), caps["s3d"], f"s3d item {i}")
        assert_bitexact(L.rows(got["flat"], i, 4096), caps["flat"], f"flat item {i}")
        assert_bitexact(L.rows(got["x"], i, D), xo, f"x item {i}")


def test_pre_encode_golden(cuda, golden):
    """The reference's own outputs (tests/golden), one utterance of 11 frames."""
    params = {k: golden["pre_p_" + k] for k in po.PRE_PARAM_ROLES}
    si = {k: golden["pre_si_" + k] for k in ("y2", "y3", "proj")}
    L, got = run_gpu(cuda, [11], params, [(si, golden["pre_mel"])])
    assert_bitexact(L.plane(got["s2d"], 0, 2), golden["pre_cap_s2d"], "s2d")
    assert_bitexact(L.plane(got["s3d"], 0, 3), golden["pre_cap_s3d"], "s3d")
    assert_bitexact(L.rows(got["flat"], 0, 4096), golden["pre_cap_flat"], "flat")
    assert_bitexact(L.rows(got["x"], 0, D), golden["pre_x_out"], "x")


@pytest.mark.parametrize("lengths", [[1], [2], [3, 4, 5], [8, 1, 9, 16, 17],
                                     [257, 33, 100, 7], [3000, 3000], [3264, 3328, 3264]])
def test_pre_encode_batch(cuda, oracle, lengths):
    """Ragged and uniform batches, odd and even lengths down to one frame, the
    30 s utterance (3000 mel frames -> 375) and long-audio chunk lengths."""
    params, items = make_items(lengths, seed=sum(lengths))
    L, got = run_gpu(cuda, lengths, params, items)
    check_items(oracle, L, got, params, items)


class TorchGemmHook:
    """A pkcu_gemm_hook that runs the stage's three GEMMs with torch on the
    caller's stream: pw1 = W3 s2d, pw2 = W6 s3d, proj = flat W_out."""

    def __init__(self, cuda, seed):
        import torch
        r = np.random.default_rng(seed)
        self.w3 = dev((0.06 * r.standard_normal((C, C))).astype(np.float32))
        self.w6 = dev((0.06 * r.standard_normal((C, C))).astype(np.float32))
        self.wo = dev((0.02 * r.standard_normal((4096, D))).astype(np.float32))
        self.calls = []
        self.torch = torch
        self.fn = cuda.GEMM_HOOK(self._hook)

    def bind(self, pd, gout, gin):
        self.gout, self.gin = gout, gin

    def _hook(self, user, block, gemm, stream):
        t = self.torch
        self.calls.append((block, gemm))
        # stream None is the legacy default stream, torch's current one here
        with t.cuda.stream(t.cuda.ExternalStream(stream)) if stream else contextlib.nullcontext():
            if gemm == 16:
                s = self.gin["s2d"].view(C, -1)
                self.gout["pw1"].view(C, -1).copy_(self.w3 @ s)
            elif gemm == 17:
                s = self.gin["s3d"].view(C, -1)
                self.gout["pw2"].view(C, -1).copy_(self.w6 @ s)
            elif gemm == 18:
                f = self.gin["flat"].view(-1, 4096)
                self.gout["proj"].view(-1, D).copy_(f @ self.wo)
            else:
                return 1
        return 0


def test_pre_encode_gemm_hook(cuda, oracle):
    """GEMMs enqueued by the hook, in stream order, at the three GEMM points:
    the stage must consume each product only after the hook's work. The oracle
    is then fed the products the hook wrote."""
    lengths = [40, 13, 64]
    params, items = make_items(lengths, seed=5)
    hook = TorchGemmHook(cuda, seed=6)
    L, got = run_gpu(cuda, lengths, params, items, hook=hook)
    assert hook.calls == [(-1, 16), (-1, 17), (-1, 18)]
    for i, (_, mel) in enumerate(items):
        si = {"y2": np.ascontiguousarray(L.plane(got["pw1"], i, 2)),
              "y3": np.ascontiguousarray(L.plane(got["pw2"], i, 3)),
              "proj": np.ascontiguousarray(L.rows(got["proj"], i, D))}
        xo, caps = oracle.pre_encode(mel, params, si)
        assert_bitexact(L.plane(got["s2d"], i, 2), caps["s2d"], f"s2d {i}")
        assert_bitexact(L.plane(got["s3d"], i, 3), caps["s3d"], f"s3d {i}")
        assert_bitexact(L.rows(got["flat"], i, 4096), caps["flat"], f"flat {i}")
        assert_bitexact(L.rows(got["x"], i, D), xo, f"x {i}")
