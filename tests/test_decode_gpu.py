"""GPU parity of the batched greedy RNN-T decode (pkcu_greedy_decode) against
the restatement of csrc/decoder.c:80-132 (pinned to the reference's own
pk_greedy_decode on the CPU).

The matrix-vector products are stand-ins: each utterance has a seeded table of
products (pyoracle.random_dec_products), and the test's GEMM hook writes row b
of every batched product from utterance b's table at the current iteration.
The restatement replays each utterance alone with the same table, so the two
decodes see the same products, and:
  * tokens, token counts and joint evaluations per utterance match exactly;
  * the joint hidden rows (the input of joint.out) match bit for bit, and so
    do the embedding rows fed to the LSTM;
  * the LSTM hidden states (inputs of W_r and joint.pred) match within the
    tolerance (CUDA expf / tanhf against glibc's).
"""
import contextlib

import numpy as np
import pytest

import pyoracle as po
from conftest import assert_bitexact, assert_close
from gpuhelp import _DeviceView, dev, from_device

pytestmark = pytest.mark.gpu

H, V = po.DEC_H, po.DEC_V
NAME = {32: "enc", 33: "l0_wi", 34: "l0_wr", 35: "l1_wi", 36: "l1_wr", 37: "pred", 38: "out"}
OUT_FIELD = {"enc": "enc", "pred": "pred", "out": "out", "l0_wi": "g0i", "l0_wr": "g0r",
             "l1_wi": "g1i", "l1_wr": "g1r"}
IN_FIELD = {"l0_wi": "x0", "l0_wr": "h0", "l1_wi": "h0", "l1_wr": "h1", "pred": "h1",
            "out": "hidden"}


def to_device(ptr, a):
    """Copies a host array into device memory at ptr (owned elsewhere)."""
    import torch
    from gpuhelp import _DeviceView
    a = np.ascontiguousarray(a, np.float32).reshape(-1)
    t = torch.as_tensor(_DeviceView(ptr, a.size, np.float32), device="cuda")
    t.copy_(torch.from_numpy(a))


class TableHook:
    """Batched products from per-utterance tables, iteration by iteration;
    records every product's input rows per iteration."""

    def __init__(self, cuda, dec, tables):
        self.dec, self.tables = dec, tables
        self.B = len(tables)
        self.iter = 0
        self.inputs = {k: [] for k in IN_FIELD}
        self.calls = []
        self.fn = cuda.GEMM_HOOK(self._hook)

    def _rows(self, name):
        n = V if name == "out" else (4 * H if name.startswith("l") else H)
        a = np.zeros((self.B, n), np.float32)
        for b, t in enumerate(self.tables):
            if self.iter < t[name].shape[0]:
                a[b] = t[name][self.iter]
        return a

    def _hook(self, user, block, gemm, stream):
        import torch
        name = NAME[gemm]
        self.calls.append(gemm)
        ctx = (torch.cuda.stream(torch.cuda.ExternalStream(stream)) if stream
               else contextlib.nullcontext())
        with ctx:
            if name == "enc":
                to_device(self.dec.gemm_out["enc"],
                          np.concatenate([t["enc"][:f] for t, f in zip(self.tables, self.dec.frames)]))
                return 0
            src = self.dec.gemm_in[IN_FIELD[name]]
            self.inputs[name].append(from_device(src, self.B * H, np.float32).reshape(self.B, H))
            to_device(self.dec.gemm_out[OUT_FIELD[name]], self._rows(name))
        if name == "out":
            self.iter += 1
        return 0


def device_params(params):
    return {"embed": dev(params["embed"]), "lstm0_b": dev(params["B0"]),
            "lstm1_b": dev(params["B1"]), "joint_enc_b": dev(params["enc_b"]),
            "joint_pred_b": dev(params["pred_b"]), "joint_out_b": dev(params["out_b"])}


def run_case(cuda, frames, p_blank, seed):
    rng = np.random.default_rng(seed)
    params = po.random_dec_params(rng)
    tables = [po.random_dec_products(rng, T, pb) for T, pb in zip(frames, p_blank)]
    with cuda.Decoder(frames) as dec:
        hook = TableHook(cuda, dec, tables)
        dec.decode(device_params(params), hook=hook.fn)
        n_tok, evals, tokens = dec.results()
        iters = dec.iterations
        h_final = from_device(dec.gemm_in["h0"], 2 * len(frames) * H, np.float32).reshape(2, -1, H)
    assert hook.calls[0] == 32 and hook.calls[1:7] == [33, 34, 35, 36, 37, 38]
    assert iters == hook.iter
    for b, (T, table) in enumerate(zip(frames, tables)):
        prod = po.DecodeProducts(table)
        tok_o, it_o, state = po.oracle_greedy_decode(T, params, prod)
        assert n_tok[b] == len(tok_o), (b, n_tok[b], len(tok_o))
        assert_bitexact(tokens[b], tok_o.astype(np.int32), f"tokens of utterance {b}")
        assert evals[b] == it_o, (b, evals[b], it_o)
        for k in range(it_o):
            assert_bitexact(hook.inputs["out"][k][b], prod.inputs["out"][k], f"hidden {b} iter {k}")
            assert_close(hook.inputs["pred"][k][b], prod.inputs["pred"][k], f"h1 {b} iter {k}")
        for k, x in prod.inputs["l0_wi"].items():
            assert_bitexact(hook.inputs["l0_wi"][k][b], x, f"embedding row {b} iter {k}")
            assert_close(hook.inputs["l0_wr"][k][b], prod.inputs["l0_wr"][k], f"h0 {b} iter {k}")
            assert_close(hook.inputs["l1_wr"][k][b], prod.inputs["l1_wr"][k], f"h1 {b} iter {k}")
        assert_close(h_final[0, b], state[0], f"final h0 {b}")
        assert_close(h_final[1, b], state[1], f"final h1 {b}")
    return n_tok, evals


def test_decode_ragged(cuda):
    """Ragged batch: one frame, the 10-symbol cap on every frame (p_blank 0),
    mostly-blank and all-blank utterances side by side."""
    n_tok, _ = run_case(cuda, [1, 5, 13, 40, 2, 3], [0.5, 0.0, 0.6, 0.8, 0.3, 1.0], seed=71)
    assert n_tok[1] == 50 and n_tok[5] == 0


def test_decode_uniform(cuda):
    run_case(cuda, [16] * 4, [0.7] * 4, seed=72)


def test_decode_batch64(cuda):
    rng = np.random.default_rng(73)
    frames = rng.integers(1, 60, size=64).tolist()
    p_blank = rng.uniform(0.5, 0.95, size=64).tolist()
    run_case(cuda, frames, p_blank, seed=74)


def test_decode_graph_no_hook(cuda):
    """Without a hook the decode replays a captured CUDA graph of 8 iterations;
    the products are whatever the caller left in the decoder's buffers (here
    one fixed row per utterance: it always emits -- the 10-symbol cap on every
    frame -- or always advances). Run twice to reuse the captured graph."""
    frames = [3, 7, 1, 12, 5, 9]
    emits = [True, False, True, False, False, True]
    rng = np.random.default_rng(75)
    params = po.random_dec_params(rng)
    rows = {k: [] for k in ("pred", "out", "l0_wi", "l0_wr", "l1_wi", "l1_wr")}
    tables = []
    for T, em in zip(frames, emits):
        t = po.random_dec_products(rng, T, 0.0, max_iters=1)
        t["out"][0, po.DEC_BLANK] = -100.0 if em else 100.0
        for k in rows:
            rows[k].append(t[k][0])
        n = 10 * T + 2
        tables.append({k: (v if k == "enc" else np.repeat(v, n, axis=0)) for k, v in t.items()})
    with cuda.Decoder(frames) as dec:
        to_device(dec.gemm_out["enc"], np.concatenate([t["enc"][:f] for t, f in zip(tables, frames)]))
        for k, f in (("pred", "pred"), ("out", "out"), ("l0_wi", "g0i"), ("l0_wr", "g0r"),
                     ("l1_wi", "g1i"), ("l1_wr", "g1r")):
            to_device(dec.gemm_out[f], np.stack(rows[k]))
        dp = device_params(params)
        for _ in range(2):
            dec.decode(dp)
            n_tok, evals, tokens = dec.results()
            need = max(10 * T + 1 if em else T for T, em in zip(frames, emits))
            assert dec.iterations % 8 == 0 and need <= dec.iterations < need + 8
            for b, (T, table) in enumerate(zip(frames, tables)):
                tok_o, it_o, _ = po.oracle_greedy_decode(T, params, po.DecodeProducts(table))
                assert_bitexact(tokens[b], tok_o.astype(np.int32), f"tokens {b}")
                assert evals[b] == it_o
                assert n_tok[b] == (10 * T if emits[b] else 0)


def test_decode_graph_with_hook(cuda):
    """pkcu_greedy_decode_graph: the hook's products are captured into the
    decoder's two 8-iteration graphs (here device-to-device copies of one fixed
    row per utterance, as in the test above); the hook is called 8 times per
    product for each graph while capturing and, on the second decode with the
    same hook, only for DEC_ENC."""
    import torch
    frames = [4, 9, 2, 6]
    emits = [False, True, True, False]
    rng = np.random.default_rng(76)
    params = po.random_dec_params(rng)
    rows = {k: [] for k in ("pred", "out", "l0_wi", "l0_wr", "l1_wi", "l1_wr")}
    tables = []
    for T, em in zip(frames, emits):
        t = po.random_dec_products(rng, T, 0.0, max_iters=1)
        t["out"][0, po.DEC_BLANK] = -100.0 if em else 100.0
        for k in rows:
            rows[k].append(t[k][0])
        n = 10 * T + 2
        tables.append({k: (v if k == "enc" else np.repeat(v, n, axis=0)) for k, v in t.items()})
    field = {"pred": "pred", "out": "out", "l0_wi": "g0i", "l0_wr": "g0r", "l1_wi": "g1i",
             "l1_wr": "g1r"}
    src = {k: torch.as_tensor(np.stack(v)).cuda() for k, v in rows.items()}
    enc = torch.as_tensor(np.concatenate([t["enc"][:f] for t, f in zip(tables, frames)])).cuda()
    calls = []
    with cuda.Decoder(frames) as dec:
        dst = {k: torch.as_tensor(_DeviceView(dec.gemm_out[field[k]], src[k].numel(), np.float32),
                                  device="cuda") for k in rows}
        enc_dst = torch.as_tensor(_DeviceView(dec.gemm_out["enc"], enc.numel(), np.float32),
                                  device="cuda")

        def hook(user, block, gemm, stream):
            name = NAME[gemm]
            calls.append(name)
            ctx = (torch.cuda.stream(torch.cuda.ExternalStream(stream)) if stream
                   else contextlib.nullcontext())
            with ctx:
                if name == "enc":
                    enc_dst.copy_(enc.reshape(-1))
                else:
                    dst[name].copy_(src[name].reshape(-1))
            return 0

        fn = cuda.GEMM_HOOK(hook)
        dp = device_params(params)
        torch.cuda.synchronize()
        for rep in range(2):
            calls.clear()
            dec.decode(dp, hook=fn, graph=True)
            n_tok, evals, tokens = dec.results()
            want_calls = 1 + (6 * 16 if rep == 0 else 0)   # 8 iterations x 2 graphs
            assert len(calls) == want_calls and calls[0] == "enc", (rep, len(calls))
            need = max(10 * T + 1 if em else T for T, em in zip(frames, emits))
            assert dec.iterations % 8 == 0 and need <= dec.iterations < need + 8
            for b, (T, table) in enumerate(zip(frames, tables)):
                tok_o, it_o, _ = po.oracle_greedy_decode(T, params, po.DecodeProducts(table))
                assert_bitexact(tokens[b], tok_o.astype(np.int32), f"tokens {b}")
                assert evals[b] == it_o


def test_decode_fused_matches_reference(cuda):
    """pkcu_greedy_decode_fused -- the decoder's own LSTM / joint product
    kernels -- on a ragged batch, against the restatement and the reference's
    own pk_greedy_decode, both fed products computed in float64 from the same
    weights (fp32 products in the kernels: tokens and joint evaluations
    exact, LSTM states within 1e-4; the seed's smallest top-2 logit gap is
    7e-4, far above the products' rounding). Decoded twice to replay the
    captured graph."""
    rng = np.random.default_rng(78)
    frames = [23, 5, 40, 1, 17, 31, 8, 12, 64, 3]
    B = len(frames)
    params = po.random_dec_params(rng)
    params["out_b"][po.DEC_BLANK] += 3.5      # about one token per frame
    weights = po.random_dec_weights(rng)
    encs = [rng.standard_normal((T, H)).astype(np.float32) for T in frames]
    with cuda.Decoder(frames) as dec:
        to_device(dec.gemm_out["enc"], np.concatenate(encs))
        dec.set_weights({k: dev(v) for k, v in weights.items()})
        dp = device_params(params)
        for _ in range(2):
            dec.decode_fused(dp)
            n_tok, evals, tokens = dec.results()
            h0 = from_device(dec.gemm_in["h0"], B * H, np.float32).reshape(B, H)
            h1 = from_device(dec.gemm_in["h1"], B * H, np.float32).reshape(B, H)
            assert dec.iterations % 8 == 0
            err = 0.0
            for b, T in enumerate(frames):
                tok_o, it_o, st_o = po.oracle_greedy_decode(
                    T, params, po.WeightProducts(weights, encs[b], params["out_b"]))
                tok_r, it_r = po.reference_greedy_decode(
                    T, params, po.WeightProducts(weights, encs[b], params["out_b"]))
                assert_bitexact(tok_o, tok_r, f"restatement vs reference, utterance {b}")
                assert it_o == it_r
                assert_bitexact(tokens[b], tok_o.astype(np.int32), f"tokens {b}")
                assert evals[b] == it_o and n_tok[b] == len(tok_o)
                err = max(err, float(np.abs(h0[b] - st_o[0]).max()), float(np.abs(h1[b] - st_o[1]).max()))
            assert err < 1e-4, err
    print(f"fused decode: {int(sum(n_tok))} tokens over {sum(frames)} frames, "
          f"max |h - oracle| = {err:.3g}")
