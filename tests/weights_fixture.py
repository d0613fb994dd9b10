"""Checkpoint files in the reference's weights.bin / weights.json format, for
the loader tests.

Layout as the reference exporter writes it (extract_weights.py:894-945): every
tensor's bytes back to back in sorted-name order; manifest entries
{offset, shape, numel, dtype} plus "scale" for int8 and, for int4, the
packed [K, N/2] bytes followed by K*N/32 fp32 group scales at
"scales_offset" ("n_scales" of them). Numbers are written by json.dump, as the
exporter does. Names follow csrc/weights.c:330-376.

Blocks beyond the ones written with their own data can be added as aliases:
manifest entries that point at block 0's bytes. The reference loader builds
the fused QKV of all 24 blocks, so a file it can load needs 24 blocks of
q, k, v and their biases; aliases keep such files small."""
from __future__ import annotations

import json
import os

import numpy as np

D, H, DH, FF = 1024, 8, 128, 4096

# manifest name (after "layers.{b}.") of each non-GEMM block parameter
ROLE_NAMES = {
    "norm_ff1_w": "norm_feed_forward1.weight", "norm_ff1_b": "norm_feed_forward1.bias",
    "ff1_b1": "feed_forward1.linear1.bias", "ff1_b2": "feed_forward1.linear2.bias",
    "norm_sa_w": "norm_self_att.weight", "norm_sa_b": "norm_self_att.bias",
    "pos_u": "self_attn.pos_bias_u", "pos_v": "self_attn.pos_bias_v",
    "out_b": "self_attn.linear_out.bias", "norm_conv_w": "norm_conv.weight",
    "norm_conv_b": "norm_conv.bias", "pw1_b": "conv.pointwise_conv1.bias",
    "dw_w": "conv.depthwise_conv.weight", "dw_b": "conv.depthwise_conv.bias",
    "pw2_b": "conv.pointwise_conv2.bias", "norm_ff2_w": "norm_feed_forward2.weight",
    "norm_ff2_b": "norm_feed_forward2.bias", "ff2_b1": "feed_forward2.linear1.bias",
    "ff2_b2": "feed_forward2.linear2.bias", "norm_out_w": "norm_out.weight",
    "norm_out_b": "norm_out.bias",
}
ROLE_SHAPES = {"ff1_b1": (FF,), "ff2_b1": (FF,), "pos_u": (H, DH), "pos_v": (H, DH),
               "pw1_b": (2 * D,), "dw_w": (D, 1, 9)}
QKV = ("q", "k", "v")
MATRICES = {"self_attn.linear_q.weight": (D, D), "self_attn.linear_k.weight": (D, D),
            "self_attn.linear_v.weight": (D, D), "self_attn.linear_out.weight": (D, D),
            "self_attn.linear_pos.weight": (D, D), "feed_forward1.linear1.weight": (D, FF),
            "feed_forward1.linear2.weight": (FF, D), "feed_forward2.linear1.weight": (D, FF),
            "feed_forward2.linear2.weight": (FF, D)}


# pre-encode parameters the non-GEMM stage takes (csrc/weights.c:310-321), by role
PRE_NAMES = {"conv0_w": "pre_encode.conv.0.weight", "conv0_b": "pre_encode.conv.0.bias",
             "conv2_w": "pre_encode.conv.2.weight", "conv2_b": "pre_encode.conv.2.bias",
             "conv3_b": "pre_encode.conv.3.bias", "conv5_w": "pre_encode.conv.5.weight",
             "conv5_b": "pre_encode.conv.5.bias", "conv6_b": "pre_encode.conv.6.bias",
             "out_b": "pre_encode.out.bias"}


def pack_int4(q: np.ndarray) -> np.ndarray:
    """[K, N] values in [-8, 7] -> [K, N/2] bytes, even column in the low nibble."""
    return ((q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)).astype(np.uint8)


def make_tensors(rng, n_blocks: int, attn: str, ff: str) -> dict:
    """{name: {"data": array, "scale": float | None, "scales": array | None}}."""
    t = {}
    for role, nm in PRE_NAMES.items():
        shape = (256, 1, 3, 3) if role.endswith("_w") else (D if role == "out_b" else 256,)
        t[nm] = {"data": (0.3 * rng.standard_normal(shape)).astype(np.float32), "scale": None,
                 "scales": None}
    for b in range(n_blocks):
        for role, nm in ROLE_NAMES.items():
            shape = ROLE_SHAPES.get(role, (D,))
            if role.startswith("norm") and role.endswith("_w"):
                a = 1.0 + 0.1 * rng.standard_normal(shape)
            elif role == "dw_w":
                a = 0.3 * rng.standard_normal(shape)
            else:
                a = 0.1 * rng.standard_normal(shape)
            t[f"layers.{b}.{nm}"] = {"data": a.astype(np.float32), "scale": None, "scales": None}
        for m in QKV:
            t[f"layers.{b}.self_attn.linear_{m}.bias"] = {
                "data": (0.1 * rng.standard_normal(D)).astype(np.float32), "scale": None,
                "scales": None}
        for nm, (K, N) in MATRICES.items():
            kind = ff if nm.startswith("feed_forward") else attn
            if kind == "int8":
                t[f"layers.{b}.{nm}"] = {
                    "data": rng.integers(-127, 128, size=(K, N), dtype=np.int8),
                    "scale": float(rng.uniform(1e-3, 1e-2)), "scales": None}
            elif kind == "int4":
                q = rng.integers(-8, 8, size=(K, N)).astype(np.int8)
                t[f"layers.{b}.{nm}"] = {
                    "data": pack_int4(q), "scale": None,
                    "scales": rng.uniform(1e-3, 2e-2, size=(K, N // 32)).astype(np.float32)}
            else:
                t[f"layers.{b}.{nm}"] = {
                    "data": (0.05 * rng.standard_normal((K, N))).astype(np.float32),
                    "scale": None, "scales": None}
    return t


def write_checkpoint(dirpath, tensors: dict, alias_blocks: int = 0):
    """Writes weights.bin / weights.json; blocks 1 .. alias_blocks-1 missing
    from `tensors` get q, k, v (+ biases) entries that alias block 0's bytes."""
    bin_path = os.path.join(dirpath, "weights.bin")
    json_path = os.path.join(dirpath, "weights.json")
    manifest, offset = {}, 0
    with open(bin_path, "wb") as f:
        for name in sorted(tensors):
            w = tensors[name]
            arr = w["data"]
            data = arr.tobytes()
            f.write(data)
            if w["scales"] is not None:
                entry = {"offset": offset, "shape": list(arr.shape), "numel": int(arr.size),
                         "dtype": "int4"}
                offset += len(data)
                sd = w["scales"].astype(np.float32).tobytes()
                entry["scales_offset"] = offset
                entry["n_scales"] = int(w["scales"].size)
                f.write(sd)
                offset += len(sd)
            else:
                entry = {"offset": offset, "shape": list(arr.shape), "numel": int(arr.size),
                         "dtype": "int8" if arr.dtype == np.int8 else "float32"}
                if w["scale"] is not None:
                    entry["scale"] = w["scale"]
                offset += len(data)
            manifest[name] = entry
    for b in range(1, alias_blocks):
        for m in QKV:
            for kind in ("weight", "bias"):
                nm = f"layers.{b}.self_attn.linear_{m}.{kind}"
                if nm not in manifest:
                    manifest[nm] = dict(manifest[f"layers.0.self_attn.linear_{m}.{kind}"])
    with open(json_path, "w") as f:
        json.dump(manifest, f, indent=2)
    return bin_path, json_path, manifest


def block_params(tensors: dict, b: int) -> dict:
    """The 22 non-GEMM parameters of block b as the encoder sequence takes them."""
    p = {role: tensors[f"layers.{b}.{nm}"]["data"].reshape(-1) for role, nm in ROLE_NAMES.items()}
    p["pos_u"] = p["pos_u"].reshape(H, DH)
    p["pos_v"] = p["pos_v"].reshape(H, DH)
    p["dw_w"] = p["dw_w"].reshape(D, 9)
    p["qkv_b"] = np.concatenate(
        [tensors[f"layers.{b}.self_attn.linear_{m}.bias"]["data"] for m in QKV])
    return p


def pre_params(tensors: dict) -> dict:
    """The pre-encode stage's parameters (the restatement's roles)."""
    return {role: tensors[nm]["data"] for role, nm in PRE_NAMES.items()}


def _int8(rng, K, N):
    """int8 [K, N] with the per-tensor scale that gives the dequantised weights
    a standard deviation of about 1/sqrt(K) (U{-127..127} has sd ~73.3)."""
    return {"data": rng.integers(-127, 128, size=(K, N), dtype=np.int8),
            "scale": float(np.float32(1.0 / (73.3 * np.sqrt(K)))), "scales": None}


def _f32(a):
    return {"data": np.ascontiguousarray(a, np.float32), "scale": None, "scales": None}


def full_model_tensors(rng, enc_gain: float = 1.0, blank_bias: float = 1.5,
                       fp32_matrices: bool = False) -> dict:
    """Every tensor pk_load_weights looks up (csrc/weights.c:309-396) for one
    conformer block plus the pre-encode, positional table and decoder:
    attention, feed-forward and pre-encode projections int8 (the reference's
    int8 manifest), everything else float32. Scales keep activations O(1).
    fp32_matrices: the block's projections stored instead as float32 holding
    the same values (float32(q) * scale, the reference's dequantisation)."""
    t = {}
    for role, nm in PRE_NAMES.items():
        shape = (256, 1, 3, 3) if role.endswith("_w") else (D if role == "out_b" else 256,)
        t[nm] = _f32(0.3 * rng.standard_normal(shape))
    for k in ("3", "6"):
        t[f"pre_encode.conv.{k}.weight"] = _f32(rng.standard_normal((256, 256, 1, 1)) / 16.0)
    t["pre_encode.out.weight"] = _int8(rng, 4096, D)
    pos = np.arange(9999, dtype=np.float64)[:, None] - 4999.0
    inv = np.exp(-np.log(10000.0) * np.arange(0, D, 2, dtype=np.float64) / D)
    pe = np.zeros((9999, D))
    pe[:, 0::2], pe[:, 1::2] = np.sin(pos * inv), np.cos(pos * inv)
    t["pos_encoding.pe_table"] = _f32(pe)
    for role, nm in ROLE_NAMES.items():
        shape = ROLE_SHAPES.get(role, (D,))
        if role.startswith("norm") and role.endswith("_w"):
            a = 1.0 + 0.1 * rng.standard_normal(shape)
        elif role == "dw_w":
            a = 0.3 * rng.standard_normal(shape)
        else:
            a = 0.1 * rng.standard_normal(shape)
        t[f"layers.0.{nm}"] = _f32(a)
    for m in QKV:
        t[f"layers.0.self_attn.linear_{m}.bias"] = _f32(0.1 * rng.standard_normal(D))
    for nm, (K, N) in MATRICES.items():
        q = _int8(rng, K, N)
        if fp32_matrices:
            q = _f32(q["data"].astype(np.float32) * np.float32(q["scale"]))
        t[f"layers.0.{nm}"] = q
    t["layers.0.conv.pointwise_conv1.weight"] = _f32(rng.standard_normal((2 * D, D, 1)) / 32.0)
    t["layers.0.conv.pointwise_conv2.weight"] = _f32(rng.standard_normal((D, D, 1)) / 32.0)
    Hd, V = 640, 1025
    t["decoder.prediction.embed.weight"] = _f32(0.5 * rng.standard_normal((V, Hd)))
    for l in range(2):
        t[f"decoder.lstm.{l}.W_i"] = _f32(rng.standard_normal((1, 4 * Hd, Hd)) / np.sqrt(Hd))
        t[f"decoder.lstm.{l}.W_r"] = _f32(rng.standard_normal((1, 4 * Hd, Hd)) / np.sqrt(Hd))
        t[f"decoder.lstm.{l}.B"] = _f32(0.1 * rng.standard_normal((1, 8 * Hd)))
    t["joint.enc.weight"] = _f32(enc_gain * rng.standard_normal((D, Hd)) / np.sqrt(D))
    t["joint.enc.bias"] = _f32(0.1 * rng.standard_normal(Hd))
    t["joint.pred.weight"] = _f32(rng.standard_normal((Hd, Hd)) / np.sqrt(Hd))
    t["joint.pred.bias"] = _f32(0.1 * rng.standard_normal(Hd))
    t["joint.out.weight"] = _f32(rng.standard_normal((Hd, V)) / np.sqrt(Hd))
    out_b = 0.1 * rng.standard_normal(V)
    out_b[1024] += blank_bias   # blank wins some of the time
    t["joint.joint_net.2.bias"] = _f32(out_b)
    return t


def write_full_checkpoint(dirpath, rng, n_blocks: int = 24, **kw):
    """A complete checkpoint: block 0's tensors written once, blocks
    1 .. n_blocks-1 as manifest entries aliasing block 0's bytes."""
    tensors = full_model_tensors(rng, **kw)
    bin_path, json_path, manifest = write_checkpoint(dirpath, tensors)
    for b in range(1, n_blocks):
        for name in [n for n in manifest if n.startswith("layers.0.")]:
            manifest[name.replace("layers.0.", f"layers.{b}.", 1)] = dict(manifest[name])
    with open(json_path, "w") as f:
        json.dump(manifest, f, indent=2)
    return tensors, bin_path, json_path
