"""CPU: the checkpoint loader's host side (pkcu_weights_open / find / name /
count), against the files' own manifests and the reference's manifest parser
(csrc/weights.c:102-207, built from the reference tree in oracle/_ref)."""
import ctypes as C

import numpy as np
import pytest

import weights_fixture as wf


@pytest.fixture(scope="module")
def pk():
    import pkcuda
    pkcuda.lib()
    return pkcuda


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt_i8_i4")
    rng = np.random.default_rng(71)
    tensors = wf.make_tensors(rng, 2, attn="int8", ff="int4")
    bp, jp, man = wf.write_checkpoint(str(d), tensors, alias_blocks=24)
    return tensors, bp, jp, man


def test_open_reads_every_manifest_entry(pk, ckpt, reference):
    tensors, bp, jp, man = ckpt
    blob = open(bp, "rb").read()
    with pk.Weights(bp, jp) as w:
        names = w.names()
        assert sorted(names) == sorted(man)
        assert w.blocks() == 24
        int8 = [n for n, e in man.items() if e["dtype"] == "int8"]
        ref_scales = reference.manifest_scales(jp, int8)
        for n, e in man.items():
            t = w.find(n)
            assert t.dtype == {"float32": 0, "int8": 1, "int4": 2}[e["dtype"]], n
            assert t.dims == tuple(e["shape"]), n
            assert t.numel == e["numel"], n
            nbytes = e["numel"] * (4 if e["dtype"] == "float32" else 1)
            assert C.string_at(t.host, nbytes) == blob[e["offset"]:e["offset"] + nbytes], n
            assert t.dev is None                       # not uploaded
            if e["dtype"] == "int4":
                assert t.n_scales == e["n_scales"]
                sb = 4 * e["n_scales"]
                assert C.string_at(t.host_scales, sb) == blob[e["scales_offset"]:e["scales_offset"] + sb]
        got = np.array([w.find(n).scale for n in int8], np.float32)
        assert np.array_equal(got.view(np.uint32), ref_scales.view(np.uint32))


# Scale texts of the forms a manifest can hold: json.dump's shortest
# round-trip floats (up to 17 significant digits), exponent forms, integers.
SCALE_TEXTS = ["0.0031234567890123457", "0.004", "1e-05", "2.5E-3", "7", "0.1",
               "0.0099999999999999985", "6.103515625e-05", "1.1754943508222875e-38",
               "0.00012345678901234567", "3.0000000000000004", "9.999999747378752e-06",
               "0.0072000000000000003", "1E+2", "0.000977"]


def test_scale_text_matches_reference_parser(pk, reference, tmp_path):
    """The scale is converted from the manifest's text with the reference's own
    digit accumulation, so it matches the reference's parse bit for bit."""
    bp = tmp_path / "weights.bin"
    jp = tmp_path / "weights.json"
    bp.write_bytes(bytes(16))
    rng = np.random.default_rng(5)
    texts = SCALE_TEXTS + [repr(float(v)) for v in rng.uniform(1e-4, 1e-1, 200)]
    names = [f"t{i}" for i in range(len(texts))]
    body = ",\n".join(f'  "{n}": {{"offset": 0, "shape": [1], "numel": 1, "dtype": "int8", '
                      f'"scale": {s}}}' for n, s in zip(names, texts))
    jp.write_text("{\n" + body + "\n}\n")
    want = reference.manifest_scales(jp, names)
    with pk.Weights(bp, jp) as w:
        got = np.array([w.find(n).scale for n in names], np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_open_rejects_bad_files(pk, ckpt, tmp_path):
    tensors, bp, jp, man = ckpt
    L = pk.lib()
    h = pk.VP()
    assert L.pkcu_weights_open(str(tmp_path / "none.bin").encode(), jp.encode(), C.byref(h)) == 1
    short = tmp_path / "short.bin"
    short.write_bytes(open(bp, "rb").read()[:1000])
    assert L.pkcu_weights_open(str(short).encode(), jp.encode(), C.byref(h)) == 1
    assert b"outside" in L.pkcu_last_error()
    bad = tmp_path / "bad.json"
    bad.write_text('{"a": {"offset": 0, "numel": 4, "dtype": "float16"}}')
    assert L.pkcu_weights_open(bp.encode(), str(bad).encode(), C.byref(h)) == 1
    bad.write_text('{"a": {"offset": 0, "numel": 4')
    assert L.pkcu_weights_open(bp.encode(), str(bad).encode(), C.byref(h)) == 1
    assert b"not a weights manifest" in L.pkcu_last_error()
    with pk.Weights(bp, jp) as w:
        t = pk.Tensor()
        assert L.pkcu_weights_find(w.h, b"no.such.tensor", C.byref(t)) == 1
        out = pk.VP(1)
        assert L.pkcu_weights_dequant(w.h, b"layers.0.norm_out.weight", out, None) == 1
        assert b"not uploaded" in L.pkcu_last_error()
