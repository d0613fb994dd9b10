"""CPU: the chunked encoder's plan (host logic only, no CUDA call).

pkcu_should_chunk and pkcu_chunk_bounds against a restatement of the
reference's rule and chunk loop: should_chunk (csrc/encoder.c:602-610, the
PK_CHUNK override included) and encode_blocks_chunked's bounds
(csrc/encoder.c:517-541; PK_CHUNK_SIZE 400, PK_CHUNK_OVERLAP 8,
PK_CHUNK_THRESHOLD 500 from csrc/parakeet.h:132-134)."""
import ctypes as C

import pytest

import pkcuda

AUTO, OFF, ON = pkcuda.PKCU_CHUNK_AUTO, pkcuda.PKCU_CHUNK_OFF, pkcuda.PKCU_CHUNK_ON


def ref_should_chunk(T, env):
    if env is not None:
        if env[:1] == "0" or env == "off":
            return False
        if env[:1] == "1" or env == "on":
            return True
    return T > 500


def ref_bounds(T):
    """(in_start, in_len, out_start, out_len) per chunk, as encoder.c:531-541."""
    Cs, ov = 400, 8
    out = []
    for ci in range((T + Cs - 1) // Cs):
        o0 = ci * Cs
        o1 = min(o0 + Cs, T)
        i0 = max(o0 - ov, 0)
        i1 = min(o1 + ov, T)
        out.append((i0, i1 - i0, o0, o1 - o0))
    return out


def bounds(L, T, mode):
    n = L.pkcu_chunk_bounds(T, mode, 0, None, None, None, None)
    arr = [(C.c_int * n)() for _ in range(4)]
    assert L.pkcu_chunk_bounds(T, mode, n, *arr) == n
    if n > 1:
        assert L.pkcu_chunk_bounds(T, mode, n - 1, *arr) == -1   # capacity checked
    return list(zip(*[list(a) for a in arr]))


@pytest.fixture(scope="module")
def L():
    return pkcuda.lib()


@pytest.mark.parametrize("env", [None, "auto", "0", "off", "1", "on", "2"])
def test_should_chunk_follows_the_reference_rule(L, monkeypatch, env):
    if env is None:
        monkeypatch.delenv("PK_CHUNK", raising=False)
    else:
        monkeypatch.setenv("PK_CHUNK", env)
    for T in (1, 32, 375, 400, 416, 499, 500, 501, 513, 800, 3200, 5000):
        assert bool(L.pkcu_should_chunk(T, AUTO)) == ref_should_chunk(T, env), (env, T)
        assert L.pkcu_should_chunk(T, OFF) == 0 and L.pkcu_should_chunk(T, ON) == 1


@pytest.mark.parametrize("T", [1, 7, 400, 401, 408, 416, 500, 501, 513, 800, 801, 808, 1201, 3200, 5000])
def test_chunk_bounds_match_encode_blocks_chunked(L, monkeypatch, T):
    monkeypatch.delenv("PK_CHUNK", raising=False)
    assert bounds(L, T, ON) == ref_bounds(T)
    assert bounds(L, T, OFF) == [(0, T, 0, T)]
    want = ref_bounds(T) if T > 500 else [(0, T, 0, T)]
    got = bounds(L, T, AUTO)
    assert got == want
    # the owned ranges tile [0, T) and every chunk reads its owned range
    assert sum(ol for _, _, _, ol in got) == T
    for i0, il, o0, ol in got:
        assert i0 <= o0 and o0 + ol <= i0 + il <= T


def test_config3_chunk_lengths(L):
    """3200 frames -> edge chunks of 408 and interior ones of 416."""
    assert [il for _, il, _, _ in bounds(L, 3200, ON)] == [408] + [416] * 6 + [408]


def test_bad_arguments(L):
    assert L.pkcu_chunk_bounds(0, AUTO, 0, None, None, None, None) == -1
    h = C.c_void_p()
    n = (C.c_int * 1)(600)
    assert L.pkcu_chunk_plan_create(n, 1, 7, C.byref(h)) == pkcuda.PKCU_ERR_ARG
    bad = (C.c_int * 1)(0)
    assert L.pkcu_chunk_plan_create(bad, 1, AUTO, C.byref(h)) == pkcuda.PKCU_ERR_ARG
    assert L.pkcu_chunk_plan_create(n, 0, AUTO, C.byref(h)) == pkcuda.PKCU_ERR_ARG
