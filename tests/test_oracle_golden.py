"""CPU: pin the oracle's KV codecs against gguf-py golden vectors.

tests/golden/kv_codecs.npz was produced by tests/golden/make_golden.py from
gguf-py 0.19.0 quants.py (the reference converter's quantizer, documented as
bit-exact with ggml-quants.c).  The oracle must reproduce every byte, with one
documented exception: where a 32-element block's scale d (Q4_0/Q5_0) or min m
(Q4_1/Q5_1) is a zero whose sign depends on the scan order over +-0.0 ties,
the oracle follows ggml's sequential first-occurrence loop while numpy's SIMD
argmax/min may return the other zero.  Only the f16 sign bit of such a zero
may differ, and the dequantized values compare equal.
"""
from __future__ import annotations

import numpy as np
import pytest

GOLDEN = None


def golden():
    global GOLDEN
    if GOLDEN is None:
        import os
        GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "kv_codecs.npz"))
    return GOLDEN


NAMES = ["f32", "f16", "q8_0", "q5_1", "q5_0", "q4_1", "q4_0"]
HEADER_F16_FIELDS = {"q4_0": [0], "q5_0": [0], "q4_1": [0, 2], "q5_1": [0, 2], "q8_0": [0]}


def _allowed_zero_sign_diff(name, mine, gold, O):
    """True if every differing byte is the sign byte of an f16 zero in a block header."""
    t = getattr(O, name.upper())
    be, bb = O.BLOCK[t]
    diff = np.nonzero(mine != gold)[0]
    for i in diff:
        blk, off = divmod(int(i), bb)
        field = off - 1 if off % 2 else off
        if field not in HEADER_F16_FIELDS.get(name, []):
            return False
        a = int(mine[blk * bb + field]) | int(mine[blk * bb + field + 1]) << 8
        b = int(gold[blk * bb + field]) | int(gold[blk * bb + field + 1]) << 8
        if (a & 0x7FFF) != 0 or (b & 0x7FFF) != 0:
            return False
    return True


@pytest.mark.parametrize("name", NAMES)
def test_quantize_matches_gguf(oracle, name):
    g = golden()
    t = getattr(oracle, name.upper())
    x, q = g[f"{name}_x"], g[f"{name}_q"]
    mine = oracle.quantize(t, x)
    assert mine.shape == q.shape
    n_sign_only = 0
    for r in range(x.shape[0]):
        if np.array_equal(mine[r], q[r]):
            continue
        assert _allowed_zero_sign_diff(name, mine[r], q[r], oracle), f"{name} row {r} differs from gguf-py"
        n_sign_only += 1
    assert n_sign_only <= 1, "zero-sign differences should only come from the +-0 tie rows"


@pytest.mark.parametrize("name", NAMES)
def test_dequantize_matches_gguf(oracle, name):
    g = golden()
    t = getattr(oracle, name.upper())
    x, q, dq = g[f"{name}_x"], g[f"{name}_q"], g[f"{name}_dq"]
    mine = oracle.dequantize(t, q, x.shape[1])
    same = (mine.view(np.uint32) == dq.view(np.uint32)) | (np.isnan(mine) & np.isnan(dq))
    assert same.all(), f"{name}: dequantized bits differ at {np.argwhere(~same)[:5]}"


def test_f16_conversion_exhaustive_roundtrip(oracle):
    """Every finite f16 value survives f16 -> f32 -> f16, and random f32 round like numpy."""
    h = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    f = h.view(np.float16).astype(np.float32)
    finite = np.isfinite(f)
    back = oracle.quantize(oracle.F16, f[finite].reshape(1, -1)).view(np.uint16).ravel()
    assert np.array_equal(back, h[finite])
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-7, 1e-5, 1e-3, 1, 1e3, 6e4, 1e5)]).astype(np.float32)
    mine = oracle.quantize(oracle.F16, x.reshape(1, -1)).view(np.uint16).ravel()
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)


def test_causal_mask_matches_reference_loop(oracle):
    # src/cosyvoice-llm.cpp:20-29 restated in Python
    for n, L in [(1, 1), (4, 4), (3, 10), (256, 300)]:
        m = oracle.causal_mask(n, L)
        exp = np.zeros((n, L), np.uint16)
        vis = L - n
        for i in range(n):
            for j in range(L):
                exp[i, j] = 0xFC00 if j > vis else 0
            vis += 1
        assert np.array_equal(m, exp)


def test_chunk_mask_matches_reference_loop(oracle):
    # src/cosyvoice-token2wav.cpp:285-298 restated in Python
    for n, bounds in [(600, list(range(50, 601, 50))), (100, [30, 70]), (64, []), (10, [10])]:
        m = oracle.chunk_mask(n, bounds)
        exp = np.zeros((n, n), np.uint16)
        for i in range(n):
            be = next((b for b in bounds if b > i), n)
            exp[i] = np.where(np.arange(n) < be, 0, 0xFC00)
        assert np.array_equal(m, exp)


def test_attention_f64_small_known_answer(oracle):
    """Two keys, hand-computed softmax."""
    q = np.array([[[1.0, 0.0]]], np.float32)           # n_q=1, Hq=1, D=2
    k = np.array([[[1.0, 0.0]], [[0.0, 1.0]]], np.float32)
    v = np.array([[[1.0, 2.0]], [[3.0, 4.0]]], np.float32)
    out = oracle.attention_f64(q, k, v, 1.0)
    p0 = np.exp(1.0) / (np.exp(1.0) + 1.0)
    exp = p0 * np.array([1, 2]) + (1 - p0) * np.array([3, 4])
    assert np.allclose(out[0, 0], exp, rtol=1e-6)
    # fully masked row gives zeros
    mask = np.full((1, 2), -np.inf, np.float32)
    assert np.all(oracle.attention_f64(q, k, v, 1.0, mask) == 0)


def test_flash_cpu_matches_f64(oracle):
    """The timed ggml-CPU-style baseline agrees with the fp64 oracle."""
    rng = np.random.default_rng(3)
    Hq, Hkv, D, L = 14, 2, 64, 300
    for kt, vt in [(oracle.Q8_0, oracle.Q8_0), (oracle.F16, oracle.Q4_0), (oracle.Q5_1, oracle.Q5_1)]:
        kx = rng.standard_normal((L, Hkv * D)).astype(np.float32)
        vx = rng.standard_normal((L, Hkv * D)).astype(np.float32)
        kq, vq = oracle.quantize(kt, kx), oracle.quantize(vt, vx)
        q = rng.standard_normal((1, 1, Hq, D)).astype(np.float32)
        got = oracle.flash_cpu(q, [kq], [vq], kt, vt, Hkv, np.array([L]), False, 0.125, n_threads=2)
        kd = oracle.dequantize(kt, kq, Hkv * D).reshape(L, Hkv, D)
        vd = oracle.dequantize(vt, vq, Hkv * D).reshape(L, Hkv, D)
        ref = oracle.attention_f64(q[0], kd, vd, 0.125)
        assert np.abs(got[0] - ref).max() < 1e-5
