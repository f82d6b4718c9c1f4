"""CPU: the RoPE restatement in the oracle and the host-side checks of the RoPE
entry points (no kernel is launched).

The oracle follows ggml's CPU backend for ggml_rope_ext with ext_factor 0
(src/cosyvoice-llm.cpp:56-57,180 NEOX per head; src/cosyvoice-graph.cpp:354-355
NORMAL on the first head_dim elements of the 1024-wide DiT row).  ggml itself
cannot run here, so it is checked against the float64 formula (angles p *
base^(-2k/n_dims)) within the error the float angle products allow, and for the
properties a rotation has.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest


def rope_f64(x, pos, unit, n_dims, neox, base):
    out = x.astype(np.float64).copy()
    half = n_dims // 2
    for r in range(x.shape[0]):
        for u in range(0, x.shape[1], unit):
            for k in range(half):
                th = float(pos[r]) * base ** (-2.0 * k / n_dims)
                i0, i1 = (k, k + half) if neox else (2 * k, 2 * k + 1)
                a, b = float(x[r, u + i0]), float(x[r, u + i1])
                out[r, u + i0] = a * np.cos(th) - b * np.sin(th)
                out[r, u + i1] = a * np.sin(th) + b * np.cos(th)
    return out


@pytest.mark.parametrize("mode,unit,n_dims,base,row", [(2, 64, 64, 1e6, 14 * 64), (2, 64, 64, 1e6, 128),
                                                        (0, 1024, 64, 1e4, 1024), (0, 64, 32, 1e4, 128)])
def test_oracle_rope_matches_formula(oracle, mode, unit, n_dims, base, row):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((9, row)).astype(np.float32)
    pos = np.array([0, 1, 2, 17, 255, 600, 1023, 2047, 4095], dtype=np.int32)
    y = oracle.rope(x, pos, unit, n_dims, mode, base)
    ref = rope_f64(x, pos, unit, n_dims, mode == 2, base)
    # f32 angles: p * s^k by k rounded products, off by up to ~k ulp of p, i.e. ~4e-4 rad at p = 4095
    err = np.abs(y - ref).max(axis=1)
    bound = 2e-6 + 1.5e-7 * pos.astype(np.float64) * (n_dims // 2) * np.abs(x).max()
    assert np.all(err <= bound), (err, bound)
    assert np.array_equal(y[0], x[0])  # position 0 is the identity
    # unrotated tail is copied exactly
    for u in range(0, row, unit):
        assert np.array_equal(y[:, u + n_dims:u + unit], x[:, u + n_dims:u + unit])
    # a rotation keeps each pair's norm
    half = n_dims // 2
    for k in range(half):
        i0, i1 = (k, k + half) if mode == 2 else (2 * k, 2 * k + 1)
        n_in = x[:, i0].astype(np.float64) ** 2 + x[:, i1].astype(np.float64) ** 2
        n_out = y[:, i0].astype(np.float64) ** 2 + y[:, i1].astype(np.float64) ** 2
        assert np.allclose(n_out, n_in, rtol=1e-5, atol=1e-6)


def test_rope_entry_points_reject_bad_descriptions():
    import cvattn as cv
    bad = [cv.rope_params(1, 64, 64, 1e4), cv.rope_params(cv.ROPE_NEOX, 63, 64, 1e4),
           cv.rope_params(cv.ROPE_NEOX, 128, 64, 1e4), cv.rope_params(cv.ROPE_NEOX, 64, 64, 0.0),
           cv.rope_params(cv.ROPE_NEOX, 0, 64, 1e4)]
    buf = ctypes.c_void_p(16)  # never dereferenced: every call fails validation first
    for rp in bad:
        st = cv.lib.cvattn_rope(None, ctypes.byref(rp), buf, 256, buf, 256, buf, 1, 64)
        assert st == 1, st  # CVATTN_ERR_INVALID_ARGUMENT
    good = cv.rope_params(cv.ROPE_NEOX, 64, 64, 1e4)
    assert cv.lib.cvattn_rope(None, ctypes.byref(good), buf, 400, buf, 400, buf, 1, 100) == 1  # 100 % 64 != 0
    assert cv.lib.cvattn_rope(None, ctypes.byref(good), buf, 256, buf, 512, buf, 1, 64) == 1   # in place, strides differ
    assert cv.lib.cvattn_rope(None, ctypes.byref(good), buf, 256, buf, 256, buf, 0, 64) == 0   # nothing to do
    assert cv.lib.cvattn_decode_rope(None, None, None, ctypes.byref(good)) == 1
