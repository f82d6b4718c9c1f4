"""GPU: cvattn_decode_noalloc, the decode entry point that allocates nothing.

Some callers cannot call cudaMalloc.  Examples: a ggml custom-op callback
inside a scheduled graph compute that sees only its own tensors, or a
real-time streaming worker that must not block on the allocator.  For them
the decode workspace comes from a static device array inside libcvattn.so.
This file checks, through the C ABI, that two back-to-back calls of that
entry point give the same output as cvattn_decode with a caller workspace,
within the decode tolerance (rel-L2 1e-5, max-abs 2e-3).  It also checks that
a request larger than the static scratch is refused before anything runs.
The file is named to be collected last.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HQ, HKV, D = 14, 2, 64


def _rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def test_noalloc_decode_matches_workspace_decode_twice(ctx, cv, cuda, oracle):
    torch = cuda
    rng = np.random.default_rng(2024)
    lens = [1, 130, 700, 1500, 2048, 257]
    n, cap = len(lens), 2048
    kx = rng.standard_normal((n, cap, HKV * D)).astype(np.float32)
    vx = rng.standard_normal((n, cap, HKV * D)).astype(np.float32)
    kbuf = torch.tensor(oracle.quantize(cv.Q8_0, kx).reshape(-1), device="cuda")
    vbuf = torch.tensor(oracle.quantize(cv.Q4_0, vx).reshape(-1), device="cuda")
    kd = cv.kv_tensor(kbuf, cv.Q8_0, HKV, D, cap, n)
    vd = cv.kv_tensor(vbuf, cv.Q4_0, HKV, D, cap, n)
    q = torch.tensor(rng.standard_normal((n, HQ, D)).astype(np.float32), device="cuda")
    knew = torch.tensor(rng.standard_normal((n, HKV * D)).astype(np.float32), device="cuda")
    vnew = torch.tensor(rng.standard_normal((n, HKV * D)).astype(np.float32), device="cuda")
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")

    ref = torch.empty_like(q)
    cv.Decoder(ctx, kd, vd, n, HQ, cap, q, ref, kl, k_new=knew, v_new=vnew)()
    torch.cuda.synchronize()

    out = torch.empty_like(q)
    p = cv.Decoder(ctx, kd, vd, n, HQ, cap, q, out, kl, k_new=knew, v_new=vnew).params
    p.workspace, p.workspace_size = None, 0          # the entry point must not need one
    stream = torch.cuda.current_stream().cuda_stream
    expected = ref.cpu().numpy()
    for call in range(2):
        out.fill_(float("nan"))
        st = cv.lib.cvattn_decode_noalloc(ctx.handle, stream, ctypes.byref(p))
        assert st == 0, f"call {call}: status {st}"
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert _rel_l2(got, expected) <= 1e-5 and np.abs(got - expected).max() <= 2e-3, f"call {call}"


def test_noalloc_decode_refuses_requests_beyond_the_scratch(ctx, cv, cuda):
    torch = cuda
    n, cap = 512, 4096
    need = cv.decode_workspace_size(cv.Q8_0, cv.Q8_0, n, cap, HQ, HKV, D)
    assert need > 8 * 1024 * 1024
    kbuf = torch.zeros(16, dtype=torch.uint8, device="cuda")
    kd = cv.kv_tensor(kbuf, cv.Q8_0, HKV, D, cap, n)
    q = torch.zeros((n, HQ, D), device="cuda")
    out = torch.full_like(q, 7.0)
    kl = torch.zeros(n, dtype=torch.int32, device="cuda")
    p = cv.DecodeParams()
    p.q, p.q_seq_stride, p.out, p.out_seq_stride = q.data_ptr(), HQ * D, out.data_ptr(), HQ * D
    p.k, p.v, p.kv_len = kd, kd, kl.data_ptr()
    p.n_seq, p.n_q_heads, p.max_kv_len, p.scale = n, HQ, cap, 0.125
    st = cv.lib.cvattn_decode_noalloc(ctx.handle, torch.cuda.current_stream().cuda_stream, ctypes.byref(p))
    assert st == 3                                     # CVATTN_ERR_LENGTH
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())                    # nothing ran
