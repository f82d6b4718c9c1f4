"""GPU: quantize-on-append (ggml_set_rows into the KV cache) is bit-exact.

The CUDA append kernel must write the same bytes as the oracle's codecs
(pinned to gguf-py in test_oracle_golden.py) for every KV type, for the
reference's row shapes: Qwen2 LLM rows (2 heads x 64) with shared 1-D
positions (src/cosyvoice-kv-cache.cpp:315-316) and DiT rows (16 heads x 64)
with per-batch positions (src/cosyvoice-graph.cpp:447-449).
"""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NAMES = ["f32", "f16", "q8_0", "q5_1", "q5_0", "q4_1", "q4_0"]


def _golden():
    return np.load(os.path.join(os.path.dirname(__file__), "golden", "kv_codecs.npz"))


@pytest.mark.parametrize("name", NAMES)
def test_append_golden_rows_bit_exact(ctx, cv, cuda, oracle, name):
    torch = cuda
    t = cv.TYPE_BY_NAME[name]
    x = _golden()[f"{name}_x"]                      # [55, 128]
    n = x.shape[0]
    cap = 80
    buf, desc = cv.alloc_kv(t, 2, 64, ne1=cap, ne2=1)
    pos = torch.tensor(np.random.default_rng(0).permutation(cap)[:n], dtype=torch.int32, device="cuda")
    src = torch.tensor(x, device="cuda")[None].contiguous()
    cv.kv_append(ctx, desc, src, pos)
    rb = cv.row_size(t, 128)
    got = buf.view(cap, rb)[pos.long()].cpu().numpy()
    exp = oracle.quantize(t, x)
    bad = np.nonzero((got != exp).any(1))[0]
    assert bad.size == 0, f"{name}: rows {bad[:8]} differ from the oracle"


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("heads,batch,n_new,shared", [(2, 1, 256, True), (2, 1, 1, True), (16, 2, 37, False)])
def test_append_random_bit_exact(ctx, cv, cuda, oracle, name, heads, batch, n_new, shared):
    torch = cuda
    t = cv.TYPE_BY_NAME[name]
    rng = np.random.default_rng(heads * 1000 + n_new)
    row = heads * 64
    cap = n_new + 50
    x = rng.standard_normal((batch, n_new, row)).astype(np.float32)
    hit = rng.random(x.shape) < 0.01
    x[hit] *= 8.0
    buf, desc = cv.alloc_kv(t, heads, 64, ne1=cap, ne2=batch)
    if shared:
        p = rng.permutation(cap)[:n_new]
        pos = torch.tensor(p, dtype=torch.int32, device="cuda")
        pnp = np.broadcast_to(p, (batch, n_new))
    else:
        pnp = np.stack([rng.permutation(cap)[:n_new] for _ in range(batch)])
        pos = torch.tensor(pnp, dtype=torch.int32, device="cuda")
    cv.kv_append(ctx, desc, torch.tensor(x, device="cuda"), pos)
    rb = cv.row_size(t, row)
    got = buf.view(batch, cap, rb).cpu().numpy()
    for b in range(batch):
        exp = oracle.quantize(t, x[b])
        assert np.array_equal(got[b][pnp[b]], exp), f"{name} batch {b}"


@pytest.mark.parametrize("name", ["q8_0", "q5_1", "q5_0", "q4_1", "q4_0"])
def test_append_dit_launch_bit_exact(ctx, cv, cuda, oracle, name):
    """A DiT-sized append (8 entries x 600 rows of 16 heads x 64: 153,600 blocks) takes the
    thread-per-block quantizer for the 4- and 5-bit types (q8_0 keeps the warp form, checked
    here at the same size); the sequential scans must keep ggml's tie rules: the first
    element of largest magnitude gives q4_0/q5_0 their sign, an all-zero block a zero scale and
    a constant block a zero range.  One position is out of range: that row is skipped and
    reported, the rest are written."""
    torch = cuda
    t = cv.TYPE_BY_NAME[name]
    rng = np.random.default_rng(11)
    batch, n_new, heads = 8, 600, 16
    row = heads * 64
    cap = n_new + 50
    x = rng.standard_normal((batch, n_new, row)).astype(np.float32)
    blk = x.reshape(-1, 32)
    sel = rng.random(blk.shape[0])
    ties = np.nonzero(sel < 0.05)[0]
    a, b = rng.integers(0, 32, ties.size), rng.integers(0, 32, ties.size)
    b = np.where(a == b, (b + 1) % 32, b)
    m = rng.choice([4.0, 7.5], ties.size).astype(np.float32)
    blk[ties, a] = m                      # +m and -m: whichever comes first sets the sign
    blk[ties, b] = -m
    blk[(sel >= 0.05) & (sel < 0.06)] = 0.0
    blk[(sel >= 0.06) & (sel < 0.07)] = 1.25
    pnp = np.stack([rng.permutation(cap)[:n_new] for _ in range(batch)]).astype(np.int32)
    pnp[3, 5] = cap
    buf, desc = cv.alloc_kv(t, heads, 64, ne1=cap, ne2=batch)
    cv.kv_append(ctx, desc, torch.tensor(x, device="cuda"), torch.tensor(pnp, device="cuda"))
    st, detail = ctx.sync_status()
    assert st == 6 and detail == 1
    got = buf.view(batch, cap, cv.row_size(t, row)).cpu().numpy()
    for bb in range(batch):
        ok = pnp[bb] < cap
        exp = oracle.quantize(t, x[bb])
        assert np.array_equal(got[bb][pnp[bb][ok]], exp[ok]), f"{name} batch {bb}"
    assert not got[3][np.setdiff1d(np.arange(cap), pnp[3])].any()


def test_append_bad_position_is_skipped_and_reported(ctx, cv, cuda, oracle):
    torch = cuda
    t = cv.Q8_0
    buf, desc = cv.alloc_kv(t, 2, 64, ne1=8, ne2=1)
    x = np.ones((1, 3, 128), np.float32)
    pos = torch.tensor([1, 8, -1], dtype=torch.int32, device="cuda")
    cv.kv_append(ctx, desc, torch.tensor(x, device="cuda"), pos)
    st, detail = ctx.sync_status()
    assert st == 6 and detail == 1          # CVATTN_ERR_DEVICE, bad position
    got = buf.view(8, -1).cpu().numpy()
    assert np.array_equal(got[1], oracle.quantize(t, x[0, :1])[0])
    assert not got[[0, 2, 3, 4, 5, 6, 7]].any()
    assert ctx.sync_status()[0] == 0        # the word was cleared


def test_dequantize_roundtrip_matches_oracle(ctx, cv, cuda, oracle):
    torch = cuda
    rng = np.random.default_rng(5)
    for name in NAMES:
        t = cv.TYPE_BY_NAME[name]
        x = rng.standard_normal((2, 20, 128)).astype(np.float32)
        buf, desc = cv.alloc_kv(t, 2, 64, ne1=20, ne2=2)
        pos = torch.arange(20, dtype=torch.int32, device="cuda")
        cv.kv_append(ctx, desc, torch.tensor(x, device="cuda"), pos)
        got = cv.kv_dequantize(ctx, desc, 20).cpu().numpy()
        exp = oracle.dequantize(t, oracle.quantize(t, x), 128)
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32)), name
