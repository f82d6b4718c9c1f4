"""GPU: RoPE (ggml_rope_ext, ext_factor 0) standalone, fused with the KV
append, and fused into the decode step.

Reference call sites: src/cosyvoice-llm.cpp:56-57 (Q and K, NEOX per head,
n_dims = head_dim, freq_base = rope_theta) and :180 (K of the prefill's last
layer); src/cosyvoice-graph.cpp:354-355 (DiT Q and K, NORMAL on the first
head_dim elements of the 1024-wide row, freq_base 10000) followed by
update_cache at :365.  The oracle restates ggml's CPU backend; angles are
formed with the same f32 products on both sides, so the only difference is
cos / sin (a few ulp).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HQ, HKV, D = 14, 2, 64
SCALE = 1.0 / 8.0
THETA = 1_000_000.0  # Qwen2 rope_theta


def rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


CASES = [  # (mode, unit_len, n_dims, base, row_len): LLM Q rows, LLM K rows, DiT rows, partial rotation
    ("neox", 64, 64, THETA, HQ * D),
    ("neox", 64, 64, THETA, HKV * D),
    ("normal", 1024, 64, 1e4, 1024),
    ("normal", 64, 32, 1e4, 128),
]


@pytest.mark.parametrize("mode,unit,n_dims,base,row", CASES)
def test_rope_matches_oracle(ctx, cv, cuda, oracle, mode, unit, n_dims, base, row):
    torch = cuda
    m = cv.ROPE_NEOX if mode == "neox" else cv.ROPE_NORMAL
    rng = np.random.default_rng(row + n_dims)
    n = 300
    x = (rng.standard_normal((n, row)) * 3).astype(np.float32)
    pos = rng.integers(0, 9000, n).astype(np.int32)
    pos[:3] = [0, 1, 8999]
    rp = cv.rope_params(m, n_dims, unit, base)
    xt = torch.tensor(x, device="cuda")
    pt = torch.tensor(pos, device="cuda")
    got = cv.rope(xt, pt, rp).cpu().numpy()
    exp = oracle.rope(x, pos, unit, n_dims, m, base)
    assert np.abs(got - exp).max() <= 1e-6 * np.abs(x).max() * 4, np.abs(got - exp).max()
    assert np.array_equal(got[0], x[0])
    cv.rope(xt, pt, rp, out=xt)  # in place gives the same values
    assert np.array_equal(xt.cpu().numpy(), got)


@pytest.mark.parametrize("name", ["f32", "f16", "q8_0", "q5_1", "q4_0"])
@pytest.mark.parametrize("shape", ["llm", "dit"])
def test_append_rope_equals_rope_then_append(ctx, cv, cuda, oracle, name, shape):
    """The fused kernel writes the bytes of cvattn_rope followed by cvattn_kv_append,
    and those match the oracle's rope + quantize up to cos/sin rounding."""
    torch = cuda
    t = cv.TYPE_BY_NAME[name]
    rng = np.random.default_rng(7)
    if shape == "llm":
        heads, batch, n_new, rp = HKV, 1, 200, cv.rope_params(cv.ROPE_NEOX, D, D, THETA)
        unit, n_dims, m, base = D, D, cv.ROPE_NEOX, THETA
    else:
        heads, batch, n_new, rp = 16, 2, 60, cv.rope_params(cv.ROPE_NORMAL, D, 16 * D, 1e4)
        unit, n_dims, m, base = 16 * D, D, cv.ROPE_NORMAL, 1e4
    row = heads * D
    cap = n_new + 40
    x = rng.standard_normal((batch, n_new, row)).astype(np.float32)
    pnp = np.stack([rng.permutation(cap)[:n_new] for _ in range(batch)]).astype(np.int32)
    pos = torch.tensor(pnp, device="cuda")
    src = torch.tensor(x, device="cuda")
    buf_f, desc_f = cv.alloc_kv(t, heads, D, ne1=cap, ne2=batch)
    cv.kv_append(ctx, desc_f, src, pos, rope=rp)
    # two-step: rope then append
    rot = cv.rope(src.view(-1, row).contiguous(), pos.view(-1).contiguous(), rp).view(batch, n_new, row)
    buf_2, desc_2 = cv.alloc_kv(t, heads, D, ne1=cap, ne2=batch)
    cv.kv_append(ctx, desc_2, rot.contiguous(), pos)
    torch.cuda.synchronize()
    assert torch.equal(buf_f, buf_2)
    # against the oracle: rope + quantize, compared after dequantization
    rb = cv.row_size(t, row)
    got = buf_f.view(batch, cap, rb).cpu().numpy()
    # a few-ulp cos / sin difference may move an f32 / f16 value by an ulp or a quant by one step
    tol = {"f32": 1e-5, "f16": 4e-3, "q8_0": 0.06, "q5_1": 0.35, "q4_0": 0.7}[name]
    for b in range(batch):
        exp_rot = oracle.rope(x[b], pnp[b], unit, n_dims, m, base)
        exp_q = oracle.quantize(t, exp_rot)
        rows = got[b][pnp[b].astype(np.int64)]
        if name not in ("f32", "f16"):
            assert (rows == exp_q).all(1).mean() >= 0.9
        dq = oracle.dequantize(t, rows, row)
        assert np.abs(dq - oracle.dequantize(t, exp_q, row)).max() <= tol
    assert ctx.sync_status()[0] == 0


def build_cache(cv, cuda, oracle, kt, vt, lens, rng, cap, unit, n_dims, m, base):
    """Caches whose K rows were rotated at their positions (as update_cache stores them)."""
    torch = cuda
    n = len(lens)
    kx = rng.standard_normal((n, cap, HKV * D)).astype(np.float32)
    vx = rng.standard_normal((n, cap, HKV * D)).astype(np.float32)
    posr = np.arange(cap, dtype=np.int32)
    krot = np.stack([oracle.rope(kx[s], posr, unit, n_dims, m, base) for s in range(n)])
    kq, vq = oracle.quantize(kt, krot), oracle.quantize(vt, vx)
    kbuf = torch.tensor(kq.reshape(-1), device="cuda")
    vbuf = torch.tensor(vq.reshape(-1), device="cuda")
    return kq, vq, kbuf, vbuf, cv.kv_tensor(kbuf, kt, HKV, D, cap, n), cv.kv_tensor(vbuf, vt, HKV, D, cap, n)


@pytest.mark.parametrize("kname,vname", [("q8_0", "q8_0"), ("q4_1", "q5_1"), ("q8_0", "q4_0")])
@pytest.mark.parametrize("mode", ["neox", "normal"])
@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_rope_fused(ctx, cv, cuda, oracle, kname, vname, mode, path):
    """One decode step with the RoPE of Q and the new K row fused in: Q and k_new turn
    by kv_len - 1, the rotated k_new (and v_new) are appended, then attention; on both
    persistent kernels that apply it."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    m = cv.ROPE_NEOX if mode == "neox" else cv.ROPE_NORMAL
    base = THETA if mode == "neox" else 1e4
    rng = np.random.default_rng(61)
    lens = rng.integers(1, 1500, 40).tolist()
    lens[:3] = [1, 64, 1500]
    cap, n = 1500, len(lens)
    kq, vq, kbuf, vbuf, kd, vd = build_cache(cv, cuda, oracle, kt, vt, lens, rng, cap, D, D, m, base)
    q = rng.standard_normal((n, HQ, D)).astype(np.float32)
    kn = rng.standard_normal((n, HKV * D)).astype(np.float32)
    vn = rng.standard_normal((n, HKV * D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    qt = torch.tensor(q, device="cuda")
    out = torch.empty_like(qt)
    rp = cv.rope_params(m, D, D, base)
    dec = cv.Decoder(ctx, kd, vd, n, HQ, cap, qt, out, kl, k_new=torch.tensor(kn, device="cuda"),
                     v_new=torch.tensor(vn, device="cuda"), rope=rp, **{path: True})
    dec()
    got = out.cpu().numpy()
    assert ctx.sync_status()[0] == 0
    p = np.array(lens, dtype=np.int32) - 1
    q_rot = oracle.rope(q.reshape(n * HQ, D), np.repeat(p, HQ), D, D, m, base).reshape(n, HQ, D)
    kn_rot = oracle.rope(kn, p, D, D, m, base)
    # the appended K rows are the engine's (checked below); the reference covers Q's rotation
    appended = kbuf.view(n, cap, -1).cpu().numpy()[np.arange(n), p]
    kq2, vq2 = kq.copy(), vq.copy()
    for s in range(n):
        kq2[s, lens[s] - 1] = appended[s]
        vq2[s, lens[s] - 1] = oracle.quantize(vt, vn[s][None])[0]
    # and they hold the oracle's rotation up to cos / sin rounding (one quant step at most)
    dk = oracle.dequantize(kt, appended, HKV * D) - oracle.dequantize(kt, oracle.quantize(kt, kn_rot), HKV * D)
    assert np.abs(dk).max() <= 0.35
    ref = np.zeros_like(q)
    for s, L in enumerate(lens):
        kdq = oracle.dequantize(kt, kq2[s, :L], HKV * D).reshape(L, HKV, D)
        vdq = oracle.dequantize(vt, vq2[s, :L], HKV * D).reshape(L, HKV, D)
        ref[s] = oracle.attention_f64(q_rot[s][None], kdq, vdq, SCALE)[0]
    assert rel_l2(got, ref) <= 1e-5, rel_l2(got, ref)
    # the appended rows: the engine's own rotation of k_new, quantized bit-exactly
    rot_gpu = cv.rope(torch.tensor(kn, device="cuda"), torch.tensor(p, device="cuda"), rp).cpu().numpy()
    assert np.array_equal(appended, oracle.quantize(kt, rot_gpu))


def test_decode_rope_unsupported_paths(ctx, cv, cuda):
    torch = cuda
    n, cap = 2, 64
    kb, kd = cv.alloc_kv(cv.F16, HKV, D, cap, n)
    vb, vd = cv.alloc_kv(cv.F16, HKV, D, cap, n)
    q = torch.zeros(n, HQ, D, device="cuda")
    out = torch.empty_like(q)
    kl = torch.full((n,), 10, dtype=torch.int32, device="cuda")
    rp = cv.rope_params(cv.ROPE_NEOX, D, D, THETA)
    with pytest.raises(cv.CvattnError):  # f16 K: neither persistent kernel
        cv.Decoder(ctx, kd, vd, n, HQ, cap, q, out, kl, rope=rp)()
    kb, kd = cv.alloc_kv(cv.Q8_0, HKV, D, cap, n)
    vb, vd = cv.alloc_kv(cv.Q8_0, HKV, D, cap, n)
    with pytest.raises(cv.CvattnError):  # a flag that selects another kernel
        cv.Decoder(ctx, kd, vd, n, HQ, cap, q, out, kl, rope=rp, cuda_cores=True)()
    with pytest.raises(cv.CvattnError):  # not a per-head rope
        cv.Decoder(ctx, kd, vd, n, HQ, cap, q, out, kl, rope=cv.rope_params(cv.ROPE_NEOX, 32, D, THETA))()
    torch.cuda.synchronize()
