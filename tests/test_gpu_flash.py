"""GPU: tcgen05 flash attention (prefill / DiT) vs the fp64 oracle.

ggml_flash_attn_ext semantics as used by llm_prefill (causal mask,
src/cosyvoice-llm.cpp:20-29,101-108) and the DiT (uncached f32 K/V,
src/cosyvoice-graph.cpp:373-377; cached typed K/V :363-366; chunk mask
src/cosyvoice-token2wav.cpp:285-298; cut_len query slicing :337-342).
Operands run through f16 tensor cores, so the bar is the north-star's
f16 one: max-abs <= 2e-3 and relative L2 <= 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

D = 64
MAX_ABS, REL_L2 = 2e-3, 1e-3
ALL = ["f32", "f16", "q8_0", "q5_1", "q5_0", "q4_1", "q4_0"]


def rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def make_kv(cv, cuda, oracle, t, n_kv, Hkv, batch, rng, cap=None):
    cap = cap or n_kv
    x = rng.standard_normal((batch, cap, Hkv * D)).astype(np.float32)
    q = oracle.quantize(t, x)
    buf = cuda.tensor(q.reshape(-1), device="cuda")
    return q, buf, cv.kv_tensor(buf, t, Hkv, D, cap, batch)


def reference(oracle, t_k, t_v, kq, vq, q, n_kv, Hkv, mask=None):
    """q [B, n_q, Hq, D]; mask f32 [B or 1, n_q, n_kv] or None."""
    B = q.shape[0]
    out = np.zeros_like(q)
    for b in range(B):
        kd = oracle.dequantize(t_k, kq[b, :n_kv], Hkv * D).reshape(n_kv, Hkv, D)
        vd = oracle.dequantize(t_v, vq[b, :n_kv], Hkv * D).reshape(n_kv, Hkv, D)
        m = None if mask is None else mask[b if mask.shape[0] > 1 else 0]
        out[b] = oracle.attention_f64(q[b], kd, vd, 1.0 / 8.0, m)
    return out


@pytest.fixture(params=["split_columns", "whole_rows", "one_tile"])
def fk(request, cv):
    """flags of cvattn_flash: the persistent two-tile kernel with two softmax warpgroups per
    query tile (each on half the key columns) or one (a thread per row), or the one-tile kernel."""
    return {"split_columns": cv.FLASH_SPLIT_COLUMNS, "whole_rows": cv.FLASH_WHOLE_ROWS,
            "one_tile": cv.FLASH_ONE_TILE}[request.param]


def check(out, ref, what=""):
    e = np.abs(out - ref).max()
    r = rel_l2(out, ref)
    assert e <= MAX_ABS and r <= REL_L2, f"{what}: max-abs {e:.2e} rel-L2 {r:.2e}"


@pytest.mark.parametrize("kv_name", ["f16", "q8_0"])
@pytest.mark.parametrize("n_q,cur", [(1, 0), (37, 0), (128, 0), (256, 0), (300, 45), (256, 700)])
def test_prefill_causal_qwen2(ctx, cv, cuda, oracle, fk, kv_name, n_q, cur):
    torch = cuda
    t = cv.TYPE_BY_NAME[kv_name]
    rng = np.random.default_rng(n_q * 7 + cur)
    B, Hq, Hkv = 2, 14, 2
    n_kv = cur + n_q
    kq, kb, kd = make_kv(cv, cuda, oracle, t, n_kv, Hkv, B, rng, cap=n_kv + 5)
    vq, vb, vd = make_kv(cv, cuda, oracle, t, n_kv, Hkv, B, rng, cap=n_kv + 5)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_CAUSAL, flags=fk).cpu().numpy()
    mask = oracle.mask_bits_to_f32(oracle.causal_mask(n_q, n_kv))[None]
    ref = reference(oracle, t, t, kq, vq, q, n_kv, Hkv, mask)
    check(out, ref, f"causal {kv_name} n_q={n_q} cur={cur}")


@pytest.mark.parametrize("kname", ALL)
@pytest.mark.parametrize("vname", ALL)
def test_flash_type_pairs(ctx, cv, cuda, oracle, fk, kname, vname):
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(kt * 31 + vt)
    B, Hq, Hkv, n_q, n_kv = 1, 14, 2, 130, 200
    kq, kb, kd = make_kv(cv, cuda, oracle, kt, n_kv, Hkv, B, rng)
    vq, vb, vd = make_kv(cv, cuda, oracle, vt, n_kv, Hkv, B, rng)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, flags=fk).cpu().numpy()
    check(out, reference(oracle, kt, vt, kq, vq, q, n_kv, Hkv), f"{kname}/{vname}")


@pytest.mark.parametrize("S,chunk", [(600, 50), (200, 50), (131, 40)])
def test_dit_uncached_f32_chunk_mask(ctx, cv, cuda, oracle, fk, S, chunk):
    """Uncached DiT: f32 K/V activations, H=16 (MHA), CFG batch 2, chunk mask."""
    torch = cuda
    rng = np.random.default_rng(S)
    B, H = 2, 16
    kq, kb, kd = make_kv(cv, cuda, oracle, cv.F32, S, H, B, rng)
    vq, vb, vd = make_kv(cv, cuda, oracle, cv.F32, S, H, B, rng)
    q = rng.standard_normal((B, S, H, D)).astype(np.float32)
    bounds = list(range(chunk, S + 1, chunk))
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, S, mask_mode=cv.MASK_CHUNK,
                   chunk_bounds=bounds, flags=fk).cpu().numpy()
    mask = oracle.mask_bits_to_f32(oracle.chunk_mask(S, bounds))[None]
    check(out, reference(oracle, cv.F32, cv.F32, kq, vq, q, S, H, mask), "dit chunk")
    # the same mask given explicitly (f16 bits, ggml semantics)
    mbits = torch.tensor(oracle.chunk_mask(S, bounds).view(np.int16), device="cuda")
    out2 = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, S, mask_mode=cv.MASK_EXPLICIT,
                    mask=mbits, flags=fk).cpu().numpy()
    check(out2, reference(oracle, cv.F32, cv.F32, kq, vq, q, S, H, mask), "dit explicit")
    # unmasked
    out3 = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, S, flags=fk).cpu().numpy()
    check(out3, reference(oracle, cv.F32, cv.F32, kq, vq, q, S, H), "dit unmasked")


@pytest.mark.parametrize("kname,vname", [("q8_0", "q4_0"), ("f16", "f16"), ("q8_0", "q8_0")])
def test_dit_cached_prompt_slots(ctx, cv, cuda, oracle, fk, kname, vname):
    """Cached DiT: 300 prompt frames always visible + 600 current frames under
    the chunk mask (the benchmark layout); default DiT KV k=q8_0, v=q4_0
    (src/cosyvoice.cpp:187)."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(kt + 5 * vt)
    B, H, P, S = 2, 16, 300, 600
    n_kv = P + S
    kq, kb, kd = make_kv(cv, cuda, oracle, kt, n_kv, H, B, rng, cap=1024)
    vq, vb, vd = make_kv(cv, cuda, oracle, vt, n_kv, H, B, rng, cap=1024)
    q = rng.standard_normal((B, S, H, D)).astype(np.float32)
    bounds = list(range(50, S + 1, 50))
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_CHUNK,
                   chunk_bounds=bounds, chunk_key_offset=P, flags=fk).cpu().numpy()
    cm = oracle.mask_bits_to_f32(oracle.chunk_mask(S, bounds))
    mask = np.concatenate([np.zeros((S, P), np.float32), cm], axis=1)[None]
    check(out, reference(oracle, kt, vt, kq, vq, q, n_kv, H, mask), f"dit cached {kname}/{vname}")


def test_dit_cut_len_queries(ctx, cv, cuda, oracle, fk):
    """Final DiT block: queries are the last S - cut_len rows (strided view of Q);
    mask rows follow ggml's row order (row i of the mask for query i)."""
    torch = cuda
    rng = np.random.default_rng(77)
    B, H, S, cut = 2, 16, 260, 60
    kq, kb, kd = make_kv(cv, cuda, oracle, cv.F32, S, H, B, rng)
    vq, vb, vd = make_kv(cv, cuda, oracle, cv.F32, S, H, B, rng)
    qfull = rng.standard_normal((B, S, H, D)).astype(np.float32)
    qt = torch.tensor(qfull, device="cuda")[:, cut:]          # strided view, no copy
    bounds = [100, 200, 260]
    mbits = oracle.chunk_mask(S, bounds)
    out = cv.flash(ctx, qt, kd, vd, S, mask_mode=cv.MASK_EXPLICIT,
                   mask=torch.tensor(mbits.view(np.int16), device="cuda"), flags=fk).cpu().numpy()
    mask = oracle.mask_bits_to_f32(mbits)[: S - cut][None]
    check(out, reference(oracle, cv.F32, cv.F32, kq, vq, qfull[:, cut:].copy(), S, H, mask), "cut_len")
    # implicit chunk mask with the same row convention
    out2 = cv.flash(ctx, qt, kd, vd, S, mask_mode=cv.MASK_CHUNK, chunk_bounds=bounds, flags=fk).cpu().numpy()
    check(out2, reference(oracle, cv.F32, cv.F32, kq, vq, qfull[:, cut:].copy(), S, H, mask), "cut_len chunk")


def test_explicit_random_mask_and_fully_masked_rows(ctx, cv, cuda, oracle, fk):
    torch = cuda
    rng = np.random.default_rng(99)
    B, Hq, Hkv, n_q, n_kv = 1, 14, 2, 150, 333
    kq, kb, kd = make_kv(cv, cuda, oracle, cv.F16, n_kv, Hkv, B, rng)
    vq, vb, vd = make_kv(cv, cuda, oracle, cv.F16, n_kv, Hkv, B, rng)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    m = rng.uniform(-3, 3, (n_q, n_kv)).astype(np.float16)
    m[rng.random(m.shape) < 0.3] = -np.inf
    m[5, :] = -np.inf                      # fully masked row -> zeros
    m[140:, :200] = -np.inf                # first key tiles fully masked for some rows
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_EXPLICIT,
                   mask=torch.tensor(m.view(np.int16), device="cuda"), flags=fk).cpu().numpy()
    ref = reference(oracle, cv.F16, cv.F16, kq, vq, q, n_kv, Hkv, m.astype(np.float32)[None])
    assert not out[0, 5].any()
    check(out, ref, "explicit random mask")


def test_empty_kv_gives_zeros(ctx, cv, cuda, oracle, fk):
    torch = cuda
    kb, kd = cv.alloc_kv(cv.Q8_0, 2, 64, 16, 1)
    vb, vd = cv.alloc_kv(cv.Q8_0, 2, 64, 16, 1)
    q = torch.randn(1, 10, 14, 64, device="cuda")
    out = cv.flash(ctx, q, kd, vd, 0, flags=fk)
    assert not out.any()


@pytest.mark.parametrize("kv_name", ["f16", "q8_0"])
def test_prefill_causal_many_items_per_cta(ctx, cv, cuda, oracle, fk, kv_name):
    """Batch 8 x 1024 causal rows x 14 heads: several work items per persistent
    CTA (head pairs of one KV group, the odd head alone), longest first."""
    torch = cuda
    t = cv.TYPE_BY_NAME[kv_name]
    rng = np.random.default_rng(5)
    B, Hq, Hkv, n_q = 8, 14, 2, 1024
    kq, kb, kd = make_kv(cv, cuda, oracle, t, n_q, Hkv, B, rng)
    vq, vb, vd = make_kv(cv, cuda, oracle, t, n_q, Hkv, B, rng)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_q, mask_mode=cv.MASK_CAUSAL, flags=fk).cpu().numpy()
    mask = oracle.mask_bits_to_f32(oracle.causal_mask(n_q, n_q))[None]
    ref = reference(oracle, t, t, kq, vq, q, n_q, Hkv, mask)
    check(out, ref, f"causal many items {kv_name}")


def test_dit_cached_many_items_per_cta(ctx, cv, cuda, oracle, fk):
    """DiT layout with 16 batch entries: query-tile pairs of one head share the
    K/V tiles, the fifth tile of each head runs alone."""
    torch = cuda
    rng = np.random.default_rng(6)
    B, H, P, S = 16, 16, 300, 600
    n_kv = P + S
    kq, kb, kd = make_kv(cv, cuda, oracle, cv.F16, n_kv, H, B, rng, cap=1024)
    vq, vb, vd = make_kv(cv, cuda, oracle, cv.F16, n_kv, H, B, rng, cap=1024)
    q = rng.standard_normal((B, S, H, D)).astype(np.float32)
    bounds = list(range(50, S + 1, 50))
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_CHUNK,
                   chunk_bounds=bounds, chunk_key_offset=P, flags=fk).cpu().numpy()
    cm = oracle.mask_bits_to_f32(oracle.chunk_mask(S, bounds))
    mask = np.concatenate([np.zeros((S, P), np.float32), cm], axis=1)[None]
    check(out, reference(oracle, cv.F16, cv.F16, kq, vq, q, n_kv, H, mask), "dit cached many items")


@pytest.mark.parametrize("Hq", [2, 4, 6, 16])
def test_prefill_causal_group_sizes(ctx, cv, cuda, oracle, fk, Hq):
    """G = 1, 2, 3, 8 query heads per KV head: head pairs (even G) and query-tile pairs (G = 1, odd G)."""
    torch = cuda
    rng = np.random.default_rng(100 + Hq)
    B, Hkv, n_q, cur = 2, 2, 300, 40
    n_kv = cur + n_q
    kq, kb, kd = make_kv(cv, cuda, oracle, cv.Q8_0, n_kv, Hkv, B, rng)
    vq, vb, vd = make_kv(cv, cuda, oracle, cv.Q4_0, n_kv, Hkv, B, rng)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_CAUSAL, flags=fk).cpu().numpy()
    mask = oracle.mask_bits_to_f32(oracle.causal_mask(n_q, n_kv))[None]
    check(out, reference(oracle, cv.Q8_0, cv.Q4_0, kq, vq, q, n_kv, Hkv, mask), f"Hq={Hq}")


QUANT = ["q8_0", "q5_1", "q5_0", "q4_1", "q4_0"]


@pytest.mark.parametrize("kname", QUANT)
@pytest.mark.parametrize("vname", QUANT)
def test_staged_tma_form_type_pairs(ctx, cv, cuda, oracle, kname, vname):
    """4 KV heads make every block-quantized row a multiple of 16 bytes, so the
    persistent kernel's producer fetches the raw rows with TMA byte boxes that
    start at the 16-byte boundary below each head (head offsets 0, 4, 8, 12
    bytes for q8_0); 201 keys leave a ragged last tile read past n_kv."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(kt * 17 + vt + 5)
    B, Hq, Hkv, n_q, n_kv = 2, 8, 4, 130, 201
    kq, kb, kd = make_kv(cv, cuda, oracle, kt, n_kv, Hkv, B, rng, cap=n_kv + 7)
    vq, vb, vd = make_kv(cv, cuda, oracle, vt, n_kv, Hkv, B, rng, cap=n_kv + 7)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv).cpu().numpy()
    check(out, reference(oracle, kt, vt, kq, vq, q, n_kv, Hkv), f"{kname}/{vname}")


@pytest.mark.parametrize("kname", QUANT)
@pytest.mark.parametrize("vname", QUANT)
def test_staged_chunk_form_type_pairs(ctx, cv, cuda, oracle, kname, vname):
    """Qwen2's 2 KV heads: q8_0 / q4_0 / q5_0 rows (136 / 72 / 88 bytes) are not
    16-byte multiples but are contiguous, so the producer bulk-copies a tile's
    whole rows; 201 keys leave a 9-row last tile whose byte count is 8 past a
    16-byte multiple (the tail goes by 4-byte copies).  Pairs of 16-byte rows
    (q4_1, q5_1) take the TMA boxes."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(kt * 13 + vt + 9)
    B, Hq, Hkv, n_q, n_kv = 2, 14, 2, 150, 201
    kq, kb, kd = make_kv(cv, cuda, oracle, kt, n_kv, Hkv, B, rng, cap=n_kv + 5)
    vq, vb, vd = make_kv(cv, cuda, oracle, vt, n_kv, Hkv, B, rng, cap=n_kv + 5)
    q = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    mask = oracle.mask_bits_to_f32(oracle.causal_mask(n_q, n_kv))[None]
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_CAUSAL).cpu().numpy()
    check(out, reference(oracle, kt, vt, kq, vq, q, n_kv, Hkv, mask), f"{kname}/{vname}")


@pytest.mark.parametrize("mode", ["large", "tiny", "negative", "growing"])
@pytest.mark.parametrize("kv_name", ["f16", "q8_0"])
@pytest.mark.parametrize("mask_name", ["none", "causal", "chunk"])
@pytest.mark.parametrize("Hq,Hkv", [(14, 2), (4, 4)])
def test_flash_score_ranges(ctx, cv, cuda, oracle, fk, mode, kv_name, mask_name, Hq, Hkv):
    """Score magnitudes that exercise the softmax's reference-max logic: large scores
    (the first tile's reference max 0 overflows and is redone), scores near 0, scores far
    below 0 (the first tile's P underflows and is redone), and scores that grow along the
    keys (repeated rescales of O)."""
    torch = cuda
    t = cv.TYPE_BY_NAME[kv_name]
    rng = np.random.default_rng(11 * Hq + len(mode) + 3 * len(mask_name))
    B, n_q, n_kv = 1, 200, 300
    u = np.full(D, 1.0 / 8.0, np.float32)  # |u| = 1
    kx = rng.standard_normal((B, n_kv, Hkv * D)).astype(np.float32)
    qx = rng.standard_normal((B, n_q, Hq, D)).astype(np.float32)
    if mode == "large":
        qx *= 10.0
    elif mode == "tiny":
        qx *= 1e-3
    elif mode == "negative":  # q.k ~ -180 for every key: scores near -32 in log2 units
        kx += 3.0 * np.tile(u, Hkv)[None, None]
        qx = 0.1 * qx - 60.0 * u[None, None, None]
    else:  # growing: q.k rises from ~0 to ~300 along the keys
        ramp = (np.arange(n_kv, dtype=np.float32) / n_kv * 30.0)[None, :, None]
        kx += ramp * np.tile(u, Hkv)[None, None]
        qx = 0.3 * qx + 10.0 * u[None, None, None]
    kq = oracle.quantize(t, kx)
    kd = cv.kv_tensor(torch.tensor(kq.reshape(-1), device="cuda"), t, Hkv, D, n_kv, B)
    vq, vb, vd = make_kv(cv, cuda, oracle, t, n_kv, Hkv, B, rng)
    kw, mask = {}, None
    if mask_name == "causal":
        kw = {"mask_mode": cv.MASK_CAUSAL}
        mask = oracle.mask_bits_to_f32(oracle.causal_mask(n_q, n_kv))[None]
    elif mask_name == "chunk":
        bounds = list(range(40, n_q + 1, 40))
        kw = {"mask_mode": cv.MASK_CHUNK, "chunk_bounds": bounds, "chunk_key_offset": n_kv - n_q}
        cm = oracle.mask_bits_to_f32(oracle.chunk_mask(n_q, bounds))
        mask = np.concatenate([np.zeros((n_q, n_kv - n_q), np.float32), cm], axis=1)[None]
    out = cv.flash(ctx, torch.tensor(qx, device="cuda"), kd, vd, n_kv, flags=fk, **kw).cpu().numpy()
    # At scores of tens of log2 units the f16 rounding of Q (and of K) alone moves the output by
    # more than the f16 bar's max-abs (a float64 model of f16 operands gives 9.5e-3 for "large"),
    # so the reference takes the operands as the kernel rounds them: Q * scale * log2(e) in f32
    # rounded to f16, K and V dequantized and rounded to f16.  What remains is the softmax logic
    # under test (P in f16, fp32 accumulation).
    sl2 = np.float32(0.125 * 1.4426950408889634)
    q16 = (qx * sl2).astype(np.float16).astype(np.float64) / float(sl2)
    kr = oracle.dequantize(t, kq[0, :n_kv], Hkv * D).astype(np.float16).astype(np.float32).reshape(n_kv, Hkv, D)
    vr = oracle.dequantize(t, vq[0, :n_kv], Hkv * D).astype(np.float16).astype(np.float32).reshape(n_kv, Hkv, D)
    ref = oracle.attention_f64(q16[0].astype(np.float32), kr, vr, 1.0 / 8.0, None if mask is None else mask[0])[None]
    check(out, ref, f"{mode} {kv_name} {mask_name} {Hq}/{Hkv}")
