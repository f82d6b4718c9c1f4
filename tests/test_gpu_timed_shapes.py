"""GPU: parity at the exact shapes bench.py times.

* one decode layer, batch 1, 14/2 heads, L 512 f16 K/V ~ N(0, 0.5),
  Q ~ N(0, 1): f32 bar (rel-L2 <= 1e-5) on every decode kernel.
* 256 sequences x 4096 positions, K/V ~ N(0,1) with 1% of the
  elements at +-8 sigma, (q8_0, q4_0) and (q5_1, q5_1): the whole launch runs,
  16 sequences spread over the batch are checked against fp64 (f32 bar).
* causal prefill, batch 8 x 4096, f16 cache, one launch; and the
  reference's own way to issue it (src/cosyvoice-llm.cpp:98-99 caps a call at
  n_batch = 256 tokens): 16 calls of 256 queries against a q8_0 cache that the
  fused append grows by 256 rows per call.  Sampled query rows of the first and
  last batch entries are checked against fp64 (f16 bar).
* the DiT launch, 32 utterances x CFG 2 = 64 batch entries, 16
  heads, 600 queries over 300 cached prompt + 600 current frames, 50-frame
  chunk mask, cache K = q8_0 / V = q4_0 (the reference's default DiT cache,
  src/cosyvoice.cpp:187); three batch entries checked (f16 bar).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

D = 64
DEC_REL, FLASH_REL, MAX_ABS = 1e-5, 1e-3, 2e-3


def rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def with_outliers(rng, shape):
    x = rng.standard_normal(shape, dtype=np.float32)
    hit = rng.random(shape, dtype=np.float32) < 0.01
    x[hit] = np.where(rng.random(int(hit.sum())) < 0.5, -8.0, 8.0).astype(np.float32)
    return x


PATHS = {"warp_mma": {"warp_mma": True}, "tmem_stream": {"tmem_stream": True}, "wide": {"wide_chunks": True}, "tensor_cores": {"not_persistent": True},
         "cuda_cores": {"cuda_cores": True}}


@pytest.mark.parametrize("path", list(PATHS))
def test_configs0_single_layer_batch1_f16(ctx, cv, cuda, oracle, path):
    torch = cuda
    rng = np.random.default_rng(0)
    Hq, Hkv, L = 14, 2, 512
    q = rng.standard_normal((1, Hq, D)).astype(np.float32)
    k = (0.5 * rng.standard_normal((1, L, Hkv * D))).astype(np.float32)
    v = (0.5 * rng.standard_normal((1, L, Hkv * D))).astype(np.float32)
    kq, vq = oracle.quantize(cv.F16, k), oracle.quantize(cv.F16, v)
    kb, vb = torch.tensor(kq.reshape(-1), device="cuda"), torch.tensor(vq.reshape(-1), device="cuda")
    kd, vd = cv.kv_tensor(kb, cv.F16, Hkv, D, L, 1), cv.kv_tensor(vb, cv.F16, Hkv, D, L, 1)
    kl = torch.tensor([L], dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, L, **PATHS[path]).cpu().numpy()
    ref = oracle.attention_f64(q, oracle.dequantize(cv.F16, kq[0], Hkv * D).reshape(L, Hkv, D),
                               oracle.dequantize(cv.F16, vq[0], Hkv * D).reshape(L, Hkv, D), 0.125)
    assert rel_l2(out, ref) <= DEC_REL and np.abs(out - ref).max() <= MAX_ABS, f"rel-L2 {rel_l2(out, ref):.2e}"


@pytest.mark.parametrize("kname,vname", [("q8_0", "q4_0"), ("q5_1", "q5_1")])
def test_configs3_256_sequences_4096_outliers(ctx, cv, cuda, oracle, kname, vname):
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(77)
    n, L, Hq, Hkv = 256, 4096, 14, 2
    kq = oracle.quantize(kt, with_outliers(rng, (n, L, Hkv * D)))
    vq = oracle.quantize(vt, with_outliers(rng, (n, L, Hkv * D)))
    kb, vb = torch.tensor(kq.reshape(-1), device="cuda"), torch.tensor(vq.reshape(-1), device="cuda")
    kd, vd = cv.kv_tensor(kb, kt, Hkv, D, L, n), cv.kv_tensor(vb, vt, Hkv, D, L, n)
    q = rng.standard_normal((n, Hq, D)).astype(np.float32)
    kl = torch.full((n,), L, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, L).cpu().numpy()
    assert np.isfinite(out).all()
    for s in range(0, n, 17):
        kdq = oracle.dequantize(kt, kq[s], Hkv * D).reshape(L, Hkv, D)
        vdq = oracle.dequantize(vt, vq[s], Hkv * D).reshape(L, Hkv, D)
        ref = oracle.attention_f64(q[s][None], kdq, vdq, 0.125)[0]
        assert rel_l2(out[s], ref) <= DEC_REL and np.abs(out[s] - ref).max() <= MAX_ABS, \
            f"seq {s}: rel-L2 {rel_l2(out[s], ref):.2e}"


def _causal_rows_reference(oracle, t, kq_b, vq_b, q_b, rows, offset, Hkv):
    """fp64 attention for query rows `rows` of one batch entry with the causal rule
    key j visible iff j <= offset + row."""
    n_kv = kq_b.shape[0]
    kd = oracle.dequantize(t, kq_b, Hkv * D).reshape(n_kv, Hkv, D)
    vd = oracle.dequantize(t, vq_b, Hkv * D).reshape(n_kv, Hkv, D)
    j = np.arange(n_kv)[None, :]
    i = np.asarray(rows)[:, None] + offset
    mask = np.where(j <= i, 0.0, -np.inf).astype(np.float32)
    return oracle.attention_f64(q_b[rows], kd, vd, 0.125, mask)


SAMPLE_ROWS = [0, 1, 63, 64, 127, 128, 255, 256, 1000, 2047, 2048, 3333, 4094, 4095]


def test_configs2_prefill_8x4096_one_launch(ctx, cv, cuda, oracle):
    torch = cuda
    rng = np.random.default_rng(2)
    B, S, Hq, Hkv = 8, 4096, 14, 2
    kq = oracle.quantize(cv.F16, rng.standard_normal((B, S, Hkv * D), dtype=np.float32))
    vq = oracle.quantize(cv.F16, rng.standard_normal((B, S, Hkv * D), dtype=np.float32))
    kb, vb = torch.tensor(kq.reshape(-1), device="cuda"), torch.tensor(vq.reshape(-1), device="cuda")
    kd, vd = cv.kv_tensor(kb, cv.F16, Hkv, D, S, B), cv.kv_tensor(vb, cv.F16, Hkv, D, S, B)
    q = rng.standard_normal((B, S, Hq, D), dtype=np.float32)
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, S, mask_mode=cv.MASK_CAUSAL).cpu().numpy()
    assert np.isfinite(out).all()
    for b in (0, B - 1):
        ref = _causal_rows_reference(oracle, cv.F16, kq[b], vq[b], q[b], SAMPLE_ROWS, 0, Hkv)
        got = out[b][SAMPLE_ROWS]
        assert rel_l2(got, ref) <= FLASH_REL and np.abs(got - ref).max() <= MAX_ABS, f"batch {b}"


def test_configs2_prefill_in_256_token_calls_with_q8_0_append(ctx, cv, cuda, oracle):
    """16 calls of n_batch = 256 queries (src/cosyvoice-llm.cpp:98-99, the job driver
    flushes 256-row chunks, src/cosyvoice-llm-job.cpp:50-57), each appending its
    K/V rows to a q8_0 cache and attending causally to everything cached so far."""
    torch = cuda
    rng = np.random.default_rng(4)
    B, S, Hq, Hkv, C = 8, 4096, 14, 2, 256
    kx = rng.standard_normal((B, S, Hkv * D), dtype=np.float32)
    vx = rng.standard_normal((B, S, Hkv * D), dtype=np.float32)
    q = rng.standard_normal((B, S, Hq, D), dtype=np.float32)
    kb, kd = cv.alloc_kv(cv.Q8_0, Hkv, D, S, B)
    vb, vd = cv.alloc_kv(cv.Q8_0, Hkv, D, S, B)
    kxt, vxt, qt = (torch.tensor(a, device="cuda") for a in (kx, vx, q))
    out = torch.empty_like(qt)
    for c in range(S // C):
        pos = torch.arange(c * C, (c + 1) * C, dtype=torch.int32, device="cuda")
        cv.kv_append(ctx, kd, kxt[:, c * C:(c + 1) * C].contiguous(), pos)
        cv.kv_append(ctx, vd, vxt[:, c * C:(c + 1) * C].contiguous(), pos)
        # Q of the call is a strided view of the whole prompt; the causal offset is c * 256
        oc = cv.flash(ctx, qt[:, c * C:(c + 1) * C], kd, vd, (c + 1) * C, mask_mode=cv.MASK_CAUSAL)
        out[:, c * C:(c + 1) * C] = oc
    kq, vq = oracle.quantize(cv.Q8_0, kx), oracle.quantize(cv.Q8_0, vx)
    assert np.array_equal(kb.view(B, S, -1).cpu().numpy(), kq) and np.array_equal(vb.view(B, S, -1).cpu().numpy(), vq)
    o = out.cpu().numpy()
    for b in (0, B - 1):
        ref = _causal_rows_reference(oracle, cv.Q8_0, kq[b], vq[b], q[b], SAMPLE_ROWS, 0, Hkv)
        got = o[b][SAMPLE_ROWS]
        assert rel_l2(got, ref) <= FLASH_REL and np.abs(got - ref).max() <= MAX_ABS, f"batch {b}"


def test_configs4_dit_64_entries_q8_0_q4_0_chunk_mask(ctx, cv, cuda, oracle):
    torch = cuda
    rng = np.random.default_rng(44)
    B, H, P, S = 64, 16, 300, 600
    n_kv = P + S
    kx = rng.standard_normal((B, n_kv, H * D), dtype=np.float32)
    vx = rng.standard_normal((B, n_kv, H * D), dtype=np.float32)
    kb, kd = cv.alloc_kv(cv.Q8_0, H, D, 1024, B)
    vb, vd = cv.alloc_kv(cv.Q4_0, H, D, 1024, B)
    pos = torch.arange(n_kv, dtype=torch.int32, device="cuda")
    cv.kv_append(ctx, kd, torch.tensor(kx, device="cuda"), pos)
    cv.kv_append(ctx, vd, torch.tensor(vx, device="cuda"), pos)
    q = rng.standard_normal((B, S, H, D), dtype=np.float32)
    bounds = list(range(50, S + 1, 50))
    out = cv.flash(ctx, torch.tensor(q, device="cuda"), kd, vd, n_kv, mask_mode=cv.MASK_CHUNK,
                   chunk_bounds=bounds, chunk_key_offset=P).cpu().numpy()
    m = np.zeros((S, n_kv), np.float32)
    m[:, P:] = oracle.mask_bits_to_f32(oracle.chunk_mask(S, bounds))
    for b in (0, 33, B - 1):
        kq, vq = oracle.quantize(cv.Q8_0, kx[b]), oracle.quantize(cv.Q4_0, vx[b])
        kdq = oracle.dequantize(cv.Q8_0, kq, H * D).reshape(n_kv, H, D)
        vdq = oracle.dequantize(cv.Q4_0, vq, H * D).reshape(n_kv, H, D)
        ref = oracle.attention_f64(q[b], kdq, vdq, 0.125, m)
        assert rel_l2(out[b], ref) <= FLASH_REL and np.abs(out[b] - ref).max() <= MAX_ABS, f"batch {b}"
