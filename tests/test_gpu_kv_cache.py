"""GPU: the cvattn_kv_cache seam object, driven as the reference drives
cosyvoice_kv_cache.

* LLM (src/cosyvoice-llm.cpp:90-202 prefill, :204-300 decode): per layer
  update_cache then attention_forward, then cur_len += n_tokens.  The prefill
  call is causal flash (f16 tensor-core bar); the decode call runs the
  split-KV decode kernel (f32 bar).
* DiT (src/cosyvoice-token2wav.cpp:240-420): a batch-2 cache with fixed and
  offloadable slots; bind_slot / slide_kv_slot (src/cosyvoice-kv-cache.cpp:
  415-467); offload_slot / load_slot (:148-246,276-290), whose host bytes must
  follow the reference layout (per layer: K of every batch entry, then V,
  :153-172) and whose round trip must restore the device bytes.

Every cache row written by update() must equal the oracle's quantization of
the same f32 rows byte for byte.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

D = 64
DEC_REL, FLASH_REL, MAX_ABS = 1e-5, 1e-3, 2e-3


def rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def device_rows(cv, cuda, t, n):
    """Bytes of positions [0, n) of every batch entry of a cache tensor: [ne2, n, row]."""
    host = np.zeros((t.ne2, n, t.nb1), dtype=np.uint8)
    if n:
        cv.check(cv.lib.cvattn_kv_copy_to_host(cuda.cuda.current_stream().cuda_stream, ctypes.byref(t), n,
                                               host.ctypes.data), "copy_to_host")
    cuda.cuda.synchronize()
    return host


def oracle_attention(oracle, kt, vt, kq, vq, q, mask=None):
    """q [B, n_q, Hq, D]; kq/vq [B, n_kv, row] bytes; mask f32 [n_q, n_kv] or None."""
    B, n_q, Hq, _ = q.shape
    Hkv = kq.shape[-1] // oracle.row_bytes(kt, D)
    out = np.zeros_like(q)
    for b in range(B):
        kd = oracle.dequantize(kt, kq[b], Hkv * D).reshape(-1, Hkv, D)
        vd = oracle.dequantize(vt, vq[b], Hkv * D).reshape(-1, Hkv, D)
        out[b] = oracle.attention_f64(q[b], kd, vd, 1.0 / 8.0, mask)
    return out


@pytest.mark.parametrize("kname,vname", [("q8_0", "q4_0"), ("f16", "f16"), ("q5_1", "q5_1")])
def test_llm_prefill_then_decode_through_the_cache_object(ctx, cv, cuda, oracle, kname, vname):
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    layers, Hq, Hkv, cap = 2, 14, 2, 640
    rng = np.random.default_rng(kt * 10 + vt)
    cache = cv.KVCache(ctx, layers, D, Hkv, cap, kt, vt, batch=1)
    assert cache.cur_len == 0 and cache.slot == 0
    k_rows = [np.zeros((0, Hkv * D), np.float32) for _ in range(layers)]
    v_rows = [np.zeros((0, Hkv * D), np.float32) for _ in range(layers)]

    def step(n, chunk_mask=False):
        cur = cache.cur_len
        pos = torch.arange(cur, cur + n, dtype=torch.int32, device="cuda")
        for layer in range(layers):
            k = rng.standard_normal((1, n, Hkv * D)).astype(np.float32)
            v = rng.standard_normal((1, n, Hkv * D)).astype(np.float32)
            q = rng.standard_normal((1, n, Hq, D)).astype(np.float32)
            cache.update(layer, torch.tensor(k, device="cuda"), torch.tensor(v, device="cuda"), pos)
            mode = cv.MASK_CAUSAL if n > 1 else cv.MASK_NONE
            out = cache.attention(layer, torch.tensor(q, device="cuda"), mask_mode=mode).cpu().numpy()
            k_rows[layer] = np.concatenate([k_rows[layer], k[0]])
            v_rows[layer] = np.concatenate([v_rows[layer], v[0]])
            kq = oracle.quantize(kt, k_rows[layer])[None]
            vq = oracle.quantize(vt, v_rows[layer])[None]
            # the cache rows are the oracle's blocks, byte for byte
            assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, 0, 0), cur + n), kq)
            assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, 0, 1), cur + n), vq)
            mask = oracle.mask_bits_to_f32(oracle.causal_mask(n, cur + n)) if n > 1 else None
            ref = oracle_attention(oracle, kt, vt, kq, vq, q, mask)
            bar = FLASH_REL if n > 1 else DEC_REL
            assert rel_l2(out, ref) <= bar and np.abs(out - ref).max() <= MAX_ABS, \
                f"{kname}/{vname} n={n} cur={cur} layer {layer}: rel-L2 {rel_l2(out, ref):.2e}"
        cache.shift(n)  # llm_prefill / llm_decode: cur_len += n_tokens
        assert cache.cur_len == cur + n

    step(256)   # one n_batch prefill call
    step(37)    # a second, ragged prefill call against the cached prompt
    for _ in range(3):
        step(1)  # decode steps
    cache.close()


def test_decode_call_neither_syncs_nor_allocates(ctx, cv, cuda, oracle):
    """attention_forward on the decode path is capturable in a CUDA graph: no host
    synchronization, no allocation, device lengths written by a kernel."""
    torch = cuda
    Hq, Hkv, cap = 14, 2, 512
    rng = np.random.default_rng(3)
    cache = cv.KVCache(ctx, 1, D, Hkv, cap, cv.Q8_0, cv.Q8_0, batch=1)
    k = rng.standard_normal((1, 200, Hkv * D)).astype(np.float32)
    v = rng.standard_normal((1, 200, Hkv * D)).astype(np.float32)
    cache.update(0, torch.tensor(k, device="cuda"), torch.tensor(v, device="cuda"),
                 torch.arange(200, dtype=torch.int32, device="cuda"))
    cache.shift(200)
    knew = torch.tensor(rng.standard_normal((1, 1, Hkv * D)).astype(np.float32), device="cuda")
    vnew = torch.tensor(rng.standard_normal((1, 1, Hkv * D)).astype(np.float32), device="cuda")
    pos = torch.tensor([200], dtype=torch.int32, device="cuda")
    q = torch.tensor(rng.standard_normal((1, 1, Hq, D)).astype(np.float32), device="cuda")
    out = torch.zeros_like(q)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())  # the rows and buffers above were written on the default stream
    with torch.cuda.stream(s):
        cache.update(0, knew, vnew, pos, stream=s)
        cache.attention(0, q, out=out, stream=s)   # warm-up outside the capture
    torch.cuda.synchronize()
    expected = out.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        g.capture_begin()
        cache.update(0, knew, vnew, pos, stream=s)
        cache.attention(0, q, out=out, stream=s)
        g.capture_end()
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, expected)
    kq = oracle.quantize(cv.Q8_0, np.concatenate([k[0], knew.cpu().numpy()[0]]))[None]
    vq = oracle.quantize(cv.Q8_0, np.concatenate([v[0], vnew.cpu().numpy()[0]]))[None]
    ref = oracle_attention(oracle, cv.Q8_0, cv.Q8_0, kq, vq, q.cpu().numpy())
    assert rel_l2(out.cpu().numpy(), ref) <= DEC_REL
    del g
    cache.close()


def test_workspace_reinit_after_stale_tickets(ctx, cv, cuda, oracle):
    """A caller workspace whose ticket counters were left counting (as a decode that
    gave up early leaves them) is made usable again by cvattn_workspace_init."""
    torch = cuda
    Hq, Hkv = 14, 2
    lens = [700, 1500, 90]
    rng = np.random.default_rng(9)
    cap = max(lens)
    kx = rng.standard_normal((len(lens), cap, Hkv * D)).astype(np.float32)
    vx = rng.standard_normal((len(lens), cap, Hkv * D)).astype(np.float32)
    kq, vq = oracle.quantize(cv.Q8_0, kx), oracle.quantize(cv.Q8_0, vx)
    kb = torch.tensor(kq.reshape(-1), device="cuda")
    vb = torch.tensor(vq.reshape(-1), device="cuda")
    kd = cv.kv_tensor(kb, cv.Q8_0, Hkv, D, cap, len(lens))
    vd = cv.kv_tensor(vb, cv.Q8_0, Hkv, D, cap, len(lens))
    q = torch.tensor(rng.standard_normal((len(lens), Hq, D)).astype(np.float32), device="cuda")
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    need = cv.decode_workspace_size(cv.Q8_0, cv.Q8_0, len(lens), cap, Hq, Hkv)
    ws = cv.alloc_workspace(need)
    ws[:256].fill_(3)                     # stale counts in every sequence's ticket
    cv.check(cv.lib.cvattn_workspace_init(torch.cuda.current_stream().cuda_stream, ws.data_ptr(), ws.numel()))
    out = cv.decode(ctx, q, kd, vd, kl, cap, workspace=ws).cpu().numpy()
    ref = np.zeros_like(out)
    for s, L in enumerate(lens):
        k = oracle.dequantize(cv.Q8_0, kq[s, :L], Hkv * D).reshape(L, Hkv, D)
        v = oracle.dequantize(cv.Q8_0, vq[s, :L], Hkv * D).reshape(L, Hkv, D)
        ref[s] = oracle.attention_f64(q.cpu().numpy()[s][None], k, v, 0.125)[0]
    assert rel_l2(out, ref) <= DEC_REL
    assert int(ws[:12].view(torch.int32).abs().sum()) == 0   # the kernels leave the tickets at zero


def test_cache_attention_repeated_lengths(ctx, cv, cuda, oracle):
    """Repeated decode calls through the object with a growing view reuse one workspace."""
    torch = cuda
    Hq, Hkv, cap, B = 14, 2, 300, 2
    rng = np.random.default_rng(17)
    cache = cv.KVCache(ctx, 1, D, Hkv, cap, cv.Q8_0, cv.Q4_0, batch=B)
    k = rng.standard_normal((B, cap, Hkv * D)).astype(np.float32)
    v = rng.standard_normal((B, cap, Hkv * D)).astype(np.float32)
    for n in (1, 63, 64, 65, 200):
        cache.cur_len = 0
        cache.update(0, torch.tensor(k[:, :n].copy(), device="cuda"), torch.tensor(v[:, :n].copy(), device="cuda"),
                     torch.arange(n, dtype=torch.int32, device="cuda"))
        q = rng.standard_normal((B, 1, Hq, D)).astype(np.float32)
        out = cache.attention(0, torch.tensor(q, device="cuda")).cpu().numpy()
        ref = oracle_attention(oracle, cv.Q8_0, cv.Q4_0, oracle.quantize(cv.Q8_0, k[:, :n]),
                               oracle.quantize(cv.Q4_0, v[:, :n]), q)
        assert rel_l2(out, ref) <= DEC_REL, f"n={n}"
    cache.close()


def _dit_cache(cv, ctx, layers, cap, n_fixed, n_offl, kt=None, vt=None):
    kt = cv.Q8_0 if kt is None else kt
    vt = cv.Q4_0 if vt is None else vt
    return cv.KVCache(ctx, layers, D, 16, cap, kt, vt, batch=2, n_slots=n_fixed + (1 if n_offl else 0),
                      n_offloaded_slots=n_offl)


def test_bind_and_slide_route_updates_to_slots(ctx, cv, cuda, oracle):
    torch = cuda
    layers, cap = 2, 128
    cache = _dit_cache(cv, ctx, layers, cap, n_fixed=3, n_offl=2)
    assert cache.slot == 0
    assert not cache.bind_slot(4) and cache.slot == 0          # n_slots = 3 + 1
    assert cache.bind_slot(2) and cache.slot == 2
    rng = np.random.default_rng(1)
    rows = {}
    for slot_expected in (2, 3):
        x = rng.standard_normal((2, 10, 16 * D)).astype(np.float32)
        for layer in range(layers):
            cache.update(layer, torch.tensor(x, device="cuda"), torch.tensor(x, device="cuda"),
                         torch.arange(10, dtype=torch.int32, device="cuda"))
        rows[slot_expected] = oracle.quantize(cv.Q8_0, x)
        if slot_expected == 2:
            cache.slide_slot()                                   # slide_kv_slot: cur_slot + 1
            assert cache.slot == 3
    with pytest.raises(cv.CvattnError):
        cache.slide_slot()                                       # past the last slot
    for slot, want in rows.items():
        for layer in range(layers):
            assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, slot, 0), 10), want)
    cache.close()


@pytest.mark.parametrize("other_stream", [False, True])
def test_offload_load_round_trip_reference_layout(ctx, cv, cuda, oracle, other_stream):
    torch = cuda
    layers, cap, n = 3, 96, 70
    cache = _dit_cache(cv, ctx, layers, cap, n_fixed=1, n_offl=2)
    rng = np.random.default_rng(5)
    pos = torch.arange(n, dtype=torch.int32, device="cuda")
    written = []
    for layer in range(layers):   # offloadable steps bind device slot 0
        k = rng.standard_normal((2, n, 16 * D)).astype(np.float32)
        v = rng.standard_normal((2, n, 16 * D)).astype(np.float32)
        cache.update(layer, torch.tensor(k, device="cuda"), torch.tensor(v, device="cuda"), pos)
        written.append((oracle.quantize(cv.Q8_0, k), oracle.quantize(cv.Q4_0, v)))
    # the reference's host layout: per layer, K rows of batch 0 then batch 1, then V
    expect = b"".join(kq.tobytes() + vq.tobytes() for kq, vq in written)
    s1 = torch.cuda.Stream()
    s2 = torch.cuda.Stream() if other_stream else s1
    s1.wait_stream(torch.cuda.current_stream())  # the slot's rows were appended on the default stream
    cache.offload_slot(1, n, stream=s1)      # enqueued only: no host synchronization
    host, length = cache.offloaded_slot(1)
    assert length == n and host.tobytes() == expect
    assert cache.offloaded_size >= len(expect)
    # the device slot is reused by the next utterance, then the offloaded slot comes back
    junk = torch.zeros((2, n, 16 * D), device="cuda")
    for layer in range(layers):
        cache.update(layer, junk, junk, pos)
    cache.cur_len = 5
    cache.bind_slot(1)                       # load_cache writes the bound slot
    s2.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s2):
        cache.load_slot(1, stream=s2)
    assert cache.cur_len == n               # load restores cur_len
    s2.synchronize()
    for layer in range(layers):
        assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, 1, 0), n), written[layer][0])
        assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, 1, 1), n), written[layer][1])
    # an empty host slot loads nothing and sets cur_len to 0
    cache.load_slot(0)
    assert cache.cur_len == 0
    cache.clear_offloaded()
    assert cache.offloaded_size == 0
    cache.close()


def test_offload_twice_overwrites_while_previous_load_pending(ctx, cv, cuda, oracle):
    """A second offload into the same host slot waits for the load still reading it."""
    torch = cuda
    layers, cap = 2, 64
    cache = _dit_cache(cv, ctx, layers, cap, n_fixed=1, n_offl=1)
    rng = np.random.default_rng(8)
    pos = torch.arange(40, dtype=torch.int32, device="cuda")
    data = []
    for rep in range(2):
        cache.bind_slot(0)
        cache.cur_len = 0                    # the load of the previous round set it to 40
        rows = []
        for layer in range(layers):
            x = rng.standard_normal((2, 40, 16 * D)).astype(np.float32)
            cache.update(layer, torch.tensor(x, device="cuda"), torch.tensor(x, device="cuda"), pos)
            rows.append((oracle.quantize(cv.Q8_0, x), oracle.quantize(cv.Q4_0, x)))
        data.append(rows)
        cache.offload_slot(0, 40)
        cache.bind_slot(1)
        cache.load_slot(0)
        for layer in range(layers):
            assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, 1, 0), 40), rows[layer][0])
            assert np.array_equal(device_rows(cv, cuda, cache.tensor(layer, 1, 1), 40), rows[layer][1])
    assert not np.array_equal(data[0][0][0], data[1][0][0])
    cache.close()


def test_dit_steps_with_plan_cached_chunk_attention(ctx, cv, cuda, oracle):
    """Three ODE steps of one streaming chunk, following dit_sched_config: the
    offloadable step binds slot 0, writes the chunk's K/V after the cached prompt,
    attends with the chunk mask, offloads; fixed steps own slots; the last step
    slides.  Attention is checked against the oracle at every step."""
    torch = cuda
    n_steps, n_offl, n_fixed = 10, 1, 2
    plan = cv.dit_sched_plan(n_steps, n_offl, n_fixed, 0, 0, True, True)
    assert [i for i, p in enumerate(plan) if p["cache_kv"]] == [7, 8, 9]
    layers, cap, P, S, H = 1, 256, 40, 100, 16
    cache = _dit_cache(cv, ctx, layers, cap, n_fixed=n_fixed, n_offl=n_offl)
    rng = np.random.default_rng(12)
    bounds = [50, 100]
    slot_offset = n_fixed - n_steps + 1        # src/cosyvoice-token2wav.cpp:365
    offload_slot = 0
    prompt = rng.standard_normal((2, P, H * D)).astype(np.float32)
    for step in (7, 8, 9):
        cfg = plan[step]
        cache.bind_slot(0 if cfg["offload"] else step + slot_offset)
        # the cached prompt keys of this slot (written by the prompt pass), then the chunk
        cache.cur_len = 0
        cache.update(0, torch.tensor(prompt, device="cuda"), torch.tensor(prompt, device="cuda"),
                     torch.arange(P, dtype=torch.int32, device="cuda"))
        cache.shift(P)
        k = rng.standard_normal((2, S, H * D)).astype(np.float32)
        v = rng.standard_normal((2, S, H * D)).astype(np.float32)
        q = rng.standard_normal((2, S, H, D)).astype(np.float32)
        cache.update(0, torch.tensor(k, device="cuda"), torch.tensor(v, device="cuda"),
                     torch.arange(P, P + S, dtype=torch.int32, device="cuda"))
        # attention_forward with the DiT's explicit f16 mask (src/cosyvoice-graph.cpp:453-460):
        # prompt columns visible, the chunk mask over the current frames
        bits = np.zeros((S, P + S), np.uint16)
        bits[:, P:] = oracle.chunk_mask(S, bounds)
        mask = torch.tensor(bits.view(np.int16), device="cuda")
        o = cache.attention(0, torch.tensor(q, device="cuda"), mask_mode=cv.MASK_EXPLICIT, mask=mask).cpu().numpy()
        kq = oracle.quantize(cv.Q8_0, np.concatenate([prompt, k], axis=1))
        vq = oracle.quantize(cv.Q4_0, np.concatenate([prompt, v], axis=1))
        ref = oracle_attention(oracle, cv.Q8_0, cv.Q4_0, kq, vq, q, oracle.mask_bits_to_f32(bits))
        assert rel_l2(o, ref) <= FLASH_REL and np.abs(o - ref).max() <= MAX_ABS, f"step {step}"
        if cfg["offload"]:
            cache.offload_slot(offload_slot, cache.cur_len + S)
            offload_slot += 1
            host, n = cache.offloaded_slot(0)
            assert n == P + S and host.size == (P + S) * 2 * (kq.shape[-1] + vq.shape[-1])
        if cfg["slide"]:
            cache.slide_slot()
    cache.close()
