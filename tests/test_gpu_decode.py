"""GPU: split-KV decode attention vs the fp64 oracle.

ggml_flash_attn_ext with one query row, no mask, scale 1/sqrt(64), f32
precision requested (src/cosyvoice-kv-cache.cpp:379-386, via
src/cosyvoice-llm.cpp:62) on Qwen2 shapes: 14 query heads, 2 KV heads, D=64.
The kernel computes in fp32 on exactly dequantized K/V, so the bar is the
north-star's f32 one: relative L2 <= 1e-5 (and max-abs <= 2e-3) against fp64
attention over the oracle-dequantized cache.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HQ, HKV, D = 14, 2, 64
SCALE = 1.0 / 8.0
REL_L2 = 1e-5
MAX_ABS = 2e-3
ALL = ["f32", "f16", "q8_0", "q5_1", "q5_0", "q4_1", "q4_0"]


def rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def build(cv, cuda, oracle, kt, vt, lens, rng, cap=None, outliers=False):
    torch = cuda
    n_seq = len(lens)
    cap = cap or max(lens)
    row = HKV * D
    kx = rng.standard_normal((n_seq, cap, row)).astype(np.float32)
    vx = rng.standard_normal((n_seq, cap, row)).astype(np.float32)
    if outliers:
        for a in (kx, vx):
            hit = rng.random(a.shape) < 0.01
            a[hit] = np.where(rng.random(hit.sum()) < 0.5, -8.0, 8.0)
    kq, vq = oracle.quantize(kt, kx), oracle.quantize(vt, vx)
    kbuf = torch.tensor(kq.reshape(-1), device="cuda")
    vbuf = torch.tensor(vq.reshape(-1), device="cuda")
    kd = cv.kv_tensor(kbuf, kt, HKV, D, cap, n_seq)
    vd = cv.kv_tensor(vbuf, vt, HKV, D, cap, n_seq)
    return kq, vq, kbuf, vbuf, kd, vd


def reference(oracle, kt, vt, kq, vq, q, lens):
    out = np.zeros_like(q)
    for s, L in enumerate(lens):
        if L == 0:
            continue
        kd = oracle.dequantize(kt, kq[s, :L], HKV * D).reshape(L, HKV, D)
        vd = oracle.dequantize(vt, vq[s, :L], HKV * D).reshape(L, HKV, D)
        out[s] = oracle.attention_f64(q[s][None], kd, vd, SCALE)[0]
    return out


PATHS = {"warp_mma": {"warp_mma": True}, "tmem_stream": {"tmem_stream": True}, "wide": {"wide_chunks": True}, "tensor_cores": {"not_persistent": True},
         "cuda_cores": {"cuda_cores": True}}


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("kname", ALL)
@pytest.mark.parametrize("vname", ALL)
def test_decode_type_pairs(ctx, cv, cuda, oracle, kname, vname, path):
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(kt * 16 + vt)
    lens = [1, 64, 129, 300]
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, outliers=True)
    q = rng.standard_normal((len(lens), HQ, D)).astype(np.float32)
    qt = torch.tensor(q, device="cuda")
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, qt, kd, vd, kl, max(lens), **PATHS[path]).cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    assert rel_l2(out, ref) <= REL_L2, f"{kname}/{vname} {path} rel-L2 {rel_l2(out, ref):.3e}"
    assert np.abs(out - ref).max() <= MAX_ABS


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("kname,vname", [("q8_0", "q8_0"), ("q8_0", "q4_0"), ("q5_1", "q5_1"), ("f16", "f16")])
def test_decode_mixed_lengths_64_sequences(ctx, cv, cuda, oracle, kname, vname, path):
    """The benchmark mix: 64 sequences, lengths U[128, 2048] (seed 0)."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    lens = np.random.default_rng(0).integers(128, 2049, 64).tolist()
    rng = np.random.default_rng(11)
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, cap=2048)
    q = rng.standard_normal((64, HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, 2048, **PATHS[path]).cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    assert rel_l2(out, ref) <= REL_L2
    assert np.abs(out - ref).max() <= MAX_ABS


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("kname,vname", [("q8_0", "q8_0"), ("q5_1", "q4_1"), ("f16", "q5_0"), ("f32", "f32")])
def test_decode_fused_append(ctx, cv, cuda, oracle, kname, vname, path):
    """The step's K/V row is quantized into the cache at kv_len-1 and attended to."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(21)
    lens = [1, 128, 129, 257, 700]
    cap = 768
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, cap=cap)
    n = len(lens)
    knew = rng.standard_normal((n, HKV * D)).astype(np.float32)
    vnew = rng.standard_normal((n, HKV * D)).astype(np.float32)
    q = rng.standard_normal((n, HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, max(lens), **PATHS[path],
                    k_new=torch.tensor(knew, device="cuda"), v_new=torch.tensor(vnew, device="cuda")).cpu().numpy()
    kq2, vq2 = kq.copy(), vq.copy()
    for s, L in enumerate(lens):
        kq2[s, L - 1] = oracle.quantize(kt, knew[s:s + 1])[0]
        vq2[s, L - 1] = oracle.quantize(vt, vnew[s:s + 1])[0]
    kgot = kb.view(n, cap, -1).cpu().numpy()
    vgot = vb.view(n, cap, -1).cpu().numpy()
    assert np.array_equal(kgot, kq2) and np.array_equal(vgot, vq2), "appended rows differ from the oracle"
    ref = reference(oracle, kt, vt, kq2, vq2, q, lens)
    assert rel_l2(out, ref) <= REL_L2


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_separate_worker_buffers(ctx, cv, cuda, oracle, path):
    """Per-sequence row pointers: each worker owns its own cache buffer."""
    torch = cuda
    kt = vt = cv.Q8_0
    rng = np.random.default_rng(7)
    lens = [100, 1000, 513]
    bufs, kqs, vqs = [], [], []
    for L in lens:
        kx = rng.standard_normal((L, HKV * D)).astype(np.float32)
        vx = rng.standard_normal((L, HKV * D)).astype(np.float32)
        kq, vq = oracle.quantize(kt, kx), oracle.quantize(vt, vx)
        kqs.append(kq)
        vqs.append(vq)
        bufs.append((torch.tensor(kq.reshape(-1), device="cuda"), torch.tensor(vq.reshape(-1), device="cuda")))
    kp = torch.tensor([b[0].data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    vp = torch.tensor([b[1].data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    desc_k = cv.kv_tensor(bufs[0][0], kt, HKV, D, max(lens), len(lens))
    desc_v = cv.kv_tensor(bufs[0][1], vt, HKV, D, max(lens), len(lens))
    q = rng.standard_normal((len(lens), HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), desc_k, desc_v, kl, max(lens),
                    k_seq_ptrs=kp, v_seq_ptrs=vp, **PATHS[path]).cpu().numpy()
    for s, L in enumerate(lens):
        kd = oracle.dequantize(kt, kqs[s], HKV * D).reshape(L, HKV, D)
        vd = oracle.dequantize(vt, vqs[s], HKV * D).reshape(L, HKV, D)
        ref = oracle.attention_f64(q[s][None], kd, vd, SCALE)[0]
        assert rel_l2(out[s], ref) <= REL_L2


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_split_partials_and_combine(ctx, cv, cuda, oracle, path):
    """Long-context split-KV: two position shards emit partials, combine merges them."""
    torch = cuda
    kt, vt = cv.Q8_0, cv.Q4_0
    rng = np.random.default_rng(9)
    L = 3000
    cut = 1216
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, [L], rng)
    q = rng.standard_normal((1, HQ, D)).astype(np.float32)
    qt = torch.tensor(q, device="cuda")
    rbk, rbv = cv.row_size(kt, 128), cv.row_size(vt, 128)
    po = torch.empty((2, HQ, D), dtype=torch.float32, device="cuda")
    pml = torch.empty((2, HQ, 2), dtype=torch.float32, device="cuda")
    for part, (start, n) in enumerate([(0, cut), (cut, L - cut)]):
        kp = torch.tensor([kb.data_ptr() + start * rbk], dtype=torch.int64, device="cuda")
        vp = torch.tensor([vb.data_ptr() + start * rbv], dtype=torch.int64, device="cuda")
        kl = torch.tensor([n], dtype=torch.int32, device="cuda")
        cv.decode(ctx, qt, kd, vd, kl, n, out=po[part:part + 1], k_seq_ptrs=kp, v_seq_ptrs=vp,
                  emit_partial=True, partial_ml=pml[part:part + 1], **PATHS[path])
    out = cv.combine(po, pml).cpu().numpy().reshape(1, HQ, D)
    ref = reference(oracle, kt, vt, kq, vq, q, [L])
    assert rel_l2(out, ref) <= REL_L2


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_zero_and_invalid_lengths(ctx, cv, cuda, oracle, path):
    torch = cuda
    kt = vt = cv.Q8_0
    rng = np.random.default_rng(13)
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, [200, 200, 200], rng)
    q = torch.tensor(rng.standard_normal((3, HQ, D)).astype(np.float32), device="cuda")
    # seq 0 empty -> zeros; seq 2 longer than the launch bound -> zeros + status
    kl = torch.tensor([0, 150, 190], dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, q, kd, vd, kl, 160, **PATHS[path]).cpu().numpy()
    assert not out[0].any() and not out[2].any()
    assert np.abs(out[1]).sum() > 0
    st, detail = ctx.sync_status()
    assert st == 6 and detail == 2


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_workspace_reuse_many_calls(ctx, cv, cuda, oracle, path):
    """The ticket counters return to zero: repeated calls on one workspace agree."""
    torch = cuda
    kt = vt = cv.Q8_0
    rng = np.random.default_rng(17)
    lens = [1500, 700, 2048, 129]
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng)
    q = torch.tensor(rng.standard_normal((4, HQ, D)).astype(np.float32), device="cuda")
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    dec = cv.Decoder(ctx, kd, vd, 4, HQ, 2048, q, out, kl, **PATHS[path])
    dec()
    first = out.clone()
    for _ in range(20):
        dec()
    torch.cuda.synchronize()
    assert torch.equal(first, out)


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
@pytest.mark.parametrize("qscale,vscale", [(1e-3, 1.0), (300.0, 1.0), (1.0, 1e3), (1.0, 1e-4)])
def test_decode_tensor_core_scaling_extremes(ctx, cv, cuda, oracle, qscale, vscale, path):
    """Q and V magnitudes far from 1 keep the f32 bar (exact power-of-two scaling of the hi/lo splits)."""
    torch = cuda
    kt, vt = cv.Q8_0, cv.Q5_1
    rng = np.random.default_rng(31)
    lens = [77, 600]
    cap = 600
    kx = rng.standard_normal((2, cap, HKV * D)).astype(np.float32)
    vx = (rng.standard_normal((2, cap, HKV * D)) * vscale).astype(np.float32)
    kq, vq = oracle.quantize(kt, kx), oracle.quantize(vt, vx)
    kd = cv.kv_tensor(torch.tensor(kq.reshape(-1), device="cuda"), kt, HKV, D, cap, 2)
    vd = cv.kv_tensor(torch.tensor(vq.reshape(-1), device="cuda"), vt, HKV, D, cap, 2)
    q = (rng.standard_normal((2, HQ, D)) * qscale).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, cap, **PATHS[path]).cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    assert rel_l2(out, ref) <= REL_L2, f"rel-L2 {rel_l2(out, ref):.3e}"


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream", "wide", "tensor_cores"])
@pytest.mark.parametrize("kname,vname", [("q8_0", "q4_0"), ("q5_1", "q5_1")])
def test_decode_many_chunks_per_sm(ctx, cv, cuda, oracle, kname, vname, path):
    """Hundreds of sequences: each persistent CTA walks a range of several
    chunks, so runs merge consecutive chunks, cover whole sequences, and cross
    CTA boundaries; the combine reads only the written partials."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(41)
    lens = rng.integers(1, 3001, 300).tolist()
    lens[:4] = [1, 128, 3000, 2999]
    cap = 3000
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, cap=cap, outliers=True)
    q = rng.standard_normal((len(lens), HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, cap, **PATHS[path]).cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    assert rel_l2(out, ref) <= REL_L2, f"rel-L2 {rel_l2(out, ref):.3e}"
    assert np.abs(out - ref).max() <= MAX_ABS


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_many_chunks_emit_partial(ctx, cv, cuda, oracle, path):
    """Partials (unnormalized O, max in log2 units, sum) of the merged runs."""
    torch = cuda
    kt = vt = cv.Q8_0
    rng = np.random.default_rng(43)
    lens = rng.integers(1, 2049, 260).tolist()
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, cap=2048)
    q = rng.standard_normal((len(lens), HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    pml = torch.zeros((len(lens), HQ, 2), dtype=torch.float32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, 2048, emit_partial=True,
                    partial_ml=pml, **PATHS[path]).cpu().numpy()
    ml = pml.cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    assert rel_l2(out / ml[:, :, 1:2], ref) <= REL_L2
    for s in (0, 7, 100):  # the max is the true max score (log2 units)
        L = lens[s]
        kdq = oracle.dequantize(kt, kq[s, :L], HKV * D).reshape(L, HKV, D).astype(np.float64)
        for h in (0, 13):
            smax = (kdq[:, h // 7, :] @ q[s, h].astype(np.float64)).max() * SCALE / np.log(2.0)
            assert abs(ml[s, h, 0] - smax) <= 1e-4 * max(1.0, abs(smax))


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_long_sequences_direct_combine(ctx, cv, cuda, oracle, path):
    """More than 64 chunks per sequence: the merge streams every chunk slot and skips empty ones."""
    torch = cuda
    kt, vt = cv.Q8_0, cv.Q8_0
    rng = np.random.default_rng(47)
    lens = [9000, 8999, 129, 7000, 4000, 1] + [8500] * 6  # ~850 chunks: runs of several chunks per CTA half
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, cap=9000)
    q = rng.standard_normal((len(lens), HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, 9000, **PATHS[path]).cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    assert rel_l2(out, ref) <= REL_L2, f"rel-L2 {rel_l2(out, ref):.3e}"


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
def test_decode_step_of_layers_inputs_ready(ctx, cv, cuda, oracle, path):
    """One model step of several layers launched back to back with the fused
    append and DECODE_INPUTS_READY (each launch streams its K/V while the
    previous layer finishes), repeated for two steps: outputs and appended rows
    match the oracle."""
    torch = cuda
    kt = vt = cv.Q8_0
    rng = np.random.default_rng(53)
    layers, lens, cap = 4, rng.integers(100, 900, 24).tolist(), 1024
    n = len(lens)
    caches = [build(cv, cuda, oracle, kt, vt, lens, rng, cap=cap) for _ in range(layers)]
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    for step in range(2):
        q = rng.standard_normal((layers, n, HQ, D)).astype(np.float32)
        knew = rng.standard_normal((layers, n, HKV * D)).astype(np.float32)
        vnew = rng.standard_normal((layers, n, HKV * D)).astype(np.float32)
        qt, kt_, vt_ = (torch.tensor(x, device="cuda") for x in (q, knew, vnew))
        outs = torch.empty_like(qt)
        decs = [cv.Decoder(ctx, caches[l][4], caches[l][5], n, HQ, cap, qt[l], outs[l], kl, k_new=kt_[l], v_new=vt_[l],
                           inputs_ready=True, **PATHS[path]) for l in range(layers)]
        for d in decs:
            d()
        got = outs.cpu().numpy()
        cur = (np.array(lens) + step).tolist()
        for l in range(layers):
            kq, vq = caches[l][0], caches[l][1]
            for s, L in enumerate(cur):
                kq[s, L - 1] = oracle.quantize(kt, knew[l, s:s + 1])[0]
                vq[s, L - 1] = oracle.quantize(vt, vnew[l, s:s + 1])[0]
            ref = reference(oracle, kt, vt, kq, vq, q[l], cur)
            assert rel_l2(got[l], ref) <= REL_L2, f"step {step} layer {l}: rel-L2 {rel_l2(got[l], ref):.3e}"
        kl = torch.tensor([L + step + 1 for L in lens], dtype=torch.int32, device="cuda")  # uploaded, as the contract asks
    for l in range(layers):
        assert np.array_equal(caches[l][2].view(n, cap, -1).cpu().numpy(), caches[l][0]), "appended K rows"


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream", "wide"])
@pytest.mark.parametrize("kname,vname", [("q8_0", "q8_0"), ("q4_1", "q5_1")])
def test_decode_running_rescales(ctx, cv, cuda, oracle, kname, vname, path):
    """Scores that grow along the sequence and V magnitudes that jump by 2^+-9
    between 64-position stretches: the streaming kernel's running output is
    rescaled whenever its reference max or its P' scale has to move."""
    torch = cuda
    kt, vt = cv.TYPE_BY_NAME[kname], cv.TYPE_BY_NAME[vname]
    rng = np.random.default_rng(59)
    lens = [2000, 1999, 640, 65, 1500, 1]
    cap, n = 2000, len(lens)
    pos = np.arange(cap, dtype=np.float32)
    kx = rng.standard_normal((n, cap, HKV * D)).astype(np.float32) * (0.2 + pos / 400.0)[None, :, None]
    vx = rng.standard_normal((n, cap, HKV * D)).astype(np.float32)
    vx *= (2.0 ** rng.integers(-9, 10, (n, cap // 64 + 1)).astype(np.float32)).repeat(64, axis=1)[:, :cap, None]
    kq, vq = oracle.quantize(kt, kx), oracle.quantize(vt, vx)
    kd = cv.kv_tensor(torch.tensor(kq.reshape(-1), device="cuda"), kt, HKV, D, cap, n)
    vd = cv.kv_tensor(torch.tensor(vq.reshape(-1), device="cuda"), vt, HKV, D, cap, n)
    q = rng.standard_normal((n, HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, cap, **PATHS[path]).cpu().numpy()
    ref = reference(oracle, kt, vt, kq, vq, q, lens)
    for s in range(n):
        assert rel_l2(out[s], ref[s]) <= REL_L2, f"seq {s} rel-L2 {rel_l2(out[s], ref[s]):.3e}"


@pytest.mark.parametrize("path", ["warp_mma", "tmem_stream"])
@pytest.mark.parametrize("shape", ["one_long", "six_runs_per_cta", "headline_mix", "eight_long"])
def test_decode_merge_shapes(ctx, cv, cuda, oracle, path, shape):
    """Split sequences merged at the end of the launch: one sequence over more than 64
    warp pairs (merged by its elected warp alone), 148 sequences of six chunks (six runs
    of a sequence inside one CTA, several merges per CTA), the headline's mix of 64
    sequences with lengths in [128, 2048], and eight sequences of 2048 (each over ~33
    pairs: CTA-wide merges of more than 32 runs)."""
    torch = cuda
    kt, vt = cv.Q8_0, cv.Q4_0
    rng = np.random.default_rng(53)
    if shape == "one_long":
        lens = [5000, 1, 64, 65, 127]
    elif shape == "six_runs_per_cta":
        lens = [384] * 148
    elif shape == "eight_long":
        lens = [2048] * 8
    else:
        lens = np.random.default_rng(0).integers(128, 2049, 64).tolist()
    cap = max(lens)
    kq, vq, kb, vb, kd, vd = build(cv, cuda, oracle, kt, vt, lens, rng, cap=cap)
    q = rng.standard_normal((len(lens), HQ, D)).astype(np.float32)
    kl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the tickets are left at zero for the next launch
        out = cv.decode(ctx, torch.tensor(q, device="cuda"), kd, vd, kl, cap, **PATHS[path]).cpu().numpy()
        ref = reference(oracle, kt, vt, kq, vq, q, lens)
        assert rel_l2(out, ref) <= REL_L2, f"rel-L2 {rel_l2(out, ref):.3e}"
        assert np.abs(out - ref).max() <= MAX_ABS
