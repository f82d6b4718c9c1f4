"""Benchmark of the cvattn engine on the reference's headline workload.

Headline (N=1): Qwen2-0.5B-shaped LLM decode
attention over all 24 layers, q8_0 KV cache (ggml blocks), 64 concurrent
sequences with context lengths U[128, 2048] (numpy default_rng(0), sum 70,843),
K/V ~ N(0,1) before quantization.  One step = every layer's fused
append-of-the-new-token + split-KV attention for all 64 sequences, launched
as one CUDA graph of 24 kernels.  metric = KV bytes streamed by attention per
second (GB/s, whole job); tok/s = sequences x steps / s.

Multi-GPU (torchrun, one process per GPU): every rank serves its own 64
sequences (weak scaling: requests shard by sequence, no collective on the
path); time = max over ranks of the CUDA-event time.  At every N the line also
carries the north-star's sharded workloads (strong scaling, max over ranks):
configs[3]'s 256 sequences x 4096 split across the ranks by shard_by_length,
and configs[4]'s 32 utterances (CFG 2, 22 layers, cached prompt) split across
the ranks.

--impl reference times the reference's CPU attention path restated by the
oracle (ggml is not available to build) on the host cores, on a bounded
sample of the same workload.

Secondary figures at N=1: configs[0] latency, configs[1] at fixed lengths,
configs[2] prefill (one launch, and as the reference issues it: 256-token
calls with the fused append), configs[4] DiT attention with f16 and with the
reference's default q8_0 / q4_0 cache, and the decode step with RoPE fused in.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cosyvoice.cpp_b200"))
sys.path.insert(0, ROOT)

HQ, HKV, D, LAYERS, N_SEQ, CAP = 14, 2, 64, 24, 64, 2048
METRIC = "LLM decode-attn KV GB/s + tok/s (frac HBM peak); DiT attn TFLOP/s at 1/2/4/8 GPU"
WORKLOAD = "qwen2-0.5b decode attention, 24 layers, q8_0 KV, 64 seqs, L~U[128,2048] (seed 0)"
# DiT: 22 blocks, 16 heads, 600 query frames, 300 cached prompt frames, 50-frame chunks
DIT_LAYERS, DIT_H, DIT_P, DIT_S, DIT_UTT, DIT_STEPS = 22, 16, 300, 600, 32, 10


def seq_lengths() -> list[int]:
    return np.random.default_rng(0).integers(128, 2049, N_SEQ).tolist()


def headline_config(world: int) -> dict:
    """The `config` of the headline line (both arms print the same dict)."""
    lens = seq_lengths()
    row = 34 * (HKV * D // 32)
    bytes_per_step = sum(lens) * 2 * row * LAYERS
    return {"workload": WORKLOAD, "layers": LAYERS, "n_seq_per_gpu": N_SEQ, "q_heads": HQ,
            "kv_heads": HKV, "head_dim": D, "kv_type": "q8_0", "sum_kv_len": sum(lens),
            "kv_bytes_per_step": bytes_per_step,
            "l2": "inputs larger than L2: %.0f MB of KV per step vs 126 MB L2" % (bytes_per_step / 1e6),
            "step": "CUDA graph of 24 fused append+attention launches",
            "parallelism": f"sequence-sharded x{world}"}


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profiled_traffic() -> dict:
    """Per-launch DRAM bytes of the dominant kernels from the committed ncu summaries."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi SM clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ helpers

def _sync_max(torch, dist, ms: float) -> float:
    """The max over ranks of a device time (ms)."""
    if dist is None:
        return ms
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(torch, dist):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def _graph_of(torch, stream, fn, warm: int = 3):
    """Warm fn up on `stream`, then capture one call of it in a CUDA graph.  The inputs
    were made on the default stream: wait for them first."""
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(warm):
            fn(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        g.capture_begin()
        fn(stream)
        g.capture_end()
    torch.cuda.synchronize()
    return g


def _time_graph(torch, stream, graph, reps: int, warm: int = 2) -> float:
    """CUDA-event ms per replay of graph on stream."""
    with torch.cuda.stream(stream):
        for _ in range(warm):
            graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def _check_status(ctx, what: str):
    st, detail = ctx.sync_status()
    if st != 0:
        raise RuntimeError(f"device status {st} ({detail}) after {what}")


# ------------------------------------------------------------------ our arm

def build_decode_workload_layers(torch, cv, ctx, n_layers: int):
    return build_decode_workload(torch, cv, ctx, cv.Q8_0, 0, n_layers)


def build_decode_workload(torch, cv, ctx, kv_type: int, rank: int, n_layers: int = LAYERS, lens=None):
    """Device-resident caches for n_layers x 64 sequences (seeded), appended by the engine."""
    lens = seq_lengths() if lens is None else lens
    cap = max(CAP, max(lens))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234 + rank)
    caches = []
    pos = torch.arange(cap, dtype=torch.int32, device="cuda")
    for layer in range(n_layers):
        kb, kd = cv.alloc_kv(kv_type, HKV, D, cap, N_SEQ)
        vb, vd = cv.alloc_kv(kv_type, HKV, D, cap, N_SEQ)
        for buf_desc in (kd, vd):
            x = torch.randn(N_SEQ, cap, HKV * D, device="cuda", generator=gen)
            cv.kv_append(ctx, buf_desc, x, pos)   # quantize-on-write, bit-exact ggml blocks
            del x
        caches.append((kb, kd, vb, vd))
    torch.cuda.synchronize()
    q = torch.randn(n_layers, N_SEQ, HQ, D, device="cuda", generator=gen)
    k_new = torch.randn(n_layers, N_SEQ, HKV * D, device="cuda", generator=gen)
    v_new = torch.randn(n_layers, N_SEQ, HKV * D, device="cuda", generator=gen)
    out = torch.empty_like(q)
    kv_len = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return lens, caches, q, k_new, v_new, out, kv_len


def run_ours(args, rank: int, world: int, torch, dist) -> dict | None:
    import cvattn as cv
    dev = torch.cuda.current_device()
    ctx = cv.Context(dev)
    kv_type = cv.Q8_0
    lens, caches, q, k_new, v_new, out, kv_len = build_decode_workload(torch, cv, ctx, kv_type, rank)
    cap = CAP
    row = cv.row_size(kv_type, HKV * D)
    bytes_per_layer = sum(lens) * 2 * row            # K and V rows read by attention
    bytes_per_step = bytes_per_layer * LAYERS
    # one model step: every layer's fused append + attention; the lengths are
    # uploaded once and no layer writes another layer's cache, so each launch may
    # stream its K/V while the previous layer finishes (DECODE_INPUTS_READY)
    decs = [cv.Decoder(ctx, caches[l][1], caches[l][3], N_SEQ, HQ, cap, q[l], out[l], kv_len,
                       k_new=k_new[l], v_new=v_new[l], inputs_ready=True) for l in range(LAYERS)]
    stream = torch.cuda.Stream()

    def step(s):
        for d in decs:
            d(s)

    # warm-up and CUDA-graph capture of one step (24 launches)
    graph = _graph_of(torch, stream, step, warm=max(args.warmup, 3))
    _check_status(ctx, "warm-up")

    # ---- device-resident timed region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    _barrier(torch, dist)
    with ClockSampler(dev) as clocks:
        # the sampler reads clocks every 200 ms: keep the same load running for a
        # moment right before the timed steps so the samples reflect it
        t_soak = time.perf_counter() + 0.6
        while time.perf_counter() < t_soak:
            with torch.cuda.stream(stream):
                graph.replay()
            torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    _barrier(torch, dist)
    ms_max = _sync_max(torch, dist, ms)
    ms_per_step = ms_max / args.steps

    # ---- per-launch duration of the dominant kernel: the timed region holds only
    # the decode kernel (24 launches per step), so its average launch is the step / 24
    launch_us = 1000.0 * (ms / args.steps) / LAYERS

    e2e = run_e2e(args, torch, cv, ctx, dist, caches, q, k_new, v_new, out, kv_len, bytes_per_step, world)
    _check_status(ctx, "the e2e region")
    del graph

    lines = {}
    # north-star sharded workloads at every N (strong scaling over the ranks)
    if not args.skip_secondary:
        lines.update(run_decode_cfg4_sharded(torch, cv, ctx, rank, world, dist))
        lines.update(run_dit_sharded(torch, cv, ctx, rank, world, dist))
    if rank == 0 and world == 1 and not args.skip_secondary:
        lines.update(run_flash_secondary(torch, cv, ctx, args))
        lines.update(run_decode_rope(torch, cv, ctx, caches, q, k_new, v_new, out, kv_len, bytes_per_layer,
                                     launch_us))
        del caches, q, k_new, v_new, out, decs
        torch.cuda.empty_cache()
        lines.update(run_configs0(torch, cv, ctx))
        lines.update(run_configs1_fixed(torch, cv, ctx))
        lines.update(run_prefill_chunked(torch, cv, ctx))
        lines.update(run_dit_offload(torch, cv, ctx))
    if rank != 0:
        return None

    peaks = measured_peaks()
    value = world * bytes_per_step / (ms_per_step * 1e-3) / 1e9
    achieved = bytes_per_layer / (launch_us * 1e-6) / 1e9
    traffic = profiled_traffic().get("decode_q8_0_mix_per_launch")
    return {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) K/V quantized to q8_0 by the engine's bit-exact append)",
        "config": headline_config(world),
        "tok_per_s": round(world * N_SEQ / (ms_per_step * 1e-3), 1),
        "frac_hbm_peak": round(value / world / peaks["hbm_gbs"], 4),
        "e2e": e2e,
        "roofline": {"bound": "hbm",
                     "kernel": decode_kernel_name(N_SEQ, N_SEQ * (CAP // 64),
                                                  torch.cuda.get_device_properties(dev).multi_processor_count)
                     + "<q8_0,q8_0>", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": peaks["source"], "launch_us": round(launch_us, 3),
                     "algorithmic_bytes_per_launch": bytes_per_layer, "traffic": traffic},
        "gpu_launches": args.steps * LAYERS,
        "clocks": clocks.summary(),
        **lines,
    }


def run_e2e(args, torch, cv, ctx, dist, caches, q, k_new, v_new, out, kv_len, bytes_per_step: int, world: int) -> dict:
    """End to end through the C ABI: pinned host Q/K/V rows in and outputs back every step.

    Two buffer sets and a copy stream: the inputs of step i + 1 upload and the
    outputs of step i - 1 download while the kernels of step i run.  The 24
    cvattn_decode calls of a buffer set are captured once in a CUDA graph that
    every step replays (how a serving loop issues a fixed layer stack); the
    ungraphed calls, the copies alone and the launches alone are timed too, so
    the line says which of them bounds the step."""
    hq = torch.empty_like(q, device="cpu").pin_memory()
    hk = torch.empty_like(k_new, device="cpu").pin_memory()
    hv = torch.empty_like(v_new, device="cpu").pin_memory()
    hout = torch.empty_like(out, device="cpu").pin_memory()
    hq.copy_(q.cpu()); hk.copy_(k_new.cpu()); hv.copy_(v_new.cpu())
    h2d = hq.numel() * 4 + hk.numel() * 4 + hv.numel() * 4
    d2h = hout.numel() * 4
    cap = CAP

    q2, kn2, vn2, out2 = q.clone(), k_new.clone(), v_new.clone(), torch.empty_like(out)
    sets = []
    for (qq, kk, vv, oo) in ((q, k_new, v_new, out), (q2, kn2, vn2, out2)):
        decs = [cv.Decoder(ctx, caches[l][1], caches[l][3], N_SEQ, HQ, cap, qq[l], oo[l], kv_len,
                           k_new=kk[l], v_new=vv[l], inputs_ready=True) for l in range(LAYERS)]
        sets.append((qq, kk, vv, oo, decs))
    stream = torch.cuda.Stream()
    cstream = torch.cuda.Stream()
    graphs = [_graph_of(torch, stream, lambda s, ds=st[4]: [d(s) for d in ds]) for st in sets]
    houts = [hout, torch.empty_like(hout).pin_memory()]
    ev = lambda: torch.cuda.Event()
    h2d_done = [ev(), ev()]
    comp_done = [ev(), ev()]

    def upload(i):
        dq, dk, dv, _, _ = sets[i & 1]
        with torch.cuda.stream(cstream):
            if i >= 2:
                cstream.wait_event(comp_done[i & 1])  # step i - 2 is done with this set
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            h2d_done[i & 1].record(cstream)

    def compute(i, graphed=True, copies=True):
        if copies:
            stream.wait_event(h2d_done[i & 1])
        if graphed:
            with torch.cuda.stream(stream):
                graphs[i & 1].replay()
        else:
            for d in sets[i & 1][4]:
                d(stream)
        comp_done[i & 1].record(stream)

    def download(i):
        with torch.cuda.stream(cstream):
            cstream.wait_event(comp_done[i & 1])
            houts[i & 1].copy_(sets[i & 1][3], non_blocking=True)

    def run(n, graphed=True, copies=True, kernels=True):
        if copies:
            upload(0)
        for i in range(n):
            if copies and i + 1 < n:
                upload(i + 1)
            if kernels:
                compute(i, graphed, copies)
            else:
                comp_done[i & 1].record(cstream)
            if copies:
                download(i)

    def timed(**kw) -> float:
        run(3, **kw)
        torch.cuda.synchronize()
        _barrier(torch, dist)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cstream)
        stream.wait_stream(cstream)
        run(args.steps, **kw)
        stream.wait_stream(cstream)
        cstream.wait_stream(stream)
        e1.record(cstream)
        e1.synchronize()
        return _sync_max(torch, dist, e0.elapsed_time(e1)) / args.steps

    ms_graphed = timed(graphed=True)
    ms_calls = timed(graphed=False)
    ms_copies = timed(kernels=False)
    ms_launch = timed(graphed=False, copies=False)
    for g in graphs:
        del g
    gbs = lambda ms: round(world * bytes_per_step / (ms * 1e-3) / 1e9, 1)
    return {"value": gbs(ms_graphed), "unit": "GB/s", "ms_per_step": round(ms_graphed, 4),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "cvattn_decode via the C ABI, the 24 calls of a step captured once in a CUDA graph and replayed; "
                    "pinned host Q/K/V rows in and outputs back every step on a copy stream with two buffer sets",
            "diag_ms_per_step": {"api_calls_each_step": round(ms_calls, 4), "copies_only": round(ms_copies, 4),
                                 "api_calls_only_no_copies": round(ms_launch, 4), "graphed": round(ms_graphed, 4)},
            "api_calls_value": gbs(ms_calls)}


def run_decode_rope(torch, cv, ctx, caches, q, k_new, v_new, out, kv_len, bytes_per_layer: int, launch_us: float,
                    reps: int = 20) -> dict:
    """The headline step with the decode RoPE fused in (Q and the appended K row
    turn by kv_len - 1; NEOX, rope_theta 1e6, src/cosyvoice-llm.cpp:56-57): the
    same 24-launch graph through cvattn_decode_rope."""
    rp = cv.rope_params(cv.ROPE_NEOX, D, D, 1_000_000.0)
    decs = [cv.Decoder(ctx, caches[l][1], caches[l][3], N_SEQ, HQ, CAP, q[l], out[l], kv_len,
                       k_new=k_new[l], v_new=v_new[l], inputs_ready=True, rope=rp) for l in range(LAYERS)]
    stream = torch.cuda.Stream()
    graph = _graph_of(torch, stream, lambda s: [d(s) for d in decs])
    us = _time_graph(torch, stream, graph, reps) * 1000.0 / LAYERS
    del graph
    _check_status(ctx, "the RoPE decode")
    return {"decode_rope": {"what": "headline step with the Q / K RoPE fused into decode (NEOX, theta 1e6)",
                            "us_per_launch": round(us, 3), "gbs": round(bytes_per_layer / (us * 1e-6) / 1e9, 1),
                            "without_rope_us_per_launch": round(launch_us, 3)}}


def run_configs0(torch, cv, ctx, reps: int = 200) -> dict:
    """one decode layer, batch 1, 14 / 2 heads, L = 512 f16 K/V ~ N(0, 0.5),
    Q ~ N(0, 1) f32.  Latency: a graph of `reps` back-to-back launches (no overlap
    flag), so the figure is launch-to-launch time, not a streaming rate."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    L = 512
    res = {}
    for name, extra in (("default", {}), ("cuda_cores", {"cuda_cores": True})):
        kb, kd = cv.alloc_kv(cv.F16, HKV, D, L, 1)
        vb, vd = cv.alloc_kv(cv.F16, HKV, D, L, 1)
        pos = torch.arange(L, dtype=torch.int32, device="cuda")
        cv.kv_append(ctx, kd, 0.5 * torch.randn(1, L, HKV * D, device="cuda", generator=gen), pos)
        cv.kv_append(ctx, vd, 0.5 * torch.randn(1, L, HKV * D, device="cuda", generator=gen), pos)
        q = torch.randn(1, HQ, D, device="cuda", generator=gen)
        out = torch.empty_like(q)
        kl = torch.tensor([L], dtype=torch.int32, device="cuda")
        dec = cv.Decoder(ctx, kd, vd, 1, HQ, L, q, out, kl, **extra)
        stream = torch.cuda.Stream()
        graph = _graph_of(torch, stream, lambda s: [dec(s) for _ in range(reps)])
        us = _time_graph(torch, stream, graph, 5) * 1000.0 / reps
        nbytes = L * 2 * cv.row_size(cv.F16, HKV * D)
        res[name] = {"us_per_launch": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
        del graph
    _check_status(ctx, "configs[0]")
    return {"decode_configs0": {"what": "one decode layer, batch 1, L 512 f16 K/V (configs[0]); latency per launch",
                                "bytes_per_launch": 512 * 2 * cv.row_size(cv.F16, HKV * D), **res}}


def run_configs1_fixed(torch, cv, ctx, reps: int = 10) -> dict:
    """configs[1] at the fixed context lengths {256, 1024, 2048}: 64 sequences, 24 layers,
    q8_0, the same graph of fused append + decode launches as the headline."""
    peaks = measured_peaks()
    res = {}
    for L in (256, 1024, 2048):
        lens = [L] * N_SEQ
        _, caches, q, k_new, v_new, out, kv_len = build_decode_workload(torch, cv, ctx, cv.Q8_0, 0, LAYERS, lens)
        decs = [cv.Decoder(ctx, caches[l][1], caches[l][3], N_SEQ, HQ, max(L, CAP), q[l], out[l], kv_len,
                           k_new=k_new[l], v_new=v_new[l], inputs_ready=True) for l in range(LAYERS)]
        stream = torch.cuda.Stream()
        graph = _graph_of(torch, stream, lambda s: [d(s) for d in decs])
        ms = _time_graph(torch, stream, graph, reps)
        nbytes = N_SEQ * L * 2 * cv.row_size(cv.Q8_0, HKV * D) * LAYERS
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[f"L{L}"] = {"ms_per_step": round(ms, 4), "gbs": round(gbs, 1), "tok_per_s": round(N_SEQ / (ms * 1e-3), 1),
                        "frac_hbm_peak": round(gbs / peaks["hbm_gbs"], 4)}
        del graph, decs, caches, q, k_new, v_new, out
        torch.cuda.empty_cache()
    _check_status(ctx, "configs[1] fixed lengths")
    return {"decode_configs1_fixed": {"what": "24 layers x 64 sequences at one context length, q8_0 (configs[1])",
                                      "peak_gbs": peaks["hbm_gbs"], **res}}


def build_cfg4(torch, cv, ctx, kt: int, vt: int, gen, n: int = 256, L: int = 4096):
    """n sequences x L positions of (kt, vt) caches, K/V ~ N(0,1) with 1% of elements
    at +-8 sigma, appended by the engine."""
    pos = torch.arange(L, dtype=torch.int32, device="cuda")
    kb, kd = cv.alloc_kv(kt, HKV, D, L, n)
    vb, vd = cv.alloc_kv(vt, HKV, D, L, n)
    for desc in (kd, vd):
        for s0 in range(0, n, 64):  # in slices, so the f32 staging stays small
            s1 = min(n, s0 + 64)
            x = torch.randn(s1 - s0, L, HKV * D, device="cuda", generator=gen)
            hit = torch.rand(x.shape, device="cuda", generator=gen) < 0.01
            x[hit] = torch.where(torch.rand(int(hit.sum()), device="cuda", generator=gen) < 0.5, -8.0, 8.0)
            sub = cv.kv_tensor(desc._buf, desc.type, HKV, D, L, s1 - s0, byte_offset=s0 * desc.nb2)
            cv.kv_append(ctx, sub, x, pos)
            del x, hit
    q = torch.randn(n, HQ, D, device="cuda", generator=gen)
    out = torch.empty_like(q)
    kl = torch.full((n,), L, dtype=torch.int32, device="cuda")
    dec = cv.Decoder(ctx, kd, vd, n, HQ, L, q, out, kl)
    return dec, (kb, vb, kd, vd, q, out, kl)


def decode_kernel_name(n_seq: int, items: int, n_sms: int, max_pairs: int = 6) -> str:
    """The persistent decode kernel the dispatcher picks for n_seq block-quantized sequences and
    `items` 64-position items (the rule of dmma::mma_pays / launch_shape in
    csrc/decode_mma.cuh, for type pairs that fit six warp pairs per CTA)."""
    if items >= 32 * n_sms:
        return "decode_mma_kernel"
    if n_seq <= 0 or items < n_sms:
        return "decode_stream_kernel"
    per_sm = -(-items // n_sms)
    pairs = min(max_pairs, max(per_sm, 1))
    if per_sm <= 16:
        pairs = min(pairs, 4)
    grid = min(n_sms, max(-(-items // pairs), 1))
    return "decode_mma_kernel" if grid * pairs // n_seq + 1 <= 128 else "decode_stream_kernel"


def run_decode_cfg4_sharded(torch, cv, ctx, rank: int, world: int, dist, reps: int = 10) -> dict:
    """256 sequences x 4096 positions, (q8_0, q4_0) and (q5_1, q5_1), K/V with
    1% outliers at +-8 sigma, sharded by sequence over the ranks (shard_by_length;
    strong scaling, no collective).  Each rank times one decode launch over its shard;
    the step time is the max over ranks."""
    from cvattn.parallel import shard_by_length
    res = {}
    peaks = measured_peaks()
    traffic = profiled_traffic()
    n_total, L = 256, 4096
    mine = len(shard_by_length([L] * n_total, world)[rank])
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77 + rank)
    for kt, vt, name in ((cv.Q8_0, cv.Q4_0, "q8_0/q4_0"), (cv.Q5_1, cv.Q5_1, "q5_1/q5_1")):
        dec, keep = build_cfg4(torch, cv, ctx, kt, vt, gen, n=mine, L=L)
        stream = torch.cuda.Stream()
        graph = _graph_of(torch, stream, lambda s: dec(s))
        _barrier(torch, dist)
        ms_rank = _time_graph(torch, stream, graph, reps)
        ms = _sync_max(torch, dist, ms_rank)
        row_kv = cv.row_size(kt, HKV * D) + cv.row_size(vt, HKV * D)
        nbytes_total = n_total * L * row_kv
        nbytes_rank = mine * L * row_kv
        gbs = nbytes_total / (ms * 1e-3) / 1e9
        achieved = nbytes_rank / (ms_rank * 1e-3) / 1e9
        key = "decode_cfg4_" + name.replace("/", "_")
        n_sms = torch.cuda.get_device_properties(0).multi_processor_count
        kname = decode_kernel_name(mine, mine * (L // 64), n_sms)
        res[key] = {
            "what": f"decode 256 seqs x 4096, {name}, one layer, sequences sharded over {world} GPU(s)",
            "gbs": round(gbs, 1), "us_per_launch": round(ms * 1000.0, 2), "seqs_per_gpu": mine,
            "bytes_per_launch": nbytes_total, "frac_hbm_peak": round(gbs / world / peaks["hbm_gbs"], 4),
            "scaling": "strong",
            "roofline": {"bound": "hbm", "kernel": f"{kname}<{name.replace('/', ',')}>",
                         "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "algorithmic_bytes_per_launch": nbytes_rank,
                         "traffic": (traffic.get(key + "_per_launch") if world == 1 else None)}}
        del graph, dec, keep
        torch.cuda.empty_cache()
    _check_status(ctx, "the configs[3] decode")
    return res


def dit_visible_pairs(S: int = DIT_S, P: int = DIT_P, chunk: int = 50) -> int:
    bounds = list(range(chunk, S + 1, chunk))
    return S * P + sum(min(next(b for b in bounds if b > i), S) for i in range(S))


def run_dit_sharded(torch, cv, ctx, rank: int, world: int, dist, reps: int = DIT_STEPS) -> dict:
    """32 utterances x CFG 2 over 22 DiT layers, K = q8_0 / V = q4_0 cache
    (the reference's default, src/cosyvoice.cpp:187), 300 cached prompt frames and
    600 current frames with the 50-frame chunk mask; utterances sharded over the
    ranks.  One ODE step = per layer the cache append of the step's 600 K/V rows
    (update_cache) and the attention over 900 keys; the timed region is the 10
    ODE steps of the utterances, max over ranks."""
    from cvattn.parallel import shard_by_length
    peaks = measured_peaks()
    mine = len(shard_by_length([1] * DIT_UTT, world)[rank])
    B, H, P, S = 2 * mine, DIT_H, DIT_P, DIT_S
    n_kv = P + S
    gen = torch.Generator(device="cuda")
    gen.manual_seed(500 + rank)
    bounds = list(range(50, S + 1, 50))
    layers = []
    ppos = torch.arange(P, dtype=torch.int32, device="cuda")
    cpos = torch.arange(P, n_kv, dtype=torch.int32, device="cuda")
    for _ in range(DIT_LAYERS):
        kb, kd = cv.alloc_kv(cv.Q8_0, H, D, 1024, B)
        vb, vd = cv.alloc_kv(cv.Q4_0, H, D, 1024, B)
        cv.kv_append(ctx, kd, torch.randn(B, P, H * D, device="cuda", generator=gen), ppos)  # cached prompt
        cv.kv_append(ctx, vd, torch.randn(B, P, H * D, device="cuda", generator=gen), ppos)
        k = torch.randn(B, S, H * D, device="cuda", generator=gen)
        v = torch.randn(B, S, H * D, device="cuda", generator=gen)
        q = torch.randn(B, S, H, D, device="cuda", generator=gen)
        out = torch.empty_like(q)
        fp = cv.flash_params(q, kd, vd, n_kv, out, mask_mode=cv.MASK_CHUNK, chunk_bounds=bounds, chunk_key_offset=P)
        layers.append((kb, kd, vb, vd, k, v, q, out, fp))
    import ctypes

    def ode_step(s):
        sp = s.cuda_stream
        for (kb, kd, vb, vd, k, v, q, out, fp) in layers:
            cv.kv_append(ctx, kd, k, cpos, stream=sp)
            cv.kv_append(ctx, vd, v, cpos, stream=sp)
            cv.check(cv.lib.cvattn_flash(ctx.handle, sp, ctypes.byref(fp)), "dit flash")

    stream = torch.cuda.Stream()
    graph = _graph_of(torch, stream, ode_step)
    _barrier(torch, dist)
    ms_rank = _time_graph(torch, stream, graph, reps) * reps  # the 10 ODE steps
    ms = _sync_max(torch, dist, ms_rank)
    flops_total = 4.0 * D * H * (2 * DIT_UTT) * dit_visible_pairs() * DIT_LAYERS * reps
    tflops = flops_total / (ms * 1e-3) / 1e12
    del graph, layers
    torch.cuda.empty_cache()
    _check_status(ctx, "the sharded DiT")
    return {"dit_sharded": {
        "what": f"DiT attention of 32 utterances x CFG 2 x 10 ODE steps x 22 layers, q8_0/q4_0 cache with fused "
                f"append, utterances sharded over {world} GPU(s)",
        "tflops": round(tflops, 1), "ms_total": round(ms, 3), "utterances_per_gpu": mine,
        "flops": flops_total, "frac_bf16_peak": round(tflops / world / peaks["bf16_tflops"], 4),
        "peak_tflops": peaks["bf16_tflops"], "peak_source": peaks["source"], "scaling": "strong",
        "launches_per_ode_step": 3 * DIT_LAYERS}}


def run_dit_offload(torch, cv, ctx, reps: int = 10) -> dict:
    """Slot offload overlapped with the next ODE step, in the reference's schedule:
    an offloadable step on device slot 0, then a fixed-slot step on slot 1
    (dit_sched_config, src/cosyvoice-token2wav.cpp:100-167).  One DiT worker: one
    utterance, CFG batch 2, 22 layers, q8_0 / q4_0 cache object.  A step = per layer
    the append of 600 K/V rows after the 300 cached prompt rows and the chunk-masked
    attention over 900 keys.  Timed per pair of steps (CUDA events): the two steps
    alone; with slot 0 (900 positions of 22 layers) offloaded to pinned host memory
    on a copy stream while the slot-1 step computes; and the reference's order,
    offload then wait for it (src/cosyvoice-kv-cache.cpp:148-174 synchronizes), then
    the slot-1 step."""
    import ctypes
    B, H, P, S, Lyr = 2, DIT_H, DIT_P, DIT_S, DIT_LAYERS
    n_kv = P + S
    cache = cv.KVCache(ctx, Lyr, D, H, 1024, cv.Q8_0, cv.Q4_0, batch=B, n_slots=2, n_offloaded_slots=1)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(9)
    ppos = torch.arange(P, dtype=torch.int32, device="cuda")
    cpos = torch.arange(P, n_kv, dtype=torch.int32, device="cuda")
    kp = torch.randn(B, P, H * D, device="cuda", generator=gen)
    k = torch.randn(B, S, H * D, device="cuda", generator=gen)
    q = torch.randn(B, S, H, D, device="cuda", generator=gen)
    out = torch.empty_like(q)
    bounds = list(range(50, S + 1, 50))
    stream, cstream = torch.cuda.Stream(), torch.cuda.Stream()
    graphs = []
    for slot in (0, 1):
        cache.bind_slot(slot)
        cache.cur_len = 0
        for l in range(Lyr):
            cache.update(l, kp, kp, ppos)  # the cached prompt rows of this slot
        cache.shift(P)
        fps = [cv.flash_params(q, cache.tensor(l, slot, 0), cache.tensor(l, slot, 1), n_kv, out,
                               mask_mode=cv.MASK_CHUNK, chunk_bounds=bounds, chunk_key_offset=P) for l in range(Lyr)]

        def step(s, fps=fps):
            sp = s.cuda_stream
            for l in range(Lyr):
                cache.update(l, k, k, cpos, stream=sp)  # into the slot bound at capture
                cv.check(cv.lib.cvattn_flash(ctx.handle, sp, ctypes.byref(fps[l])), "dit step")

        graphs.append((_graph_of(torch, stream, step), fps))
    cache.offload_slot(0, n_kv, stream=cstream)  # allocates the pinned host slot once
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def run(mode):
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            stream.wait_stream(cstream)       # slot 0 is rewritten only after its last offload read it
            with torch.cuda.stream(stream):
                graphs[0][0].replay()           # offloadable step: device slot 0
            if mode == "overlap":
                cstream.wait_stream(stream)
                cache.offload_slot(0, n_kv, stream=cstream)
            elif mode == "serial":
                cache.offload_slot(0, n_kv, stream=stream)
                stream.synchronize()
            with torch.cuda.stream(stream):
                graphs[1][0].replay()           # fixed-slot step: device slot 1
        stream.wait_stream(cstream)
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    alone, overlap, serial = run("alone"), run("overlap"), run("serial")
    nbytes = Lyr * B * n_kv * (cv.row_size(cv.Q8_0, H * D) + cv.row_size(cv.Q4_0, H * D))
    del graphs
    cache.close()
    _check_status(ctx, "the offload overlap")
    return {"dit_offload": {
        "what": "one DiT worker (utterance x CFG 2, 22 layers, q8_0/q4_0): an offloadable step on slot 0 then a "
                "fixed-slot step; slot 0 offloaded to pinned host on a copy stream during the second step, against "
                "the two steps alone and the reference's offload-then-synchronize order",
        "slot_bytes": nbytes, "two_steps_ms": round(alone, 3), "two_steps_with_offload_overlapped_ms": round(overlap, 3),
        "offload_then_sync_ms": round(serial, 3)}}


def run_flash_secondary(torch, cv, ctx, args, only: str | None = None, reps: int = 10) -> dict:
    """DiT attention and causal prefill TFLOP/s, one launch each."""
    res = {}
    peaks = measured_peaks()
    traffic = profiled_traffic()
    if only == "prefill":
        return _prefill_part(torch, cv, ctx, peaks, res, reps)
    # --- DiT: H=16, D=64, 600 queries, 300 cached prompt + 600 current keys,
    # 50-frame chunk mask, CFG batch 2 x 32 utterances in one launch
    B, H, P, S = 64, DIT_H, DIT_P, DIT_S
    n_kv = P + S
    visible = dit_visible_pairs()
    flops = 4.0 * D * H * B * visible
    bounds = list(range(50, S + 1, 50))
    q = torch.randn(B, S, H, D, device="cuda")
    out = torch.empty_like(q)
    pos = torch.arange(n_kv, dtype=torch.int32, device="cuda")
    for kt, vt, key in ((cv.F16, cv.F16, "dit"), (cv.Q8_0, cv.Q4_0, "dit_q8_0_q4_0")):
        if only == "dit" and key != "dit":
            continue
        if only == "dit_q8_0_q4_0" and key != "dit_q8_0_q4_0":
            continue
        kb, kd = cv.alloc_kv(kt, H, D, 1024, B)
        vb, vd = cv.alloc_kv(vt, H, D, 1024, B)
        cv.kv_append(ctx, kd, torch.randn(B, n_kv, H * D, device="cuda"), pos)
        cv.kv_append(ctx, vd, torch.randn(B, n_kv, H * D, device="cuda"), pos)
        p = cv.flash_params(q, kd, vd, n_kv, out, mask_mode=cv.MASK_CHUNK, chunk_bounds=bounds, chunk_key_offset=P)
        tname = "f16" if kt == cv.F16 else "q8_0/q4_0"
        res[key] = _time_flash(torch, cv, ctx, p, flops, peaks, f"dit layer, 32 utt x CFG2 per launch, {tname} cache",
                               {"utterances": 32, "cfg": 2, "q_frames": S, "prompt_frames": P, "chunk": 50,
                                "visible_pairs_per_head": visible, "kv_type": tname},
                               reps, traffic.get(key + "_per_launch"))
        if key == "dit":
            # unmasked 600x600 peak-efficiency point
            p2 = cv.flash_params(q, kd, vd, S, out)
            res["dit_unmasked"] = _time_flash(torch, cv, ctx, p2, 4.0 * D * H * B * S * S, peaks,
                                              "dit 600x600 unmasked", {"utterances": 32, "cfg": 2, "frames": S}, reps)
        del kb, vb
        if only:
            return res
    return _prefill_part(torch, cv, ctx, peaks, res, reps)


def _prefill_part(torch, cv, ctx, peaks, res, reps) -> dict:
    # --- causal prefill S=4096, batch 8, Hq 14 / Hkv 2, f16 cache, one launch
    B2, S2 = 8, 4096
    kb2, kd2 = cv.alloc_kv(cv.F16, HKV, D, S2, B2)
    vb2, vd2 = cv.alloc_kv(cv.F16, HKV, D, S2, B2)
    pos2 = torch.arange(S2, dtype=torch.int32, device="cuda")
    cv.kv_append(ctx, kd2, torch.randn(B2, S2, HKV * D, device="cuda"), pos2)
    cv.kv_append(ctx, vd2, torch.randn(B2, S2, HKV * D, device="cuda"), pos2)
    q2 = torch.randn(B2, S2, HQ, D, device="cuda")
    out2 = torch.empty_like(q2)
    p3 = cv.flash_params(q2, kd2, vd2, S2, out2, mask_mode=cv.MASK_CAUSAL)
    res["prefill"] = _time_flash(torch, cv, ctx, p3, 4.0 * D * HQ * B2 * S2 * (S2 + 1) / 2, peaks,
                                 "causal prefill S=4096 batch 8 (one layer, one launch)",
                                 {"seq": S2, "batch": B2, "kv_type": "f16"}, reps,
                                 profiled_traffic().get("prefill_per_launch"))
    return res


def run_prefill_chunked(torch, cv, ctx, reps: int = 5) -> dict:
    """configs[2] as the reference issues it: llm_prefill takes at most n_batch = 256
    tokens per call (src/cosyvoice-llm.cpp:98-99), so a prompt of S tokens is S / 256
    calls, each appending its K/V rows to the cache (fused quantize-append) and
    attending causally to everything cached so far.  Batch 8, 14 / 2 heads, one
    layer per timed step (the 24 layers repeat it); f16 and q8_0 caches."""
    peaks = measured_peaks()
    res = {}
    B, C = 8, 256
    for S in (256, 1024, 4096):
        for kt, tname in ((cv.Q8_0, "q8_0"), (cv.F16, "f16")):
            kb, kd = cv.alloc_kv(kt, HKV, D, S, B)
            vb, vd = cv.alloc_kv(kt, HKV, D, S, B)
            kx = torch.randn(B, S, HKV * D, device="cuda")
            vx = torch.randn(B, S, HKV * D, device="cuda")
            q = torch.randn(B, S, HQ, D, device="cuda")
            calls = []
            for c in range(S // C):
                pos = torch.arange(c * C, (c + 1) * C, dtype=torch.int32, device="cuda")
                kc, vc = kx[:, c * C:(c + 1) * C].contiguous(), vx[:, c * C:(c + 1) * C].contiguous()
                oc = torch.empty(B, C, HQ, D, device="cuda")   # each call's output [batch][256][Hq][D]
                fp = cv.flash_params(q[:, c * C:(c + 1) * C], kd, vd, (c + 1) * C, oc, mask_mode=cv.MASK_CAUSAL)
                calls.append((pos, kc, vc, fp, oc))
            import ctypes

            def layer(s, calls=calls, kd=kd, vd=vd):
                sp = s.cuda_stream
                for pos, kc, vc, fp, _ in calls:
                    cv.kv_append(ctx, kd, kc, pos, stream=sp)
                    cv.kv_append(ctx, vd, vc, pos, stream=sp)
                    cv.check(cv.lib.cvattn_flash(ctx.handle, sp, ctypes.byref(fp)), "prefill call")

            stream = torch.cuda.Stream()
            graph = _graph_of(torch, stream, layer)
            ms = _time_graph(torch, stream, graph, reps)
            flops = 4.0 * D * HQ * B * S * (S + 1) / 2
            tf = flops / (ms * 1e-3) / 1e12
            res[f"S{S}_{tname}"] = {"us_per_layer": round(ms * 1000.0, 2), "tflops": round(tf, 1),
                                    "frac_bf16_peak": round(tf / peaks["bf16_tflops"], 4), "calls": S // C}
            del graph, calls, kb, vb, kx, vx, q
    torch.cuda.empty_cache()
    _check_status(ctx, "the chunked prefill")
    return {"prefill_chunked": {"what": "causal prefill as 256-token calls with the fused KV append, batch 8, "
                                       "one layer (configs[2]); flops = causal pairs only",
                                "peak_tflops": peaks["bf16_tflops"], "peak_source": peaks["source"], **res}}


def _time_flash(torch, cv, ctx, params, flops, peaks, what, cfg, reps: int = 10, traffic=None) -> dict:
    import ctypes
    stream = torch.cuda.Stream()

    def launch(s):
        cv.check(cv.lib.cvattn_flash(ctx.handle, s.cuda_stream, ctypes.byref(params)), what)

    graph = _graph_of(torch, stream, lambda s: [launch(s) for _ in range(reps)])
    us = _time_graph(torch, stream, graph, 1, warm=1) * 1000.0 / reps
    del graph
    tflops = flops / (us * 1e-6) / 1e12
    return {"what": what, "tflops": round(tflops, 1), "us_per_launch": round(us, 2), "flops_per_launch": flops,
            "frac_bf16_peak": round(tflops / peaks["bf16_tflops"], 4), "peak_tflops": peaks["bf16_tflops"],
            "peak_source": peaks["source"], "config": cfg,
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4), "traffic": traffic}}


# ------------------------------------------------------------ reference arm

def _reference_sample():
    """All 64 sequences of the mix, one layer, q8_0 rows quantized by the oracle."""
    from oracle import oracle as O
    O.build()
    lens = seq_lengths()
    rng = np.random.default_rng(7)
    k_rows = [O.quantize(O.Q8_0, rng.standard_normal((L, HKV * D)).astype(np.float32)) for L in lens]
    v_rows = [O.quantize(O.Q8_0, rng.standard_normal((L, HKV * D)).astype(np.float32)) for L in lens]
    q = rng.standard_normal((N_SEQ, 1, HQ, D)).astype(np.float32)
    kl = np.array(lens, np.int32)
    sample_bytes = int(kl.sum()) * 2 * O.row_bytes(O.Q8_0, HKV * D)
    threads = os.cpu_count() or 1

    def run():
        O.flash_cpu(q, k_rows, v_rows, O.Q8_0, O.Q8_0, HKV, kl, False, 0.125, n_threads=threads)
    return run, sample_bytes, threads


SAMPLE_DESC = ("all 64 sequences of the mix (70,843 keys), one of the 24 layers, per sample; "
               "ggml-CPU-style restatement oracle/cvattn_oracle.c (ggml itself is unavailable)")


def run_reference(args) -> dict:
    """The reference's CPU flash_attn_ext path (oracle restatement), all host threads."""
    run, sample_bytes, threads = _reference_sample()
    for _ in range(max(1, args.warmup)):
        run()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    gbs = sample_bytes / sec / 1e9
    step_s = sample_bytes * LAYERS / (gbs * 1e9)
    return {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": headline_config(1),
        "timing": "each step times one of the 24 layers (all 64 sequences) on the host cores; ms_per_step is that "
                  "layer time x 24, the same bytes per step as the GPU arm",
        "tok_per_s": round(N_SEQ / step_s, 3),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": SAMPLE_DESC},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def cpu_baseline_for_line(budget_s: float = 10.0) -> dict:
    """The oracle's CPU path timed for about budget_s on the host cores (rank 0, N=1)."""
    run, sample_bytes, threads = _reference_sample()
    run()
    times, t_end = [], time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    gbs = sample_bytes / statistics.median(times) / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{len(times)} samples of {SAMPLE_DESC}"}


def run_cpu_baselines(budget_s: float = 4.0) -> dict:
    """The oracle's ggml-CPU-style flash attention (the reference's CPU path restated;
    ggml itself is unavailable) on bounded samples of every config, all host threads.
    Prints reported baselines; nothing here is a GPU figure."""
    from oracle import oracle as O
    O.build()
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(3)

    def timed(fn) -> float:
        fn()
        times, t_end = [], time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 2:
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        return statistics.median(times)

    res = {"kind": "port", "cores": threads, "impl": "oracle/cvattn_oracle.c oracle_flash_cpu (ggml-CPU-style, f32)"}
    # batch 1, L 512, f16 K/V ~ N(0, 0.5)
    L = 512
    k0 = O.quantize(O.F16, 0.5 * rng.standard_normal((L, HKV * D)).astype(np.float32))
    v0 = O.quantize(O.F16, 0.5 * rng.standard_normal((L, HKV * D)).astype(np.float32))
    q0 = rng.standard_normal((1, 1, HQ, D)).astype(np.float32)
    t = timed(lambda: O.flash_cpu(q0, [k0], [v0], O.F16, O.F16, HKV, np.array([L], np.int32), False, 0.125, threads))
    res["configs0"] = {"us_per_layer": round(t * 1e6, 1), "gbs": round(L * 2 * 256 / t / 1e9, 3)}
    # the 64-sequence mix, one layer
    run, sample_bytes, _ = _reference_sample()
    t = timed(run)
    res["configs1_mix"] = {"ms_per_layer": round(t * 1e3, 2), "gbs": round(sample_bytes / t / 1e9, 3)}
    # causal prefill, batch 8, f16 cache, one layer (S = 256 and 1024)
    for S in (256, 1024):
        kk = [O.quantize(O.F16, rng.standard_normal((S, HKV * D)).astype(np.float32)) for _ in range(8)]
        vv = [O.quantize(O.F16, rng.standard_normal((S, HKV * D)).astype(np.float32)) for _ in range(8)]
        qq = rng.standard_normal((8, S, HQ, D)).astype(np.float32)
        t = timed(lambda: O.flash_cpu(qq, kk, vv, O.F16, O.F16, HKV, np.full(8, S, np.int32), True, 0.125, threads))
        res[f"configs2_S{S}"] = {"ms_per_layer": round(t * 1e3, 2),
                                 "tflops": round(4.0 * D * HQ * 8 * S * (S + 1) / 2 / t / 1e12, 4)}
    # 16 of the 256 sequences x 4096, q8_0 / q4_0 with 1% +-8 sigma outliers
    n3, L3 = 16, 4096
    def outl(shape):
        x = rng.standard_normal(shape).astype(np.float32)
        hit = rng.random(shape) < 0.01
        x[hit] = np.where(rng.random(int(hit.sum())) < 0.5, -8.0, 8.0)
        return x
    kk = [O.quantize(O.Q8_0, outl((L3, HKV * D))) for _ in range(n3)]
    vv = [O.quantize(O.Q4_0, outl((L3, HKV * D))) for _ in range(n3)]
    qq = rng.standard_normal((n3, 1, HQ, D)).astype(np.float32)
    t = timed(lambda: O.flash_cpu(qq, kk, vv, O.Q8_0, O.Q4_0, HKV, np.full(n3, L3, np.int32), False, 0.125, threads))
    res["configs3_q8_0_q4_0"] = {"sample": "16 of 256 sequences, one layer", "ms": round(t * 1e3, 2),
                                 "gbs": round(n3 * L3 * (136 + 72) / t / 1e9, 3)}
    # one utterance (CFG batch 2), 16 heads, 600 queries over 900 keys, q8_0 / q4_0, one layer
    # (the CPU restatement has no chunk mask: it runs every pair, and the rate counts every pair)
    H, S4, K4 = 16, 600, 900
    kk = [O.quantize(O.Q8_0, rng.standard_normal((K4, H * D)).astype(np.float32)) for _ in range(2)]
    vv = [O.quantize(O.Q4_0, rng.standard_normal((K4, H * D)).astype(np.float32)) for _ in range(2)]
    qq = rng.standard_normal((2, S4, H, D)).astype(np.float32)
    t = timed(lambda: O.flash_cpu(qq, kk, vv, O.Q8_0, O.Q4_0, H, np.full(2, K4, np.int32), False, 0.125, threads))
    res["configs4_one_utterance_layer"] = {"ms": round(t * 1e3, 2),
                                           "tflops": round(4.0 * D * H * 2 * S4 * K4 / t / 1e12, 4)}
    return res


def run_profile(args, torch) -> None:
    """Launch one kernel of the benchmark workload args.steps times, untimed."""
    import cvattn as cv
    ctx = cv.Context(torch.cuda.current_device())
    if args.profile == "decode":
        # the headline layer shape: one layer's caches, 64 sequences
        lens, caches, q, k_new, v_new, out, kv_len = build_decode_workload_layers(torch, cv, ctx, 1)
        dec = cv.Decoder(ctx, caches[0][1], caches[0][3], N_SEQ, HQ, CAP, q[0], out[0], kv_len,
                         k_new=k_new[0], v_new=v_new[0])
        for _ in range(args.steps):
            dec()
    elif args.profile in ("decode_cfg4", "decode_cfg4_q5_1"):
        # 256 x 4096, q8_0 K / q4_0 V (218 MB) or q5_1 / q5_1 (201 MB)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(77)
        kt, vt = (cv.Q8_0, cv.Q4_0) if args.profile == "decode_cfg4" else (cv.Q5_1, cv.Q5_1)
        dec, keep = build_cfg4(torch, cv, ctx, kt, vt, gen)
        for _ in range(args.steps):
            dec()
    elif args.profile == "dit_append":
        # the DiT step's cache append: 600 rows of 64 batch entries x 1024 f32 into q8_0 K / q4_0 V
        B, H, P, S = 64, DIT_H, DIT_P, DIT_S
        kb, kd = cv.alloc_kv(cv.Q8_0, H, D, 1024, B)
        vb, vd = cv.alloc_kv(cv.Q4_0, H, D, 1024, B)
        k = torch.randn(B, S, H * D, device="cuda")
        v = torch.randn(B, S, H * D, device="cuda")
        pos = torch.arange(P, P + S, dtype=torch.int32, device="cuda")
        for _ in range(args.steps):
            cv.kv_append(ctx, kd, k, pos)
            cv.kv_append(ctx, vd, v, pos)
    elif args.profile == "dit_append_timed":
        # the same append per cache type, timed (no ncu): CUDA events around 20 back-to-back
        # launches after 3 warm-ups; TB/s counts the f32 rows read and the cache rows written
        B, H, P, S = 64, DIT_H, DIT_P, DIT_S
        src = torch.randn(B, S, H * D, device="cuda")
        pos = torch.arange(P, P + S, dtype=torch.int32, device="cuda")
        res = {}
        for name in ("q8_0", "q4_0", "q5_1", "f16"):
            t = cv.TYPE_BY_NAME[name]
            buf, desc = cv.alloc_kv(t, H, D, 1024, B)  # buf holds the cache's memory
            for _ in range(3):
                cv.kv_append(ctx, desc, src, pos)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                cv.kv_append(ctx, desc, src, pos)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / 20
            nbytes = B * S * H * D * 4 + B * S * cv.row_size(t, H * D)
            res[name] = {"us": round(us, 1), "tbs": round(nbytes / us / 1e6, 2)}
            del buf, desc
        print(json.dumps({"dit_append": res}), flush=True)
    else:
        run_flash_secondary(torch, cv, ctx, args, only=args.profile, reps=args.steps)
    torch.cuda.synchronize()
    _check_status(ctx, "the profiled launches")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-secondary", action="store_true", help="headline only: skip every secondary line")
    ap.add_argument("--cpu-baselines", action="store_true",
                    help="time the oracle's CPU restatement on bounded samples of every config and print them")
    ap.add_argument("--profile", choices=["decode", "decode_cfg4", "decode_cfg4_q5_1", "dit", "dit_q8_0_q4_0",
                                          "prefill", "dit_append", "dit_append_timed"], default=None,
                    help="only launch the named kernel a few times (for an ncu capture; prints nothing), "
                         "or time the DiT append per cache type (dit_append_timed)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))

    if args.cpu_baselines:
        if rank == 0:
            print(json.dumps(run_cpu_baselines()), flush=True)
        return
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    import torch
    dist = None
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    if args.profile:
        run_profile(args, torch)
        return
    res = run_ours(args, rank, world, torch, dist)
    if rank == 0:
        if world == 1:
            res["cpu_baseline"] = cpu_baseline_for_line()
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
