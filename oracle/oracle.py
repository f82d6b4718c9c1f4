"""ctypes wrapper over oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA engine.  Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline / ``--impl reference``
legs import it.  Nothing under cosyvoice.cpp_b200/ imports it, and the engine
has no CPU fallback that could route through it.

Function-by-function it follows oracle/cvattn_oracle.c, whose header lists the
reference lines each routine restates (gguf-py quants.py for the KV block
codecs, src/cosyvoice-kv-cache.cpp:383 / src/cosyvoice-graph.cpp:375 for the
flash-attention semantics, src/cosyvoice-llm.cpp:20-29 and
src/cosyvoice-token2wav.cpp:100-167,285-298 for masks and the DiT step plan).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

# ggml type ids (ggml.h enum ggml_type) for the KV cache types.
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
KV_TYPES = (F32, F16, Q8_0, Q5_1, Q5_0, Q4_1, Q4_0)
TYPE_NAMES = {F32: "f32", F16: "f16", Q4_0: "q4_0", Q4_1: "q4_1", Q5_0: "q5_0", Q5_1: "q5_1", Q8_0: "q8_0"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), Q8_0: (32, 34)}

_lib = None


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(HERE, "cvattn_oracle.c")
    ):
        subprocess.run(["make", "-s", "-C", HERE, "-B", "liboracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        c = ctypes
        L.oracle_f32_to_f16.restype = c.c_uint16
        L.oracle_f32_to_f16.argtypes = [c.c_float]
        L.oracle_f16_to_f32.restype = c.c_float
        L.oracle_f16_to_f32.argtypes = [c.c_uint16]
        L.oracle_row_bytes.restype = c.c_int64
        L.oracle_row_bytes.argtypes = [c.c_int, c.c_int64]
        for fn in (L.oracle_quantize_rows, L.oracle_dequantize_rows):
            fn.restype = c.c_int
            fn.argtypes = [c.c_int, c.c_void_p, c.c_int64, c.c_int64, c.c_void_p]
        L.oracle_causal_mask.argtypes = [c.c_void_p, c.c_int32, c.c_int32]
        L.oracle_chunk_mask.argtypes = [c.c_void_p, c.c_int32, c.c_void_p, c.c_int32]
        L.oracle_attention_f64.argtypes = [
            c.c_void_p, c.c_int32, c.c_int32, c.c_int32,
            c.c_void_p, c.c_void_p, c.c_int32, c.c_int32,
            c.c_void_p, c.c_int64, c.c_double, c.c_void_p,
        ]
        L.oracle_flash_cpu.argtypes = [
            c.c_void_p, c.c_int32, c.c_int32, c.c_int32, c.c_int32, c.c_int32,
            c.c_int32, c.c_void_p, c.c_int64,
            c.c_int32, c.c_void_p, c.c_int64,
            c.c_void_p, c.c_int32, c.c_float, c.c_void_p, c.c_int32,
        ]
        L.oracle_rope.argtypes = [c.c_void_p, c.c_void_p, c.c_void_p, c.c_int32, c.c_int32, c.c_int32,
                                  c.c_int32, c.c_int32, c.c_float, c.c_float, c.c_float]
        L.oracle_max_threads.restype = c.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def row_bytes(t: int, n: int) -> int:
    be, bb = BLOCK[t]
    return n // be * bb


def quantize(t: int, x: np.ndarray) -> np.ndarray:
    """Rows of f32 [..., n] -> uint8 [..., row_bytes(t, n)] (ggml block layout)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    rows = x.size // n
    out = np.empty(x.shape[:-1] + (row_bytes(t, n),), dtype=np.uint8)
    if lib().oracle_quantize_rows(t, _ptr(x), rows, n, _ptr(out)):
        raise ValueError("quantize failed")
    return out


def dequantize(t: int, q: np.ndarray, n: int) -> np.ndarray:
    """uint8 [..., row_bytes(t, n)] -> f32 [..., n]."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rb = row_bytes(t, n)
    rows = q.size // rb
    out = np.empty(q.shape[:-1] + (n,), dtype=np.float32)
    if lib().oracle_dequantize_rows(t, _ptr(q), rows, n, _ptr(out)):
        raise ValueError("dequantize failed")
    return out


ROPE_NORMAL, ROPE_NEOX = 0, 2


def rope(x: np.ndarray, pos: np.ndarray, unit_len: int, n_dims: int, mode: int, freq_base: float,
         freq_scale: float = 1.0, attn_factor: float = 1.0) -> np.ndarray:
    """ggml_rope_ext (ext_factor 0) on rows x[..., row_len] at positions pos[rows]
    (src/cosyvoice-llm.cpp:56-57,180; src/cosyvoice-graph.cpp:354-355)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    row_len = x.shape[-1]
    rows = x.size // row_len
    p = np.ascontiguousarray(pos, dtype=np.int32).reshape(-1)
    assert p.size == rows and row_len % unit_len == 0 and n_dims % 2 == 0 and n_dims <= unit_len
    out = np.empty_like(x)
    lib().oracle_rope(_ptr(x), _ptr(out), _ptr(p), rows, row_len, unit_len, n_dims, mode,
                      float(freq_base), float(freq_scale), float(attn_factor))
    return out


def f32_to_f16_bits(x: float) -> int:
    return int(lib().oracle_f32_to_f16(float(x)))


def causal_mask(n_batch: int, seq_len: int) -> np.ndarray:
    """f16 bits [n_batch, seq_len] (src/cosyvoice-llm.cpp:20-29)."""
    m = np.empty((n_batch, seq_len), dtype=np.uint16)
    lib().oracle_causal_mask(_ptr(m), n_batch, seq_len)
    return m


def chunk_mask(n: int, bounds: Sequence[int]) -> np.ndarray:
    """f16 bits [n, n] (src/cosyvoice-token2wav.cpp:285-298)."""
    b = np.ascontiguousarray(np.asarray(bounds, dtype=np.int32))
    m = np.empty((n, n), dtype=np.uint16)
    lib().oracle_chunk_mask(_ptr(m), n, _ptr(b) if b.size else None, int(b.size))
    return m


def mask_bits_to_f32(m: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(m.astype(np.uint16).view(np.float16).astype(np.float32))


def attention_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
                  mask: np.ndarray | None = None) -> np.ndarray:
    """fp64 attention for one batch entry.

    q [n_q, Hq, D] f32, k/v [n_kv, Hkv, D] f32 (dequantized rows),
    mask [n_q, >=n_kv] f32 additive or None.  Returns [n_q, Hq, D] f32.
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    n_q, Hq, D = q.shape
    n_kv, Hkv, _ = k.shape
    out = np.empty_like(q)
    mptr, mstride = None, 0
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
        mptr, mstride = _ptr(mask), mask.shape[1]
    lib().oracle_attention_f64(_ptr(q), n_q, Hq, D, _ptr(k), _ptr(v), n_kv, Hkv, mptr, mstride,
                               float(scale), _ptr(out))
    return out


def flash_cpu(q: np.ndarray, k_rows: Sequence[np.ndarray], v_rows: Sequence[np.ndarray],
              k_type: int, v_type: int, Hkv: int, kv_len: np.ndarray, causal: bool,
              scale: float, n_threads: int = 0) -> np.ndarray:
    """ggml-CPU-style fp32 flash attention over typed cache rows (timed baseline).

    q [n_seq, n_q, Hq, D] f32; k_rows[s] / v_rows[s] uint8 [>= kv_len[s], row_bytes].
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    n_seq, n_q, Hq, D = q.shape
    kp = (ctypes.c_void_p * n_seq)(*[_ptr(a) for a in k_rows])
    vp = (ctypes.c_void_p * n_seq)(*[_ptr(a) for a in v_rows])
    kl = np.ascontiguousarray(kv_len, dtype=np.int32)
    out = np.empty_like(q)
    lib().oracle_flash_cpu(_ptr(q), n_seq, n_q, Hq, Hkv, D,
                           k_type, kp, row_bytes(k_type, Hkv * D),
                           v_type, vp, row_bytes(v_type, Hkv * D),
                           _ptr(kl), 1 if causal else 0, float(scale), _ptr(out), int(n_threads))
    return out


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def dit_sched_plan(n: int, n_offloadable: int, n_fixed: int, cut_len: int, offset: int,
                   streaming: bool, kv_slidable: bool) -> list[dict]:
    """Per-step DiT plan, restating dit_sched_config (src/cosyvoice-token2wav.cpp:100-167)."""
    keys = ("rebuild", "cache_kv", "load", "offload", "slide", "slice", "mask", "cut_len")
    plan = [dict.fromkeys(keys, False) for _ in range(n)]
    for p in plan:
        p["cut_len"] = 0
    if not streaming:
        plan[0]["rebuild"] = True
        plan[1]["rebuild"] = True
        plan[n - 1]["rebuild"] = True
        plan[n - 1]["cut_len"] = cut_len
        return plan
    if offset != 0:
        cut_len = 0
    n_no_cache = n - n_offloadable - n_fixed
    for i in range(n):
        p = plan[i]
        p["rebuild"] = (i <= 1 or (offset != 0 and i == n_no_cache - 1) or i == n_no_cache
                        or (i == n - 1 and cut_len != 0) or (not kv_slidable and i >= n_no_cache))
        p["cache_kv"] = i >= n_no_cache
        p["offload"] = n_no_cache <= i < n_no_cache + n_offloadable
        p["load"] = p["offload"] and offset != 0
        p["mask"] = i < n_no_cache and offset != 0
        p["cut_len"] = cut_len if (i == n - 1 and offset == 0) else 0
        if i == n_no_cache - 1 and offset != 0:
            p["cut_len"] = offset
        p["slice"] = offset != 0 and i == n_no_cache
        p["slide"] = (kv_slidable and p["cache_kv"]
                      and (not p["offload"] or i == n_no_cache + n_offloadable - 1) and i != n - 1)
    return plan
