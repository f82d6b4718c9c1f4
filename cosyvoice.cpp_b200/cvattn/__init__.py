"""Python host mirror of the cvattn C ABI (include/cvattn.h).

Mirrors the reference's attention seam for tests and benchmarks: the KV cache
object follows class cosyvoice_kv_cache (src/cosyvoice-kv-cache.h:10-69), the
free functions follow the ggml ops it builds (set_rows for the append,
flash_attn_ext for attention).  PyTorch tensors only carry device memory and
streams; every computation runs in libcvattn.so's CUDA kernels.  There is no
CPU path: without the library, importing this package fails.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

from . import _lib
from ._lib import DecodeParams, DitStep, FlashParams, KVCacheParams, RopeParams, Tensor, load

# ggml type ids
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
KV_TYPES = (F32, F16, Q8_0, Q5_1, Q5_0, Q4_1, Q4_0)
TYPE_NAMES = {F32: "f32", F16: "f16", Q4_0: "q4_0", Q4_1: "q4_1", Q5_0: "q5_0", Q5_1: "q5_1", Q8_0: "q8_0"}
TYPE_BY_NAME = {v: k for k, v in TYPE_NAMES.items()}

# cosyvoice_kv_cache_type_t (include/cosyvoice.h:32-42)
CV_F32, CV_F16, CV_Q8_0, CV_Q5_1, CV_Q5_0, CV_Q4_1, CV_Q4_0 = range(7)

MASK_NONE, MASK_EXPLICIT, MASK_CAUSAL, MASK_CHUNK = 0, 1, 2, 3
DECODE_EMIT_PARTIAL = 1
DECODE_CUDA_CORES = 2
DECODE_NOT_PERSISTENT = 4
DECODE_INPUTS_READY = 8
DECODE_WIDE_CHUNKS = 16
DECODE_TMEM_STREAM = 32
DECODE_WARP_MMA = 64
FLASH_ONE_TILE = 1
FLASH_SPLIT_COLUMNS = 2
FLASH_WHOLE_ROWS = 4
ROPE_NORMAL, ROPE_NEOX = 0, 2

OK = 0
STATUS_NAMES = {0: "OK", 1: "INVALID_ARGUMENT", 2: "UNSUPPORTED", 3: "LENGTH", 4: "ALLOC", 5: "CUDA",
                6: "DEVICE", 7: "NO_DEVICE", 8: "TIMEOUT"}

lib = load()


class CvattnError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = lib.cvattn_status_string(status).decode()
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)} ({msg})" if what else msg)


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise CvattnError(status, what)


def make_separate_kv_cache(k: int, v: int, fallback: int) -> int:
    """COSYVOICE_MAKE_SEPARATE_KV_CACHE (include/cosyvoice.h:205-206)."""
    return (k | (v << 5) | (fallback << 10) | (1 << 31)) & 0xFFFFFFFF


def row_size(t: int, n: int) -> int:
    return int(lib.cvattn_row_size(t, n))


def supports(k_type: int, v_type: int, head_dim: int, n_q_heads: int, n_kv_heads: int) -> bool:
    return bool(lib.cvattn_supports(k_type, v_type, head_dim, n_q_heads, n_kv_heads))


def negotiate_kv_types(kv_type_union: int, kv_fallback: bool, head_dim: int, n_q_heads: int, n_kv_heads: int):
    """Returns (status, k_type, v_type, resolved_union, fattn)."""
    k, v, u, fa = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_uint32(), ctypes.c_int32()
    st = lib.cvattn_negotiate_kv_types(kv_type_union & 0xFFFFFFFF, int(kv_fallback), head_dim, n_q_heads,
                                       n_kv_heads, ctypes.byref(k), ctypes.byref(v), ctypes.byref(u),
                                       ctypes.byref(fa))
    return st, k.value, v.value, u.value, fa.value


def dit_sched_plan(n_steps: int, n_offloadable: int, n_fixed: int, cut_len: int, offset: int,
                   streaming: bool, kv_slidable: bool) -> list[dict]:
    steps = (DitStep * n_steps)()
    check(lib.cvattn_dit_sched_plan(n_steps, n_offloadable, n_fixed, cut_len, offset, int(streaming),
                                    int(kv_slidable), steps), "dit_sched_plan")
    keys = ("rebuild", "cache_kv", "load", "offload", "slide", "slice", "mask")
    return [{**{k: bool(getattr(s, k)) for k in keys}, "cut_len": int(s.cut_len)} for s in steps]


# ---------------------------------------------------------------- device side

def _torch():
    import torch
    return torch


def _stream(stream) -> int:
    torch = _torch()
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


class Context:
    """One per worker thread: device status word (cvattn_context)."""

    def __init__(self, device: int = 0):
        self.handle = ctypes.c_void_p()
        check(lib.cvattn_context_create(device, ctypes.byref(self.handle)), "context_create")
        self.device = device

    def sync_status(self, stream=None) -> tuple[int, int]:
        detail = ctypes.c_int32(0)
        st = lib.cvattn_context_sync_status(self.handle, _stream(stream), ctypes.byref(detail))
        return st, detail.value

    def close(self) -> None:
        if self.handle:
            lib.cvattn_context_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def kv_tensor(buf, type_: int, n_heads: int, head_dim: int, ne1: int, ne2: int = 1,
              nb1: int | None = None, nb2: int | None = None, byte_offset: int = 0) -> Tensor:
    """Describe a ggml KV tensor living in a torch byte buffer (or any CUDA tensor)."""
    rb = row_size(type_, n_heads * head_dim)
    nb1 = rb if nb1 is None else nb1
    nb2 = nb1 * ne1 if nb2 is None else nb2
    t = Tensor()
    t.data = buf.data_ptr() + byte_offset
    t.type, t.n_heads, t.head_dim, t.reserved = type_, n_heads, head_dim, 0
    t.ne1, t.ne2, t.nb1, t.nb2 = ne1, ne2, nb1, nb2
    t._buf = buf  # the descriptor keeps its device memory alive
    return t


def alloc_kv(type_: int, n_heads: int, head_dim: int, ne1: int, ne2: int = 1, device="cuda"):
    """Allocate a zeroed ggml-layout KV tensor; returns (byte buffer, descriptor)."""
    torch = _torch()
    rb = row_size(type_, n_heads * head_dim)
    buf = torch.zeros(ne2 * ne1 * rb, dtype=torch.uint8, device=device)
    return buf, kv_tensor(buf, type_, n_heads, head_dim, ne1, ne2)


def rope_params(mode: int, n_dims: int, unit_len: int, freq_base: float, freq_scale: float = 1.0,
                attn_factor: float = 1.0) -> RopeParams:
    """A ggml_rope_ext description (ext_factor 0): NEOX per head for the LLM
    (src/cosyvoice-llm.cpp:56-57), NORMAL on the row prefix for the DiT
    (src/cosyvoice-graph.cpp:354-355)."""
    return RopeParams(mode, n_dims, unit_len, freq_base, freq_scale, attn_factor)


def rope(x, pos, rp: RopeParams, out=None, stream=None):
    """RoPE of f32 rows x [..., row_len] (contiguous) at positions pos (int32, one per row)."""
    torch = _torch()
    assert x.dtype == torch.float32 and x.is_contiguous()
    row_len = x.shape[-1]
    n_rows = x.numel() // row_len
    if out is None:
        out = torch.empty_like(x)
    check(lib.cvattn_rope(_stream(stream), ctypes.byref(rp), x.data_ptr(), row_len * 4, out.data_ptr(), row_len * 4,
                          pos.data_ptr(), n_rows, row_len), "rope")
    return out


def kv_append(ctx: Context, cache: Tensor, src, pos, stream=None, rope: RopeParams | None = None) -> None:
    """ggml_set_rows into the cache: src f32 [batch, n_new, row] contiguous,
    pos int32 [n_new] (shared) or [batch, n_new] on the device.  With rope the
    rows turn by their positions first (the key RoPE fused with the append)."""
    torch = _torch()
    assert src.dtype == torch.float32 and src.is_contiguous() and src.dim() == 3
    batch, n_new, row = src.shape
    pos_nb1 = 0 if pos.dim() == 1 else pos.stride(0) * 4
    if rope is None:
        check(lib.cvattn_kv_append(ctx.handle, _stream(stream), ctypes.byref(cache), src.data_ptr(), row * 4,
                                   n_new * row * 4, pos.data_ptr(), pos_nb1, n_new, batch), "kv_append")
    else:
        check(lib.cvattn_kv_append_rope(ctx.handle, _stream(stream), ctypes.byref(cache), src.data_ptr(), row * 4,
                                        n_new * row * 4, pos.data_ptr(), pos_nb1, n_new, batch, ctypes.byref(rope)),
              "kv_append_rope")


def kv_dequantize(ctx: Context, cache: Tensor, n_rows: int, stream=None):
    torch = _torch()
    out = torch.empty((cache.ne2, n_rows, cache.n_heads * cache.head_dim), dtype=torch.float32, device="cuda")
    check(lib.cvattn_kv_dequantize(ctx.handle, _stream(stream), ctypes.byref(cache), n_rows, out.data_ptr()),
          "kv_dequantize")
    return out


def decode_workspace_size(k_type, v_type, n_seq, max_kv_len, n_q_heads, n_kv_heads, head_dim=64) -> int:
    return int(lib.cvattn_decode_workspace_size(k_type, v_type, n_seq, max_kv_len, n_q_heads, n_kv_heads, head_dim))


def alloc_workspace(nbytes: int, stream=None):
    torch = _torch()
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device="cuda")
    check(lib.cvattn_workspace_init(_stream(stream), ws.data_ptr(), ws.numel()), "workspace_init")
    return ws


class Decoder:
    """Reusable decode launcher (pre-built params, one workspace): the batched
    llm_decode attention call of src/cosyvoice-llm.cpp:62 across sequences."""

    def __init__(self, ctx: Context, k: Tensor, v: Tensor, n_seq: int, n_q_heads: int, max_kv_len: int,
                 q, out, kv_len, k_new=None, v_new=None, k_seq_ptrs=None, v_seq_ptrs=None,
                 scale: float | None = None, emit_partial: bool = False, partial_ml=None, workspace=None,
                 cuda_cores: bool = False, not_persistent: bool = False, inputs_ready: bool = False,
                 wide_chunks: bool = False, tmem_stream: bool = False, warp_mma: bool = False,
                 rope: RopeParams | None = None):
        self.ctx = ctx
        self.rope = rope
        p = DecodeParams()
        p.q, p.q_seq_stride = q.data_ptr(), q.stride(0)
        p.out, p.out_seq_stride = out.data_ptr(), out.stride(0)
        p.k, p.v = k, v
        p.k_seq_ptrs, p.v_seq_ptrs = _ptr(k_seq_ptrs), _ptr(v_seq_ptrs)
        p.kv_len = kv_len.data_ptr()
        p.k_new, p.v_new = _ptr(k_new), _ptr(v_new)
        p.partial_ml = _ptr(partial_ml)
        p.n_seq, p.n_q_heads, p.max_kv_len = n_seq, n_q_heads, max_kv_len
        p.flags = ((DECODE_EMIT_PARTIAL if emit_partial else 0) | (DECODE_CUDA_CORES if cuda_cores else 0)
                   | (DECODE_NOT_PERSISTENT if not_persistent else 0) | (DECODE_INPUTS_READY if inputs_ready else 0)
                   | (DECODE_WIDE_CHUNKS if wide_chunks else 0) | (DECODE_TMEM_STREAM if tmem_stream else 0)
                   | (DECODE_WARP_MMA if warp_mma else 0))
        p.scale = 1.0 / math.sqrt(k.head_dim) if scale is None else scale
        need = decode_workspace_size(k.type, v.type, n_seq, max_kv_len, n_q_heads, k.n_heads, k.head_dim)
        if workspace is None:
            workspace = alloc_workspace(need)
        self.workspace = workspace
        p.workspace, p.workspace_size = workspace.data_ptr(), workspace.numel()
        self.params = p
        self._keep = (q, out, kv_len, k_new, v_new, k_seq_ptrs, v_seq_ptrs, partial_ml)

    def __call__(self, stream=None) -> None:
        if self.rope is None:
            check(lib.cvattn_decode(self.ctx.handle, _stream(stream), ctypes.byref(self.params)), "decode")
        else:
            check(lib.cvattn_decode_rope(self.ctx.handle, _stream(stream), ctypes.byref(self.params),
                                         ctypes.byref(self.rope)), "decode_rope")


def decode(ctx: Context, q, k: Tensor, v: Tensor, kv_len, max_kv_len: int, out=None, **kw):
    """One decode step for q f32 [n_seq, Hq, D]; returns out [n_seq, Hq, D]."""
    torch = _torch()
    n_seq, Hq, D = q.shape
    if out is None:
        out = torch.empty_like(q)
    Decoder(ctx, k, v, n_seq, Hq, max_kv_len, q, out, kv_len, **kw)(kw.get("stream"))
    return out


def combine(partial_o, partial_ml, out=None, stream=None):
    """LSE combine: partial_o [P, R, D], partial_ml [P, R, 2] -> out [R, D]."""
    torch = _torch()
    P, R, D = partial_o.shape
    if out is None:
        out = torch.empty((R, D), dtype=torch.float32, device=partial_o.device)
    check(lib.cvattn_combine(_stream(stream), partial_o.data_ptr(), partial_ml.data_ptr(), P, R, D,
                             out.data_ptr()), "combine")
    return out


def flash_params(q, k: Tensor, v: Tensor, n_kv: int, out, mask_mode: int = MASK_NONE, mask=None,
                 causal_offset: int | None = None, chunk_bounds: Sequence[int] = (), chunk_key_offset: int = 0,
                 chunk_row_offset: int = 0, scale: float | None = None, flags: int = 0) -> FlashParams:
    """q f32 [batch, n_q, Hq, D] (any strides, D contiguous); out f32 [batch, n_q, Hq, D] contiguous.
    flags: FLASH_ONE_TILE selects the one-query-tile-per-CTA kernel instead of the persistent one;
    FLASH_SPLIT_COLUMNS / FLASH_WHOLE_ROWS force the persistent kernel's softmax shape (two
    warpgroups per query tile, each on half the key columns / one, a thread per row)."""
    B, n_q, Hq, D = q.shape
    p = FlashParams()
    p.q = q.data_ptr()
    p.q_nb_batch, p.q_nb_tok, p.q_nb_head = q.stride(0), q.stride(1), q.stride(2)
    p.out = out.data_ptr()
    p.k, p.v = k, v
    p.n_q, p.n_kv, p.n_q_heads, p.batch = n_q, n_kv, Hq, B
    p.scale = 1.0 / math.sqrt(D) if scale is None else scale
    p.mask_mode = mask_mode
    if mask is not None:
        p.mask = mask.data_ptr()
        p.mask_nb1 = mask.stride(-2)
        p.mask_nb2 = mask.stride(0) if mask.dim() == 3 else 0
    p.causal_offset = (n_kv - n_q) if causal_offset is None else causal_offset
    p.n_chunk_bounds = len(chunk_bounds)
    for i, b in enumerate(chunk_bounds):
        p.chunk_bounds[i] = int(b)
    p.chunk_key_offset, p.chunk_row_offset = chunk_key_offset, chunk_row_offset
    p.flags = flags
    return p


def flash(ctx: Context, q, k: Tensor, v: Tensor, n_kv: int, out=None, stream=None, **kw):
    torch = _torch()
    if out is None:
        out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    p = flash_params(q, k, v, n_kv, out, **kw)
    check(lib.cvattn_flash(ctx.handle, _stream(stream), ctypes.byref(p)), "flash")
    return out


class KVCache:
    """cosyvoice_kv_cache (src/cosyvoice-kv-cache.h:10-69) over the C object."""

    def __init__(self, ctx: Context, layers: int, head_dim: int, n_kv_heads: int, max_seq: int,
                 k_type: int, v_type: int, batch: int = 1, n_slots: int = 1, n_offloaded_slots: int = 0):
        p = KVCacheParams(layers, head_dim, head_dim, n_kv_heads, max_seq, k_type, v_type, batch, n_slots,
                          n_offloaded_slots)
        self.ctx = ctx
        self.params = p
        self.handle = ctypes.c_void_p()
        check(lib.cvattn_kv_cache_create(ctx.handle, ctypes.byref(p), ctypes.byref(self.handle)), "kv_cache_create")

    def tensor(self, layer: int, slot: int, which: int) -> Tensor:
        t = Tensor()
        check(lib.cvattn_kv_cache_tensor(self.handle, layer, slot, which, ctypes.byref(t)), "kv_cache_tensor")
        return t

    @property
    def cur_len(self) -> int:
        return int(lib.cvattn_kv_cache_get_len(self.handle))

    @cur_len.setter
    def cur_len(self, n: int) -> None:
        lib.cvattn_kv_cache_set_len(self.handle, n)

    def update(self, layer: int, k, v, pos, stream=None) -> None:
        """k, v f32 [batch, n_new, Hkv*D] contiguous; pos int32 [n_new] or [batch, n_new]."""
        n_new = k.shape[1]
        pos_nb1 = 0 if pos.dim() == 1 else pos.stride(0) * 4
        check(lib.cvattn_kv_cache_update(self.handle, _stream(stream), layer, k.data_ptr(), v.data_ptr(),
                                         pos.data_ptr(), pos_nb1, n_new), "kv_cache_update")

    def attention(self, layer: int, q, out=None, mask_mode: int = MASK_NONE, mask=None, stream=None):
        """q f32 [batch, n_q, Hq, D] contiguous -> out [batch, n_q, Hq, D]."""
        torch = _torch()
        B, n_q, Hq, D = q.shape
        if out is None:
            out = torch.empty_like(q)
        check(lib.cvattn_kv_cache_attention(self.handle, _stream(stream), layer, q.data_ptr(), n_q, Hq, mask_mode,
                                            _ptr(mask), 0 if mask is None else mask.stride(0), out.data_ptr()),
              "kv_cache_attention")
        return out

    def shift(self, n: int) -> None:
        lib.cvattn_kv_cache_shift(self.handle, n)

    def bind_slot(self, slot: int) -> bool:
        return bool(lib.cvattn_kv_cache_bind_slot(self.handle, slot))

    def slide_slot(self) -> None:
        check(lib.cvattn_kv_cache_slide_slot(self.handle), "slide_slot")

    @property
    def slot(self) -> int:
        return int(lib.cvattn_kv_cache_current_slot(self.handle))

    def offload_slot(self, idx: int, n_tokens: int, stream=None) -> None:
        check(lib.cvattn_kv_cache_offload_slot(self.handle, _stream(stream), idx, n_tokens), "offload_slot")

    def load_slot(self, idx: int, stream=None) -> None:
        check(lib.cvattn_kv_cache_load_slot(self.handle, _stream(stream), idx), "load_slot")

    def offloaded_slot(self, idx: int):
        """(bytes of host slot idx as a numpy uint8 copy, its length in positions), once its copies completed."""
        import numpy as np
        data, nbytes, n = ctypes.c_void_p(), ctypes.c_size_t(), ctypes.c_uint32()
        check(lib.cvattn_kv_cache_offloaded_slot(self.handle, idx, ctypes.byref(data), ctypes.byref(nbytes),
                                                 ctypes.byref(n)), "offloaded_slot")
        if not nbytes.value:
            return np.zeros(0, np.uint8), int(n.value)
        buf = (ctypes.c_uint8 * nbytes.value).from_address(data.value)
        return np.frombuffer(buf, dtype=np.uint8).copy(), int(n.value)

    @property
    def offloaded_size(self) -> int:
        return int(lib.cvattn_kv_cache_offloaded_size(self.handle))

    def clear_offloaded(self) -> None:
        lib.cvattn_kv_cache_clear_offloaded(self.handle)

    def close(self) -> None:
        if self.handle:
            lib.cvattn_kv_cache_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
