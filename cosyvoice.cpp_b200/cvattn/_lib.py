"""ctypes mirror of include/cvattn.h.

Loads the in-tree libcvattn.so built by cosyvoice.cpp_b200/build.py.  There is
no fallback: if the library is missing or its ABI does not match, importing
the bindings raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcvattn.so")
ABI_VERSION = 2
MAX_CHUNK_BOUNDS = 64

c_void_p, c_int32, c_int64, c_uint32, c_float, c_size_t, c_uint8 = (
    ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float, ctypes.c_size_t, ctypes.c_uint8)


class Tensor(ctypes.Structure):
    """cvattn_tensor: a ggml KV tensor (row = one position, every head)."""
    _fields_ = [
        ("data", c_void_p), ("type", c_int32), ("n_heads", c_int32), ("head_dim", c_int32),
        ("reserved", c_int32), ("ne1", c_int64), ("ne2", c_int64), ("nb1", c_int64), ("nb2", c_int64),
    ]


class DecodeParams(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_seq_stride", c_int64), ("out", c_void_p), ("out_seq_stride", c_int64),
        ("k", Tensor), ("v", Tensor), ("k_seq_ptrs", c_void_p), ("v_seq_ptrs", c_void_p),
        ("kv_len", c_void_p), ("k_new", c_void_p), ("v_new", c_void_p), ("partial_ml", c_void_p),
        ("n_seq", c_int32), ("n_q_heads", c_int32), ("max_kv_len", c_int32), ("flags", c_int32),
        ("scale", c_float), ("reserved", c_int32), ("workspace", c_void_p), ("workspace_size", c_size_t),
    ]


class FlashParams(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_nb_tok", c_int64), ("q_nb_head", c_int64), ("q_nb_batch", c_int64),
        ("out", c_void_p), ("k", Tensor), ("v", Tensor),
        ("n_q", c_int32), ("n_kv", c_int32), ("n_q_heads", c_int32), ("batch", c_int32),
        ("scale", c_float), ("mask_mode", c_int32), ("mask", c_void_p), ("mask_nb1", c_int64),
        ("mask_nb2", c_int64), ("causal_offset", c_int32), ("n_chunk_bounds", c_int32),
        ("chunk_bounds", c_int32 * MAX_CHUNK_BOUNDS), ("chunk_key_offset", c_int32),
        ("chunk_row_offset", c_int32), ("flags", c_int32),
    ]


class KVCacheParams(ctypes.Structure):
    _fields_ = [
        ("layers", c_int32), ("k_head_dim", c_int32), ("v_head_dim", c_int32), ("n_kv_heads", c_int32),
        ("max_seq", c_uint32), ("k_type", c_int32), ("v_type", c_int32), ("batch", c_int32),
        ("n_slots", c_int32), ("n_offloaded_slots", c_int32),
    ]


class DitStep(ctypes.Structure):
    _fields_ = [
        ("rebuild", c_uint8), ("cache_kv", c_uint8), ("load", c_uint8), ("offload", c_uint8),
        ("slide", c_uint8), ("slice", c_uint8), ("mask", c_uint8), ("reserved", c_uint8),
        ("cut_len", c_int64),
    ]


class RopeParams(ctypes.Structure):
    _fields_ = [
        ("mode", c_int32), ("n_dims", c_int32), ("unit_len", c_int32),
        ("freq_base", ctypes.c_float), ("freq_scale", ctypes.c_float), ("attn_factor", ctypes.c_float),
    ]


STRUCTS = {0: Tensor, 1: DecodeParams, 2: FlashParams, 3: KVCacheParams, 4: DitStep, 5: RopeParams}

# (name, restype, argtypes) for every symbol include/cvattn.h declares.
P = ctypes.POINTER
SIGNATURES = [
    ("cvattn_status_string", ctypes.c_char_p, [c_int32]),
    ("cvattn_status_to_ggml", c_int32, [c_int32]),
    ("cvattn_abi_version", c_int32, []),
    ("cvattn_abi_sizeof", c_size_t, [c_int32]),
    ("cvattn_row_size", c_size_t, [c_int32, c_int64]),
    ("cvattn_supports", c_int32, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    ("cvattn_kv_fallback_type", c_int32, [c_int32]),
    ("cvattn_kv_cache_type_to_ggml", c_int32, [c_int32]),
    ("cvattn_ggml_to_kv_cache_type", c_int32, [c_int32]),
    ("cvattn_negotiate_kv_types", c_int32,
     [c_uint32, c_int32, c_int32, c_int32, c_int32, P(c_int32), P(c_int32), P(c_uint32), P(c_int32)]),
    ("cvattn_context_create", c_int32, [c_int32, P(c_void_p)]),
    ("cvattn_context_destroy", None, [c_void_p]),
    ("cvattn_context_sync_status", c_int32, [c_void_p, c_void_p, P(c_int32)]),
    ("cvattn_kv_append", c_int32,
     [c_void_p, c_void_p, P(Tensor), c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int32, c_int32]),
    ("cvattn_kv_dequantize", c_int32, [c_void_p, c_void_p, P(Tensor), c_int32, c_void_p]),
    ("cvattn_rope", c_int32, [c_void_p, P(RopeParams), c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int32, c_int32]),
    ("cvattn_kv_append_rope", c_int32,
     [c_void_p, c_void_p, P(Tensor), c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int32, c_int32, P(RopeParams)]),
    ("cvattn_decode_workspace_size", c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32]),
    ("cvattn_workspace_init", c_int32, [c_void_p, c_void_p, c_size_t]),
    ("cvattn_decode", c_int32, [c_void_p, c_void_p, P(DecodeParams)]),
    ("cvattn_decode_noalloc", c_int32, [c_void_p, c_void_p, P(DecodeParams)]),
    ("cvattn_decode_rope", c_int32, [c_void_p, c_void_p, P(DecodeParams), P(RopeParams)]),
    ("cvattn_combine", c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p]),
    ("cvattn_flash", c_int32, [c_void_p, c_void_p, P(FlashParams)]),
    ("cvattn_kv_copy_to_host", c_int32, [c_void_p, P(Tensor), c_int32, c_void_p]),
    ("cvattn_kv_copy_from_host", c_int32, [c_void_p, P(Tensor), c_int32, c_void_p]),
    ("cvattn_kv_cache_create", c_int32, [c_void_p, P(KVCacheParams), P(c_void_p)]),
    ("cvattn_kv_cache_destroy", None, [c_void_p]),
    ("cvattn_kv_cache_tensor", c_int32, [c_void_p, c_int32, c_int32, c_int32, P(Tensor)]),
    ("cvattn_kv_cache_device_bytes", c_size_t, [c_void_p]),
    ("cvattn_kv_cache_get_len", c_uint32, [c_void_p]),
    ("cvattn_kv_cache_set_len", None, [c_void_p, c_uint32]),
    ("cvattn_kv_cache_update", c_int32,
     [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_int64, c_int32]),
    ("cvattn_kv_cache_attention", c_int32,
     [c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p]),
    ("cvattn_kv_cache_shift", None, [c_void_p, c_uint32]),
    ("cvattn_kv_cache_bind_slot", c_int32, [c_void_p, c_int32]),
    ("cvattn_kv_cache_slide_slot", c_int32, [c_void_p]),
    ("cvattn_kv_cache_current_slot", c_int32, [c_void_p]),
    ("cvattn_kv_cache_offload_slot", c_int32, [c_void_p, c_void_p, c_int32, c_uint32]),
    ("cvattn_kv_cache_load_slot", c_int32, [c_void_p, c_void_p, c_int32]),
    ("cvattn_kv_cache_offloaded_slot", c_int32, [c_void_p, c_int32, P(c_void_p), P(c_size_t), P(c_uint32)]),
    ("cvattn_kv_cache_offloaded_size", c_size_t, [c_void_p]),
    ("cvattn_kv_cache_clear_offloaded", None, [c_void_p]),
    ("cvattn_dit_sched_plan", c_int32,
     [c_int32, c_int32, c_int32, c_int64, c_uint32, c_int32, c_int32, P(DitStep)]),
]

_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libcvattn.so, bind every signature and verify the ABI."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python cosyvoice.cpp_b200/build.py` "
            "(the engine has no fallback implementation)")
    lib = ctypes.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.cvattn_abi_version() != ABI_VERSION:
        raise RuntimeError("libcvattn ABI version mismatch")
    for which, st in STRUCTS.items():
        got = lib.cvattn_abi_sizeof(which)
        if got != ctypes.sizeof(st):
            raise RuntimeError(f"struct {st.__name__}: library size {got} != binding size {ctypes.sizeof(st)}")
    _lib = lib
    return lib
