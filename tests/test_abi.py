"""CPU: the C-ABI library loads, exports every declared symbol, and its host
logic (type maps, fallback chain, KV-type negotiation, DiT step plan, status
mapping) matches the reference's rules.  No kernel is launched here."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "cvattn.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(cvattn_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def cvl():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "cosyvoice.cpp_b200"))
    import cvattn
    return cvattn


def test_every_declared_symbol_is_exported(cvl):
    lib = ctypes.CDLL(cvl._lib.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    bound = {s[0] for s in cvl._lib.SIGNATURES}
    assert set(names) == bound, set(names) ^ bound


def test_struct_sizes_match_bindings(cvl):
    for which, st in cvl._lib.STRUCTS.items():
        assert cvl.lib.cvattn_abi_sizeof(which) == ctypes.sizeof(st)
    assert cvl.lib.cvattn_abi_version() == cvl._lib.ABI_VERSION == 2


def test_row_sizes(cvl):
    # ggml_row_size for the LLM row (2 heads x 64) and the DiT row (16 x 64)
    exp = {cvl.F32: 512, cvl.F16: 256, cvl.Q8_0: 136, cvl.Q5_1: 96, cvl.Q5_0: 88, cvl.Q4_1: 80, cvl.Q4_0: 72}
    for t, b in exp.items():
        assert cvl.row_size(t, 128) == b
        assert cvl.row_size(t, 1024) == b * 8
    assert cvl.row_size(cvl.Q8_0, 33) == 0
    assert cvl.row_size(99, 128) == 0


def test_supports_all_kv_pairs_for_qwen2_and_dit(cvl):
    for k in cvl.KV_TYPES:
        for v in cvl.KV_TYPES:
            assert cvl.supports(k, v, 64, 14, 2)
            assert cvl.supports(k, v, 64, 16, 16)
    assert not cvl.supports(cvl.Q8_0, cvl.Q8_0, 128, 14, 2)
    assert not cvl.supports(cvl.Q8_0, cvl.Q8_0, 64, 14, 3)
    assert not cvl.supports(30, cvl.Q8_0, 64, 14, 2)


def test_fallback_chain(cvl):
    # src/cosyvoice-loader.cpp:498-510
    chain = [cvl.Q4_0]
    while chain[-1] != -1:
        chain.append(cvl.lib.cvattn_kv_fallback_type(chain[-1]))
    assert chain == [cvl.Q4_0, cvl.Q4_1, cvl.Q5_0, cvl.Q5_1, cvl.Q8_0, cvl.F16, cvl.F32, -1]


def test_type_maps(cvl):
    # include/cosyvoice.h:32-42 order vs ggml ids
    exp = [cvl.F32, cvl.F16, cvl.Q8_0, cvl.Q5_1, cvl.Q5_0, cvl.Q4_1, cvl.Q4_0]
    for i, g in enumerate(exp):
        assert cvl.lib.cvattn_kv_cache_type_to_ggml(i) == g
        assert cvl.lib.cvattn_ggml_to_kv_cache_type(g) == i
    assert cvl.lib.cvattn_kv_cache_type_to_ggml(7) == -1


def test_negotiation_keeps_requested_types(cvl):
    # CLI default --llm-kv-cache-type k=q8_0,v=q4_0,fallback=q8_0 (tools/cli/cosyvoice-cli.cpp:80-88)
    u = cvl.make_separate_kv_cache(cvl.CV_Q8_0, cvl.CV_Q4_0, cvl.CV_Q8_0)
    st, k, v, ru, fa = cvl.negotiate_kv_types(u, True, 64, 14, 2)
    assert (st, k, v, fa) == (0, cvl.Q8_0, cvl.Q4_0, 1)
    assert ru == cvl.make_separate_kv_cache(cvl.CV_Q8_0, cvl.CV_Q4_0, cvl.CV_Q4_0)
    # plain (non-separate) value applies to K and V
    st, k, v, ru, fa = cvl.negotiate_kv_types(cvl.CV_Q5_1, False, 64, 14, 2)
    assert (st, k, v, ru, fa) == (0, cvl.Q5_1, cvl.Q5_1, cvl.CV_Q5_1, 1)
    # an unsupported head shape walks the fallback chain and fails cleanly
    st, *_ = cvl.negotiate_kv_types(cvl.CV_Q8_0, True, 96, 14, 2)
    assert st != 0


def test_status_strings_and_ggml_mapping(cvl):
    for s in range(9):
        assert cvl.lib.cvattn_status_string(s)
    assert cvl.lib.cvattn_status_to_ggml(0) == 0
    assert cvl.lib.cvattn_status_to_ggml(4) == -2
    assert cvl.lib.cvattn_status_to_ggml(1) == -1


@pytest.mark.parametrize("streaming", [False, True])
@pytest.mark.parametrize("offset", [0, 100])
@pytest.mark.parametrize("slots", [(0, 0), (2, 3), (1, 9), (0, 10), (5, 0)])
@pytest.mark.parametrize("slidable", [True, False])
def test_dit_plan_matches_reference_restatement(cvl, streaming, offset, slots, slidable):
    from oracle import oracle as O
    n_off, n_fix = slots
    got = cvl.dit_sched_plan(10, n_off, n_fix, 17, offset, streaming, slidable)
    exp = O.dit_sched_plan(10, n_off, n_fix, 17, offset, streaming, slidable)
    for g, e in zip(got, exp):
        assert {k: bool(v) if k != "cut_len" else int(v) for k, v in g.items()} == \
               {k: bool(v) if k != "cut_len" else int(v) for k, v in e.items()}


def test_no_device_calls_fail_cleanly_without_gpu(cvl):
    import torch
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    h = ctypes.c_void_p()
    st = cvl.lib.cvattn_context_create(0, ctypes.byref(h))
    assert st in (5, 7)     # CUDA error or no device, never a crash
