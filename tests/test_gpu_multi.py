"""GPU, 2 ranks over NCCL: long-context split-KV decode.

One sequence's q8_0/q4_0 KV positions are split across two GPUs; each rank
runs cvattn_decode with EMIT_PARTIAL on its slice, partials are all-gathered
over NCCL and merged by cvattn_combine.  The merged output must meet the
decode bar (rel-L2 1e-5) against fp64 attention over the whole sequence.
Skipped when fewer than two GPUs are visible.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q, L=5000):
    import datetime
    import sys
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "cosyvoice.cpp_b200"), root]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import cvattn as cv
        from cvattn.parallel import SplitKVDecode, split_positions
        from oracle import oracle as O
        ctx = cv.Context(rank)
        rng = np.random.default_rng(5)
        Hq, Hkv, D = 14, 2, 64
        kx = rng.standard_normal((L, Hkv * D)).astype(np.float32)
        vx = rng.standard_normal((L, Hkv * D)).astype(np.float32)
        q = rng.standard_normal((Hq, D)).astype(np.float32)
        kq, vq = O.quantize(O.Q8_0, kx), O.quantize(O.Q4_0, vx)
        start, count = split_positions(L, world)[rank]
        # an empty slice (L < 128 * world) keeps a one-row buffer: SplitKVDecode skips its decode
        kbuf = torch.tensor(kq[start:start + max(count, 1)].reshape(-1), device="cuda")
        vbuf = torch.tensor(vq[start:start + max(count, 1)].reshape(-1), device="cuda")
        kd = cv.kv_tensor(kbuf, cv.Q8_0, Hkv, D, max(count, 1), 1)
        vd = cv.kv_tensor(vbuf, cv.Q4_0, Hkv, D, max(count, 1), 1)
        dec = SplitKVDecode(ctx, kd, vd, count, Hq, D)
        out = dec(torch.tensor(q, device="cuda")).cpu().numpy()
        torch.cuda.synchronize()
        err = None
        if rank == 0:
            kdq = O.dequantize(O.Q8_0, kq, Hkv * D).reshape(L, Hkv, D)
            vdq = O.dequantize(O.Q4_0, vq, Hkv * D).reshape(L, Hkv, D)
            ref = O.attention_f64(q[None], kdq, vdq, 0.125)[0]
            err = float(np.linalg.norm(out - ref) / np.linalg.norm(ref))
        result_q.put((rank, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("L", [5000, 100])
def test_split_kv_decode_two_gpus(L):
    """L = 100 leaves rank 1 an empty slice: it must still join the gather."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_worker, args=(r, 2, port, q, L)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] is not None and res[0] <= 1e-5, f"rel-L2 {res[0]}"
