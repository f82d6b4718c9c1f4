"""CPU, world_size 2 over gloo: the multi-GPU host logic.

Requests shard by sequence (no collective on the hot path); the optional
long-context mode splits positions, all-gathers (O, max, sum) partials and
merges them with a log-sum-exp.  Here every rank computes its partials with
the fp64 oracle on its slice, the gather runs over gloo, and the merged
result must equal attention over the whole sequence.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partials(q, k, v, scale):
    """fp64 (unnormalized O, max in log2 units, sum) for q [H, D], k/v [n, Hkv, D]."""
    H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    o = np.zeros((H, D))
    ml = np.zeros((H, 2))
    for h in range(H):
        s = (k[:, h // G, :].astype(np.float64) @ q[h].astype(np.float64)) * scale / np.log(2.0)
        if s.size == 0:
            ml[h] = (-np.inf, 0.0)
            continue
        m = s.max()
        p = np.exp2(s - m)
        o[h] = p @ v[:, h // G, :]
        ml[h] = (m, p.sum())
    return o.astype(np.float32), ml.astype(np.float32)


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, os.path.join(root, "cosyvoice.cpp_b200"))
        from cvattn.parallel import gather_partials, shard_by_length, split_positions

        # --- request sharding: same plan on every rank, a partition, balanced
        lens = np.random.default_rng(0).integers(128, 2049, 64).tolist()
        plan = shard_by_length(lens, world)
        mine = torch.tensor(plan[rank], dtype=torch.int64)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([len(mine)]))
        gathered = [torch.zeros(int(s.item()), dtype=torch.int64) for s in sizes]
        if len(set(int(s.item()) for s in sizes)) == 1:
            dist.all_gather(gathered, mine)
        else:
            for r in range(world):
                buf = mine.clone() if r == rank else gathered[r]
                dist.broadcast(buf, src=r)
                gathered[r] = buf
        union = sorted(int(x) for g in gathered for x in g.tolist())
        loads = [sum(lens[i] for i in g.tolist()) for g in gathered]

        # --- split-KV long context: partials of this rank's slice, gathered and merged
        rng = np.random.default_rng(42)
        L, Hq, Hkv, D = 3000, 14, 2, 64
        k = rng.standard_normal((L, Hkv, D)).astype(np.float32)
        v = rng.standard_normal((L, Hkv, D)).astype(np.float32)
        q = rng.standard_normal((Hq, D)).astype(np.float32)
        start, count = split_positions(L, world)[rank]
        o, ml = _partials(q, k[start:start + count], v[start:start + count], 0.125)
        po, pml = gather_partials(torch.from_numpy(o), torch.from_numpy(ml))
        po, pml = po.numpy(), pml.numpy()
        M = pml[:, :, 0].max(axis=0)
        w = np.exp2(pml[:, :, 0] - M)
        merged = (w[:, :, None] * po).sum(0) / (w * pml[:, :, 1]).sum(0)[:, None]
        full_o, full_ml = _partials(q, k, v, 0.125)
        full = full_o / full_ml[:, 1:2]
        err = float(np.abs(merged - full).max())

        # --- a sequence shorter than 128 * world: the trailing rank's slice is empty;
        # it still joins the gather with the partial the merge skips (max -inf, sum 0)
        Ls = 100
        start, count = split_positions(Ls, world)[rank]
        assert (count == 0) == (rank > 0)
        if count:
            o, ml = _partials(q, k[start:start + count], v[start:start + count], 0.125)
        else:
            o = np.zeros((Hq, D), np.float32)
            ml = np.tile(np.array([-np.inf, 0.0], np.float32), (Hq, 1))
        po, pml = gather_partials(torch.from_numpy(o), torch.from_numpy(ml))
        po, pml = po.numpy(), pml.numpy()
        M = pml[:, :, 0].max(axis=0)
        w = np.where(np.isinf(pml[:, :, 0]), 0.0, np.exp2(pml[:, :, 0] - M))
        merged = (w[:, :, None] * po).sum(0) / (w * pml[:, :, 1]).sum(0)[:, None]
        full_o, full_ml = _partials(q, k[:Ls], v[:Ls], 0.125)
        err = max(err, float(np.abs(merged - full_o / full_ml[:, 1:2]).max()))
        result_q.put((rank, union, loads, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_ranks_shard_and_split_kv_combine():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=100) for _ in procs]
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    lens = np.random.default_rng(0).integers(128, 2049, 64).tolist()
    for rank, union, loads, err in results:
        assert union == list(range(64)), "every sequence on exactly one rank"
        assert max(loads) - min(loads) <= max(lens), "balanced by KV length"
        assert err < 1e-5, f"rank {rank}: merged split-KV differs by {err}"


def test_split_positions_cover_and_align():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "cosyvoice.cpp_b200"))
    from cvattn.parallel import shard_by_length, split_positions
    for L in (1, 127, 128, 129, 3000, 4096):
        for world in (1, 2, 4, 8):
            sl = split_positions(L, world)
            assert sum(c for _, c in sl) == L
            pos = 0
            for s, c in sl:
                assert s == pos and (c == 0 or s % 128 == 0)
                pos += c
    plan = shard_by_length([5, 5, 5, 5], 3)
    assert sorted(i for p in plan for i in p) == [0, 1, 2, 3]
