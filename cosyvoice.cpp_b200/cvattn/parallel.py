"""Multi-GPU host logic for the attention path (one process per GPU).

The reference serves concurrent requests with one worker context per request
slot, all on one device (src/cosyvoice-model.cpp:82-107,
tools/server/cosyvoice-server.cpp:267,318-327).  Across GPUs the same model
shards by request: each sequence's KV cache lives wholly on one GPU, so the
decode/prefill/DiT attention needs no collective on the hot path.

Two helpers cover the multi-GPU modes:
  * shard_by_length - assign sequences to ranks, balancing the KV bytes each
    rank streams (sum of context lengths), deterministically on every rank;
  * SplitKVDecode   - optional long-context mode: one sequence's positions are
    split into contiguous slices across ranks; every rank runs cvattn_decode
    with CVATTN_DECODE_EMIT_PARTIAL over its slice, the (O, max, sum) partials
    are all-gathered over NCCL, and cvattn_combine merges them (log-sum-exp).
"""
from __future__ import annotations

from typing import Sequence


def shard_by_length(lens: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-first assignment of sequence indices to `world` ranks.

    Deterministic (ties break by index), so every rank computes the same plan
    without communication.  Each returned list is sorted.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i))
    loads = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        shards[r].append(i)
        loads[r] += int(lens[i])
    return [sorted(s) for s in shards]


def split_positions(length: int, world: int, align: int = 128) -> list[tuple[int, int]]:
    """Contiguous (start, count) slices of [0, length), boundaries on `align`.

    Slices are as even as the alignment allows; trailing ranks may get an
    empty slice for short sequences.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    blocks = (length + align - 1) // align
    out, start = [], 0
    for r in range(world):
        nb = blocks // world + (1 if r < blocks % world else 0)
        end = min(length, start + nb * align)
        out.append((start, max(0, end - start)))
        start = end
    return out


def gather_partials(partial_o, partial_ml, group=None):
    """All-gather per-rank partials: [R, D] and [R, 2] -> [world, R, D] and [world, R, 2]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    po = [torch.empty_like(partial_o) for _ in range(world)]
    pml = [torch.empty_like(partial_ml) for _ in range(world)]
    dist.all_gather(po, partial_o.contiguous(), group=group)
    dist.all_gather(pml, partial_ml.contiguous(), group=group)
    return torch.stack(po), torch.stack(pml)


class SplitKVDecode:
    """Decode one long sequence whose KV positions are split across ranks.

    k_slice / v_slice: this rank's contiguous positions [start, start+count)
    as cvattn tensors (rows of the sequence on this GPU).  Call with q
    [n_q_heads, head_dim] (identical on every rank); returns the merged output
    on every rank.
    """

    def __init__(self, ctx, k_slice, v_slice, count: int, n_q_heads: int, head_dim: int = 64, group=None):
        import torch
        import cvattn as cv
        self.cv, self.ctx, self.group = cv, ctx, group
        self.k, self.v, self.count = k_slice, v_slice, count
        self.hq, self.d = n_q_heads, head_dim
        self.kv_len = torch.tensor([count], dtype=torch.int32, device="cuda")
        self.po = torch.zeros((1, n_q_heads, head_dim), dtype=torch.float32, device="cuda")
        self.pml = torch.zeros((1, n_q_heads, 2), dtype=torch.float32, device="cuda")

    def __call__(self, q):
        cv = self.cv
        if self.count > 0:
            self.cv.decode(self.ctx, q.reshape(1, self.hq, self.d), self.k, self.v, self.kv_len, self.count,
                           out=self.po, emit_partial=True, partial_ml=self.pml)
        else:
            # an empty slice (a sequence shorter than align * world) still joins the
            # gather, with the partial the combine skips: max -inf, sum 0
            self.po.zero_()
            self.pml[..., 0] = float("-inf")
            self.pml[..., 1] = 0.0
        po, pml = gather_partials(self.po[0], self.pml[0], self.group)
        return cv.combine(po, pml)
