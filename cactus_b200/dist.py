"""Data-parallel serving across GPUs of one node: one process per GPU, no data-path collective.

Batch-1 decode runs as independent replicas (each rank serves its own request stream).
Batched decode partitions independent sequences contiguously across ranks (B_g = ceil(B/n));
every rank holds a full weight replica and its own KV cache, runs its shard through the
engine, and the host gathers the generated tokens. The only collectives are host-side
bookkeeping (barriers, the max of the per-rank device times, the gather of the token
arrays), never on the per-token data path.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np


@dataclass
class DistEnv:
    rank: int = 0
    local_rank: int = 0
    world: int = 1


def env() -> DistEnv:
    """Rank layout from the torchrun environment (single process when unset)."""
    return DistEnv(int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
                   int(os.environ.get("WORLD_SIZE", 1)))


def shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous shard [start, end) of n independent items for `rank`: the first ranks get
    ceil(n/world) items, the rest what is left (possibly nothing)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    per = -(-n // world)
    start = min(n, rank * per)
    return start, min(n, start + per)


def generate_sharded(engine, prompts: np.ndarray, max_new: int, rank: int, world: int, pg=None) -> np.ndarray | None:
    """Greedy decode of independent sequences `prompts` [B, P] split across ranks.

    Each rank runs its shard through `engine.generate_batch_greedy` (or `generate_greedy` for
    a shard of one); rank 0 returns the gathered [B, max_new] tokens in input order, the other
    ranks return None. `pg` is a torch.distributed module/group (None for one process)."""
    prompts = np.ascontiguousarray(prompts, np.uint32)
    B = prompts.shape[0]
    s0, s1 = shard(B, rank, world)
    mine = np.zeros((s1 - s0, max_new), np.uint32)
    if s1 > s0:
        if s1 - s0 == 1:
            mine[0] = engine.generate_greedy(prompts[s0], max_new)
        else:
            mine[:] = engine.generate_batch_greedy(prompts[s0:s1], max_new)
    if pg is None or world == 1:
        return mine
    parts = [None] * world
    pg.all_gather_object(parts, (s0, mine))
    if rank != 0:
        return None
    out = np.zeros((B, max_new), np.uint32)
    for start, arr in parts:
        out[start:start + arr.shape[0]] = arr
    return out


def max_over_ranks(values, pg=None, device=None):
    """Element-wise max (timing) and sum (counts) of a float vector over ranks."""
    import torch
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if pg is None:
        return t.tolist(), t.tolist()
    mx, sm = t.clone(), t.clone()
    pg.all_reduce(mx, op=pg.ReduceOp.MAX)
    pg.all_reduce(sm, op=pg.ReduceOp.SUM)
    return mx.tolist(), sm.tolist()
