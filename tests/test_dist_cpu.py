"""Host logic of the multi-GPU path on CPU: two gloo ranks split independent sequences,
decode their shards with an engine stand-in and gather the tokens; the per-rank times are
combined as max (timing) and sum (counts), as bench.py does."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from cactus_b200 import dist as D


class FakeEngine:
    """Deterministic stand-in for the device engine: token t of a sequence is a hash of its
    prompt and t (the multi-GPU logic only moves whole sequences)."""

    def generate_greedy(self, prompt, max_new):
        return self.generate_batch_greedy(np.asarray(prompt)[None], max_new)[0]

    def generate_batch_greedy(self, prompts, max_new):
        prompts = np.asarray(prompts, np.uint64)
        h = (prompts.sum(axis=1, keepdims=True) * 2654435761 + prompts[:, :1]) % 50021
        return ((h + np.arange(max_new)[None] * 7919) % 50021).astype(np.uint32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, B, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    prompts = np.random.default_rng(1).integers(0, 1000, (B, 16)).astype(np.uint32)
    toks = D.generate_sharded(FakeEngine(), prompts, 5, rank, world, dist)
    mx, sm = D.max_over_ranks([1.0 + rank, 10.0], dist)
    if rank == 0:
        np.save(out_path, toks)
        np.save(out_path + ".red.npy", np.array(mx + sm))
    dist.barrier()
    dist.destroy_process_group()


def test_shard_partition():
    for n in (0, 1, 5, 7, 8, 256):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s0, s1 = D.shard(n, r, world)
                assert 0 <= s0 <= s1 <= n
                seen += list(range(s0, s1))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        D.shard(4, 2, 2)


@pytest.mark.parametrize("B", [1, 5, 8])
def test_two_gloo_ranks_gather_in_order(tmp_path, B):
    out = str(tmp_path / "toks.npy")
    mp.spawn(_worker, args=(2, _free_port(), B, out), nprocs=2, join=True)
    got = np.load(out)
    prompts = np.random.default_rng(1).integers(0, 1000, (B, 16)).astype(np.uint32)
    assert np.array_equal(got, FakeEngine().generate_batch_greedy(prompts, 5))
    red = np.load(out + ".red.npy")
    assert red.tolist() == [2.0, 10.0, 3.0, 20.0]  # max of (1, 2), max of (10, 10), sums
