"""Multi-rank host logic of the sequence-sharded round, on CPU with gloo.

Two processes stand in for two GPUs: each owns a contiguous range of whole
prompt groups, produces per-rollout values, and the one collective of the
path (an all-gather of per-rollout accepted lengths, plus the max-over-ranks
time and the summed token count) must reproduce the global view in global
rollout order.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashgrpo_b200.engine import shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_prompt_shards_are_contiguous_disjoint_and_cover():
    for n in range(0, 23):
        for world in range(1, 9):
            seen = []
            for r in range(world):
                rg = shard.prompt_shard(n, world, r)
                seen.extend(rg)
                assert len(rg) in (n // world, n // world + 1)
            assert seen == list(range(n))
    assert shard.rollout_rows(range(3, 5), 8) == range(24, 40)
    with pytest.raises(ValueError):
        shard.prompt_shard(4, 2, 2)


def _rollout_value(global_row: int) -> int:
    return (global_row * 7919) % 97 + 1


def _worker(rank: int, world: int, port: int, n_prompts: int, samples: int):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prompts = shard.prompt_shard(n_prompts, world, rank)
        rows = shard.rollout_rows(prompts, samples)
        local = torch.tensor([_rollout_value(i) for i in rows], dtype=torch.int32)
        got = shard.gather_rollout_values(local)
        want = torch.tensor([_rollout_value(i) for i in range(n_prompts * samples)], dtype=torch.int32)
        assert torch.equal(got, want), (rank, got, want)
        # slowest rank's time and total tokens, as bench.py reports them
        assert shard.reduce_scalar(1.5 + rank, "max", "cpu") == 1.5 + world - 1
        assert shard.reduce_scalar(float(local.sum()), "sum", "cpu") == float(want.sum())
        # the single all-gather bench.py runs: sizes from the shard plan, the
        # per-rank time and token count riding in the same buffer
        counts = [len(shard.rollout_rows(shard.prompt_shard(n_prompts, world, r), samples)) for r in range(world)]
        got2, per_rank = shard.gather_rollouts(local, counts, extras=(1.5 + rank, float(local.sum())))
        assert torch.equal(got2, want), (rank, got2, want)
        assert per_rank.shape == (world, 2)
        assert per_rank[:, 0].max().item() == 1.5 + world - 1
        assert per_rank[:, 1].sum().item() == float(want.sum())
        with pytest.raises(ValueError):
            shard.gather_rollouts(local, [c + 1 for c in counts])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_prompts", [4, 5, 1])
def test_gather_of_accepted_lengths_two_ranks(n_prompts):
    # n_prompts = 5 gives ragged shards (3 + 2 groups), 1 leaves rank 1 empty
    mp.spawn(_worker, args=(2, _free_port(), n_prompts, 8), nprocs=2, join=True)


def test_single_process_gather_is_identity():
    x = torch.arange(5, dtype=torch.int32)
    assert torch.equal(shard.gather_rollout_values(x), x)
    assert shard.reduce_scalar(3.0, "max", "cpu") == 3.0
    vals, per_rank = shard.gather_rollouts(x, [5], extras=(2.0, 7.0))
    assert torch.equal(vals, x) and per_rank.tolist() == [[2.0, 7.0]]
