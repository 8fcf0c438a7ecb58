"""Sequence sharding of a rollout batch across ranks (one process per GPU).

The verify round needs no collective: rollouts are independent, and the
reference's GRPO grouping keeps the samples of one prompt contiguous (rollout
index ``prompt_idx * samples + r``, flashgrpo_trainer.py:2277-2278), so each
rank owns whole prompt groups.  After generation one all-gather of the
per-rollout accepted lengths gives every rank the global statistics the GRPO
advantage and the metrics need.
"""
from __future__ import annotations

import torch


def prompt_shard(n_prompts: int, world: int, rank: int) -> range:
    """Contiguous prompt range of ``rank``: sizes differ by at most one, the
    first ``n_prompts % world`` ranks take the extra prompt."""
    if world <= 0 or not 0 <= rank < world or n_prompts < 0:
        raise ValueError(f"bad shard request: n_prompts={n_prompts} world={world} rank={rank}")
    base, extra = divmod(n_prompts, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def rollout_rows(prompts: range, samples: int) -> range:
    """Global rollout indices of a prompt range (samples of a prompt contiguous)."""
    return range(prompts.start * samples, prompts.stop * samples)


def gather_rollout_values(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gathers a 1-D per-rollout tensor whose length may differ by rank and
    returns the concatenation in rank order (i.e. in global rollout order when
    shards come from ``prompt_shard``).  Works on any backend that implements
    ``all_gather`` (NCCL for CUDA tensors, gloo for CPU tensors); with one
    process it returns a copy."""
    import torch.distributed as dist

    if local.dim() != 1:
        raise ValueError("gather_rollout_values expects a 1-D tensor")
    if not dist.is_available() or not dist.is_initialized():
        return local.clone()
    world = dist.get_world_size(group)
    n = torch.tensor([local.numel()], dtype=torch.int64, device=local.device)
    sizes = [torch.empty_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    width = max(sizes) if sizes else 0
    padded = torch.zeros(width, dtype=local.dtype, device=local.device)
    padded[: local.numel()] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)])


def reduce_scalar(value: float, op: str, device, group=None) -> float:
    """max / sum of one number over ranks (the slowest rank's time, the total
    accepted tokens); identity with one process."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM}[op], group=group)
    return float(t.item())


def gather_rollouts(local: torch.Tensor, counts: list[int], extras=(), group=None):
    """The round's one collective: a single all-gather of every rank's
    per-rollout values together with a few per-rank numbers (device time,
    token counts), the per-rank row counts known from the shard plan
    (``counts[r] = len(rollout_rows(prompt_shard(...)))``).

    Every rank sends ``max(counts) + len(extras)`` float64 slots (integers
    below 2**53 round-trip exactly).  Returns ``(values, per_rank)``: the
    per-rollout values in global rollout order, in ``local``'s dtype, and a
    ``[world, len(extras)]`` float64 tensor of every rank's numbers.  With one
    process no collective runs."""
    import torch.distributed as dist

    if local.dim() != 1:
        raise ValueError("gather_rollouts expects a 1-D tensor")
    extras = [float(x) for x in extras]
    ne = len(extras)
    if not dist.is_available() or not dist.is_initialized():
        if len(counts) != 1 or counts[0] != local.numel():
            raise ValueError(f"shard plan {counts} does not match one rank holding {local.numel()} rollouts")
        return local.clone(), torch.tensor([extras], dtype=torch.float64).reshape(1, ne)
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    if len(counts) != world or counts[rank] != local.numel():
        raise ValueError(f"shard plan {counts} does not match rank {rank} holding {local.numel()} rollouts")
    width = max(counts) + ne
    send = torch.zeros(width, dtype=torch.float64, device=local.device)
    send[: local.numel()] = local.to(torch.float64)
    if ne:
        send[width - ne:] = torch.tensor(extras, dtype=torch.float64, device=local.device)
    recv = torch.empty(world * width, dtype=torch.float64, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    recv = recv.view(world, width)
    values = torch.cat([recv[r, : counts[r]] for r in range(world)]).to(local.dtype)
    return values, recv[:, width - ne:].cpu()
