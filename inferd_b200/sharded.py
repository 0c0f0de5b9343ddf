"""Sequence sharding across the GPUs of one node.

Decode attention needs no cross-GPU exchange: each sequence's KV pages live in one GPU's
pool, so every rank owns a slice of the batch (its own PagedKVCache, block tables and
kernels) and the only collective is gathering the per-rank attention outputs, in global
sequence order, after each step.  The reference runs one process on one GPU
(core/model_runner.py); this module is what spreads its batch over N of them.

    lo, hi = shard_range(num_seqs, world, rank)              # contiguous, equal counts
    owners = assign_by_tokens(context_lens, world)           # balanced KV bytes, ragged counts
    full = gather_outputs(local_out, counts, group=None)     # all ranks get [sum(counts), ...]

`gather_outputs` uses NCCL's all-gather into one tensor when the process group is NCCL and
every shard has the same size, else a padded all-gather (also what gloo ranks on CPU use).
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def shard_range(num_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) slice of num_items for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if num_items < 0:
        raise ValueError("num_items must be >= 0")
    base, extra = divmod(num_items, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def assign_by_tokens(context_lens, world: int) -> list[list[int]]:
    """Sequence indices per rank so that each rank's total context (its KV bytes, the
    attention kernel's work) is balanced: longest sequence first onto the least-loaded rank.
    Each rank's list is sorted, so its outputs keep the global order within the shard."""
    if world <= 0:
        raise ValueError("world must be >= 1")
    lens = [int(v) for v in context_lens]
    if any(v < 0 for v in lens):
        raise ValueError("context lengths must be >= 0")
    heap = [(0, r) for r in range(world)]
    owners: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda j: (-lens[j], j)):
        load, r = heapq.heappop(heap)
        owners[r].append(i)
        heapq.heappush(heap, (load + lens[i], r))
    return [sorted(o) for o in owners]


def gather_outputs(local: torch.Tensor, counts: list[int] | None = None, *, group=None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather each rank's [count_r, ...] output along dim 0 into [sum(counts), ...], rank
    order.  counts=None means every rank holds local.shape[0] rows."""
    world = dist.get_world_size(group)
    if counts is None:
        counts = [local.shape[0]] * world
    if len(counts) != world:
        raise ValueError(f"{len(counts)} counts for a world of {world}")
    if local.shape[0] != counts[dist.get_rank(group)]:
        raise ValueError("local rows differ from this rank's count")
    total = sum(counts)
    tail = tuple(local.shape[1:])
    if out is None:
        out = torch.empty((total,) + tail, dtype=local.dtype, device=local.device)
    elif tuple(out.shape) != (total,) + tail:
        raise ValueError("out has the wrong shape")
    local = local.contiguous()
    equal = all(c == counts[0] for c in counts)
    if equal and dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
        return out
    width = max(counts)
    padded = torch.zeros((width,) + tail, dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    row = 0
    for c, part in zip(counts, parts):
        out[row:row + c] = part[:c]
        row += c
    return out
