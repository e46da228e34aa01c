"""Batch-row sharding over one process per GPU.

Rows of a Dispatcher-Hybrid batch never interact: the parallel forward is
row-independent and the lockstep decoder keeps per-row caches (the
reference's batched == solo test, tests/test_decoding.py:134-153).  So a
multi-GPU run replicates the weights, gives each rank a contiguous block of
rows, and exchanges only what the caller needs back: the sampled tokens of
each decode step and, for output, logits rows.  Collectives go through
`torch.distributed` (NCCL between GPUs, gloo on the CPU for tests).
"""

import torch
import torch.distributed as dist


def world_info():
    """(world_size, rank) of the default process group, (1, 0) without one."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def shard_rows(n_rows, world, rank):
    """Contiguous block of rows owned by `rank`: [rank*n//world, (rank+1)*n//world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_rows < world:
        raise ValueError(f"{n_rows} rows cannot be sharded over {world} ranks")
    return slice(rank * n_rows // world, (rank + 1) * n_rows // world)


def shard_sizes(n_rows, world):
    return [shard_rows(n_rows, world, r).stop - shard_rows(n_rows, world, r).start
            for r in range(world)]


def gather_rows(local, n_rows, group=None):
    """Concatenate every rank's block of rows (dim 0) in rank order.  Blocks
    may differ in size by one row (shard_rows); they are padded to the
    largest for the collective and trimmed after."""
    world, _ = world_info()
    if world == 1:
        return local
    sizes = shard_sizes(n_rows, world)
    if local.shape[0] != sizes[dist.get_rank(group)]:
        raise ValueError(f"local block has {local.shape[0]} rows, shard owns "
                         f"{sizes[dist.get_rank(group)]}")
    cap = max(sizes)
    if local.shape[0] < cap:
        pad = local.new_zeros((cap - local.shape[0],) + tuple(local.shape[1:]))
        local = torch.cat([local, pad])
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)])


def max_over_ranks(value, device=None):
    """Largest `value` (a Python float) over all ranks."""
    world, _ = world_info()
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(device=None):
    world, _ = world_info()
    if world > 1:
        if device is not None and torch.device(device).type == "cuda":
            dist.barrier(device_ids=[torch.device(device).index or 0])
        else:
            dist.barrier()


class ShardedGreedyDecode:
    """Lockstep greedy decode of a batch split over ranks.

    `decoder` is this rank's decoder (any object with the reference decoder's
    `prefill(idx) -> logits (B, T, V)` and `step(tokens) -> logits (B, V)`),
    built for this rank's block of rows.  Every step samples locally and
    all-gathers the tokens, so every rank ends with the whole batch's tokens
    (n_rows, steps), in row order."""

    def __init__(self, decoder, n_rows):
        self.decoder = decoder
        self.n_rows = n_rows

    @torch.no_grad()
    def run(self, local_prompt, steps):
        logits = self.decoder.prefill(local_prompt)
        tok = logits[:, -1].argmax(-1)
        out = [gather_rows(tok, self.n_rows)]
        for _ in range(steps - 1):
            tok = self.decoder.step(tok).argmax(-1)
            out.append(gather_rows(tok, self.n_rows))
        return torch.stack(out, dim=1)
