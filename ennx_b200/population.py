"""Population data parallelism: antithetic pairs shard over ranks.

One process per GPU.  Every rank holds a replica of the base weights,
evaluates its own contiguous range of antithetic pairs (regenerating their
noise from the population seed), and the only exchange per step is an
all-gather of the fp32 fitness vector plus a broadcast of the next seed from
rank 0 -- NCCL on GPUs, gloo on CPU (tests).  The reference has no
multi-device path (its CUDA runtime is pinned to device 0,
cuda/src/lib.rs:144); this module is the B200 design's scale-out.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def shard_pairs(num_pairs: int, world: int, rank: int) -> tuple[int, int]:
    """(first_pair, count) of `rank`; pairs are split as evenly as possible."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, extra = divmod(num_pairs, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


@dataclass
class StepResult:
    fitness: torch.Tensor  # [2 * num_pairs], candidate 2p+s at index 2p+s
    next_seed: int


class PopulationStep:
    """Runs one population step: local evaluation + fitness exchange.

    `evaluate(tokens, seed, sigma, first_pair, count) -> tensor[2*count]` is
    the per-rank evaluator (``PopulationEvaluator`` on a GPU)."""

    def __init__(self, evaluate: Callable, num_pairs: int, sigma: float, group=None):
        self.evaluate, self.num_pairs, self.sigma, self.group = evaluate, num_pairs, sigma, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.first, self.count = shard_pairs(num_pairs, self.world, self.rank)
        counts = [shard_pairs(num_pairs, self.world, r)[1] for r in range(self.world)]
        if len(set(counts)) != 1:
            raise ValueError(f"{num_pairs} pairs do not shard evenly over {self.world} ranks")

    def __call__(self, tokens: torch.Tensor, seed: int, device=None) -> StepResult:
        local = self.evaluate(tokens, seed, self.sigma, self.first, self.count)
        if self.world == 1:
            return StepResult(local, seed + 1)
        full = torch.empty(2 * self.num_pairs, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(full, local.contiguous(), group=self.group)
        nxt = torch.tensor([seed + 1 if self.rank == 0 else -1], dtype=torch.int64, device=local.device)
        dist.broadcast(nxt, src=0, group=self.group)
        return StepResult(full, int(nxt.item()))
