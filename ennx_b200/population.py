"""Population data parallelism: antithetic pairs shard over ranks.

One process per GPU.  Every rank holds a replica of the base weights,
evaluates its own contiguous range of antithetic pairs (regenerating their
noise from the population seed), and the only exchange per step is an
all-gather of the fp32 fitness vector plus one broadcast from rank 0 of the
next seed and the update coefficients -- NCCL on GPUs, gloo on CPU (tests).
Each rank then applies the update to its own replica by regenerating every
pair's noise from the seed, so no weight ever crosses the interconnect.
The reference has no multi-device path (its CUDA runtime is pinned to
device 0, cuda/src/lib.rs:144); this module is the B200 design's scale-out.

``ResidentEsState`` mirrors the reference's ask -> evaluate -> tell session
(``ResidentBoState::ask`` / ``tell`` / ``ask_evaluate``,
rust/crates/ennx/src/forward_program.rs:633-729) for a Gaussian population.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

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
    fitness: torch.Tensor          # [2 * num_pairs], candidate 2p+s at index 2p+s
    next_seed: int
    coefficients: Optional[torch.Tensor] = None  # [num_pairs] update coefficients (lr given)


class PopulationStep:
    """One population step: local evaluation, fitness exchange, and (with a
    learning rate) the update coefficients.

    ``evaluate(tokens, seed, sigma, first_pair, count) -> tensor[2*count]`` is
    the per-rank evaluator (``PopulationEvaluator`` on a GPU).
    ``coefficients(fitness, sigma, lr, num_pairs) -> tensor[num_pairs]`` runs
    on rank 0 only; ``update(seed, coefficients)`` runs on every rank after
    the broadcast and moves its replica (``PopulationEvaluator.update``)."""

    def __init__(self, evaluate: Callable, num_pairs: int, sigma: float, group=None, lr: float | None = None,
                 coefficients: Callable | None = None, update: Callable | None = None):
        self.evaluate, self.num_pairs, self.sigma, self.group = evaluate, num_pairs, sigma, group
        self.lr, self.coefficients, self.update = lr, coefficients, update
        if lr is not None and coefficients is None:
            raise ValueError("a learning rate needs a coefficients function")
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.first, self.count = shard_pairs(num_pairs, self.world, self.rank)
        counts = [shard_pairs(num_pairs, self.world, r)[1] for r in range(self.world)]
        if len(set(counts)) != 1:
            raise ValueError(f"{num_pairs} pairs do not shard evenly over {self.world} ranks")

    def _src(self) -> int:
        return dist.get_global_rank(self.group, 0) if self.group is not None else 0

    def __call__(self, tokens: torch.Tensor, seed: int) -> StepResult:
        local = self.evaluate(tokens, seed, self.sigma, self.first, self.count)
        P = self.num_pairs
        if self.world == 1:
            full = local
        else:
            full = torch.empty(2 * P, dtype=local.dtype, device=local.device)
            dist.all_gather_into_tensor(full, local.contiguous(), group=self.group)
        coef = None
        # rank 0 decides; one broadcast carries the next seed (int64) and the
        # coefficients (f32[P]) as bytes
        msg = torch.empty(8 + (4 * P if self.lr is not None else 0), dtype=torch.uint8, device=local.device)
        if self.rank == 0:
            msg[:8].view(torch.int64).fill_(seed + 1)
            if self.lr is not None:
                msg[8:].view(torch.float32).copy_(self.coefficients(full, self.sigma, self.lr, P))
        if self.world > 1:
            dist.broadcast(msg, src=self._src(), group=self.group)
        if self.lr is not None:
            coef = msg[8:].view(torch.float32)
            if self.update is not None:
                self.update(seed, coef)
        return StepResult(full, int(msg[:8].view(torch.int64).item()), coef)


@dataclass(frozen=True)
class EsRound:
    """One pending population round: the seed its noise is drawn from."""
    seed: int
    step: int


class ResidentEsState:
    """ask -> evaluate -> tell over a resident Gaussian population
    (``ResidentBoState``, forward_program.rs:633-729): ``ask`` opens a round
    for the current seed, ``tell`` takes the round's fitness vector (device
    f32 [2P], the evaluator's output, no host copy), computes the update
    coefficients and moves the resident weights, and ``ask_evaluate`` chains
    the three through a ``PopulationStep``.  The reference's error strings
    are kept for the round bookkeeping."""

    def __init__(self, step: PopulationStep, seed: int = 0):
        if step.lr is None or step.update is None:
            raise ValueError("the resident state needs a step with a learning rate and an update")
        self.step, self.seed = step, seed
        self.pending: EsRound | None = None
        self.rounds = 0
        self.fitness: list[torch.Tensor] = []

    def ask(self) -> EsRound:
        if self.pending is not None:
            raise ValueError("tell must finish the resident forward round before ask")
        self.pending = EsRound(self.seed, self.rounds)
        return self.pending

    def tell(self, round_: EsRound, fitness: torch.Tensor) -> torch.Tensor:
        """Apply the update of a round whose fitness vector is already known
        on every rank (single process, or after a gather); returns the
        coefficients."""
        self._take(round_)
        coef = self.step.coefficients(fitness, self.step.sigma, self.step.lr, self.step.num_pairs)
        self.step.update(round_.seed, coef)
        self._finish(round_.seed + 1, fitness)
        return coef

    def _take(self, round_: EsRound):
        if self.pending is None:
            raise ValueError("no resident forward round is pending")
        if round_ != self.pending:
            raise ValueError("resident forward round does not match pending trial")
        self.pending = None

    def _finish(self, next_seed: int, fitness: torch.Tensor):
        self.seed = next_seed
        self.rounds += 1
        self.fitness.append(fitness)

    def ask_evaluate(self, tokens: torch.Tensor) -> tuple[EsRound, torch.Tensor]:
        """Evaluate the round on every rank's shard, exchange, update: the
        fitness vector of the whole population is returned."""
        round_ = self.ask()
        try:
            res = self.step(tokens, round_.seed)
        except BaseException:
            self.pending = None
            raise
        self._take(round_)
        self._finish(res.next_seed, res.fitness)
        return round_, res.fitness
