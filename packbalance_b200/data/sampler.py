"""Deterministic two-level step/rank scheduler.

Every rank builds the same schedule from the same pack list and seed, so balancing
costs no communication.  Levels (reference ``data/sampler.py:108-195``):

1. packs -> steps: longest-processing-time first; each pack (most expensive first,
   seeded random tie-break) goes to the currently cheapest step that still has one
   of its ``world_size * grad_accum`` slots free;
2. step -> ranks: within a step, packs (most expensive first) go to the rank with
   the smallest ``(epoch-to-date load + load in this step, load in this step, rank)``
   among ranks with fewer than ``grad_accum`` packs, which rotates heavy packs
   across ranks over the epoch.

Step order is then shuffled.  ``random`` mode deals a random subset round-robin and
ignores cost.  The RNG call order matches the reference so schedules agree.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np

from packbalance_b200.data.packer import Pack


@dataclass
class StepPlan:
    step: int
    rank_packs: list[list[int]]
    step_tokens: int
    step_compute_tokens: int
    step_cost: float
    rank_costs: list[float]


@dataclass
class Schedule:
    steps: list[StepPlan]
    world_size: int
    grad_accum: int

    def rank_indices(self, rank: int) -> list[int]:
        return [i for plan in self.steps for i in plan.rank_packs[rank]]

    @property
    def steps_per_epoch(self) -> int:
        return len(self.steps)

    @property
    def tokens_per_epoch(self) -> int:
        return sum(p.step_tokens for p in self.steps)

    def stats(self) -> dict[str, float]:
        if not self.steps:
            return {}
        step_cost = np.array([p.step_cost for p in self.steps], dtype=np.float64)
        cells = np.array([p.rank_costs for p in self.steps], dtype=np.float64)
        mean = float(step_cost.mean())
        cell_mean = float(cells.mean())
        return {
            "steps": len(self.steps),
            "step_cost_mean": mean,
            "step_cost_cv": float(step_cost.std() / mean) if mean else 0.0,
            "step_cost_p99_over_mean": float(np.percentile(step_cost, 99) / mean) if mean else 0.0,
            "rank_cost_imbalance": float(cells.max() / cell_mean - 1.0) if cell_mean else 0.0,
            "tokens": int(sum(p.step_tokens for p in self.steps)),
        }


def _plan(step: int, rank_packs: list[list[int]], packs: list[Pack], step_cost: float | None = None) -> StepPlan:
    ids = [i for r in rank_packs for i in r]
    return StepPlan(
        step=step,
        rank_packs=rank_packs,
        step_tokens=sum(packs[i].tokens for i in ids),
        step_compute_tokens=sum(packs[i].compute_tokens for i in ids),
        step_cost=step_cost if step_cost is not None else sum(packs[i].cost for i in ids),
        rank_costs=[sum(packs[i].cost for i in r) for r in rank_packs],
    )


def _assign_ranks(
    pack_ids: list[int],
    packs: list[Pack],
    world_size: int,
    grad_accum: int,
    global_costs: list[float],
) -> tuple[list[list[int]], list[float]]:
    """Greedy min-max list scheduling with ``grad_accum`` slots per rank."""
    slots: list[list[int]] = [[] for _ in range(world_size)]
    load = [0.0] * world_size
    for pid in sorted(pack_ids, key=lambda i: packs[i].cost, reverse=True):
        open_ranks = [r for r in range(world_size) if len(slots[r]) < grad_accum]
        if not open_ranks:
            raise RuntimeError("rank assignment failed; step does not have W*A slots")
        r = min(open_ranks, key=lambda q: (global_costs[q] + load[q], load[q], q))
        slots[r].append(pid)
        load[r] += packs[pid].cost
    return slots, load


def build_schedule(
    packs: list[Pack],
    world_size: int,
    grad_accum: int,
    *,
    seed: int = 0,
    mode: str = "balanced",
) -> Schedule:
    if world_size < 1 or grad_accum < 1:
        raise ValueError("world_size and grad_accum must be >= 1")
    slots_per_step = world_size * grad_accum
    n_steps = len(packs) // slots_per_step
    if n_steps == 0:
        raise ValueError(
            f"not enough packs ({len(packs)}) for W*A={slots_per_step}; reduce grad_accum or add data"
        )
    rng = np.random.default_rng(seed)
    chosen = [int(i) for i in rng.permutation(len(packs))[: n_steps * slots_per_step]]

    if mode == "random":
        rng.shuffle(chosen)
        plans = []
        for s in range(n_steps):
            group = chosen[s * slots_per_step : (s + 1) * slots_per_step]
            rank_packs = [group[r::world_size] for r in range(world_size)]
            plans.append(_plan(s, rank_packs, packs, step_cost=sum(packs[i].cost for i in group)))
        return Schedule(plans, world_size, grad_accum)
    if mode != "balanced":
        raise ValueError(f"unknown schedule mode {mode}")

    by_cost = sorted(chosen, key=lambda i: (-packs[i].cost, rng.random()))
    members: list[list[int]] = [[] for _ in range(n_steps)]
    totals = [0.0] * n_steps
    frontier = [(0.0, s) for s in range(n_steps)]
    heapq.heapify(frontier)
    for pid in by_cost:
        if not frontier:
            raise RuntimeError("step assignment failed")
        _, s = heapq.heappop(frontier)
        members[s].append(pid)
        totals[s] += packs[pid].cost
        if len(members[s]) < slots_per_step:
            heapq.heappush(frontier, (totals[s], s))

    plans = []
    epoch_load = [0.0] * world_size
    for s, ids in enumerate(members):
        rank_packs, load = _assign_ranks(ids, packs, world_size, grad_accum, epoch_load)
        for r in range(world_size):
            epoch_load[r] += load[r]
        plan = _plan(s, rank_packs, packs, step_cost=totals[s])
        plan.rank_costs = load
        plans.append(plan)

    order = rng.permutation(len(plans))
    plans = [plans[int(i)] for i in order]
    for i, p in enumerate(plans):
        p.step = i
    return Schedule(plans, world_size, grad_accum)


def schedule_cost_curve(schedule: Schedule) -> list[float]:
    return [p.step_cost for p in schedule.steps]
