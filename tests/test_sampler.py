import pytest

from packbalance_b200.data.packer import Pack
from packbalance_b200.data.sampler import build_schedule


def _packs(costs, tokens=None):
    tokens = tokens or [10] * len(costs)
    return [Pack(pack_id=i, segments=[], tokens=tokens[i], compute_tokens=100, cost=c) for i, c in enumerate(costs)]


def test_balanced_schedule_is_complete_and_capacity_respecting() -> None:
    packs = _packs(list(range(1, 13)))
    sch = build_schedule(packs, world_size=2, grad_accum=2, seed=0, mode="balanced")
    seen = []
    for plan in sch.steps:
        assert len(plan.rank_packs) == 2 and all(len(ids) == 2 for ids in plan.rank_packs)
        for ids in plan.rank_packs:
            seen.extend(ids)
    assert sorted(seen) == list(range(len(packs)))
    assert sch.stats()["rank_cost_imbalance"] < 1e-9


def test_balanced_beats_random_on_skew() -> None:
    packs = _packs([1.0] * 24 + [50.0] * 8)
    bal = build_schedule(packs, world_size=4, grad_accum=1, seed=3, mode="balanced")
    rnd = build_schedule(packs, world_size=4, grad_accum=1, seed=3, mode="random")
    assert bal.stats()["step_cost_cv"] < rnd.stats()["step_cost_cv"]
    assert bal.stats()["step_cost_p99_over_mean"] < rnd.stats()["step_cost_p99_over_mean"]
    assert bal.stats()["rank_cost_imbalance"] <= rnd.stats()["rank_cost_imbalance"] + 1e-9


def test_rank_indices_match_plans() -> None:
    sch = build_schedule(_packs(list(range(1, 17))), world_size=2, grad_accum=2, seed=1)
    for r in range(2):
        assert sch.rank_indices(r) == [i for p in sch.steps for i in p.rank_packs[r]]


def test_schedule_is_deterministic() -> None:
    packs = _packs([float(i % 7 + 1) for i in range(40)])
    a = build_schedule(packs, world_size=4, grad_accum=2, seed=5)
    b = build_schedule(packs, world_size=4, grad_accum=2, seed=5)
    assert [p.rank_packs for p in a.steps] == [p.rank_packs for p in b.steps]


def test_too_few_packs_raises() -> None:
    with pytest.raises(ValueError):
        build_schedule(_packs([1.0, 2.0]), world_size=2, grad_accum=2)
