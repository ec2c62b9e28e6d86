"""Lagged step timing of the trainer: each record comes back exactly once, one step
after it was launched, in step order, with the device scalars it was given."""

import torch

from packbalance_b200.train.train import LaggedSteps


def test_records_resolve_one_step_late_in_order():
    lag = LaggedSteps(cuda=False)
    seen = []
    for i in range(5):
        lag.begin()
        scal = {"loss": torch.tensor(float(i) + 0.5)} if i % 2 == 0 else None
        out = lag.launched({"step": i, "log": i % 2 == 0}, scal)
        if i == 0:
            assert out == []
        else:
            assert [r["step"] for r in out] == [i - 1]
        seen += out
    seen += lag.drain()
    assert [r["step"] for r in seen] == list(range(5))
    assert lag.drain() == []
    for r in seen:
        assert r["step_ms"] >= 0.0
        if r["log"]:
            assert r["loss"] == r["step"] + 0.5
        else:
            assert "loss" not in r


def test_lag_two_keeps_two_in_flight():
    lag = LaggedSteps(cuda=False, lag=2)
    got = []
    for i in range(4):
        lag.begin()
        got.append([r["step"] for r in lag.launched({"step": i, "log": False})])
    assert got == [[], [], [0], [1]]
    assert [r["step"] for r in lag.drain()] == [2, 3]
