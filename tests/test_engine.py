"""The fused-microbatch step and the reference microbatch loop give the same update."""

from dataclasses import replace

import torch

from packbalance_b200.config import PackBalanceConfig, TrainConfig
from packbalance_b200.data.dataset import PackedDataset
from packbalance_b200.data.packer import build_packs
from packbalance_b200.train.engine import TrainEngine


def test_fused_microbatches_match_loop(store, data_cfg, model_cfg, flop_model) -> None:
    packs = build_packs(store, data_cfg, flop_model)[:4]
    ds = PackedDataset(store, packs, data_cfg)
    batches = [ds[i] for i in range(4)]
    tokens = sum(p.tokens for p in packs)
    base = PackBalanceConfig(model=model_cfg, data=data_cfg, train=TrainConfig(lr=1e-2, warmup_steps=1, max_steps=5,
                                                                              grad_accum=4, dtype="fp32"))
    torch.manual_seed(0)
    e1 = TrainEngine(replace(base, train=replace(base.train, fuse_microbatches=True)), torch.device("cpu"))
    torch.manual_seed(0)
    e2 = TrainEngine(replace(base, train=replace(base.train, fuse_microbatches=False)), torch.device("cpu"))
    for _ in range(2):
        o1 = e1.step(batches, tokens)
        o2 = e2.step(batches, tokens)
        torch.testing.assert_close(o1["loss_sum"], o2["loss_sum"], atol=1e-4, rtol=1e-5)
        torch.testing.assert_close(o1["grad_norm"], o2["grad_norm"], atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(e1.flat.data, e2.flat.data, atol=2e-5, rtol=1e-3)


def test_host_scalars_lagged_reads():
    from packbalance_b200.train.engine import HostScalars

    r = HostScalars(lag=2)
    got = [r.push(torch.tensor(float(i))) for i in range(5)]
    assert got == [None, None, 0.0, 1.0, 2.0]
    assert r.drain() == [3.0, 4.0]
    assert r.drain() == []
