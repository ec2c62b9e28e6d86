"""Deterministic mode (``train.deterministic``): reductions in a fixed order.

Two runs of three optimizer steps on the same data give bitwise identical weights, and
they stay within the usual tolerance of the default (atomic, split-K) path.  The batch
repeats token ids (so the embedding gradient adds several rows into one) and the
gradient clip is active (so the norm enters every update)."""

import pytest
import torch

from packbalance_b200.config import ModelConfig, PackBalanceConfig, TrainConfig
from packbalance_b200.data.dataset import doc_starts_from_ids
from packbalance_b200.ops import _native
from packbalance_b200.train.engine import TrainEngine

pytestmark = pytest.mark.gpu


def _batch(t=1536, vocab=512, seed=3):
    g = torch.Generator().manual_seed(seed)
    lengths = [700, 5, 1, 300, 530]
    ids = torch.randint(1, 64, (t,), generator=g)  # few distinct ids: many repeats
    doc = torch.cat([torch.full((n,), i) for i, n in enumerate(lengths)])
    pos = torch.cat([torch.arange(n) for n in lengths])
    labels = torch.cat([ids[1:], torch.tensor([-100])])
    labels[torch.cumsum(torch.tensor(lengths), 0) - 1] = -100
    return dict(input_ids=ids, labels=labels, position_ids=pos, doc_ids=doc,
                doc_start=torch.from_numpy(doc_starts_from_ids(doc.numpy()))), int((labels != -100).sum())


def _run(deterministic: bool, steps: int = 3):
    cfg = PackBalanceConfig(
        model=ModelConfig(vocab_size=512, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=512,
                          max_seq_len=2048),
        train=TrainConfig(lr=1e-3, warmup_steps=1, max_steps=10, grad_clip=0.05, deterministic=deterministic),
    )
    torch.manual_seed(0)
    eng = TrainEngine(cfg, torch.device("cuda", 0))
    assert eng.deterministic == deterministic
    batch, tokens = _batch()
    init = {n: p.detach().float().clone() for n, p in eng.model.named_parameters()}
    norms = []
    try:
        for _ in range(steps):
            out = eng.step([batch], tokens)
            norms.append(float(out["grad_norm"]))
        torch.cuda.synchronize()
        _native.check_status()
        params = {n: p.detach().float().clone() for n, p in eng.model.named_parameters()}
    finally:
        eng.close()
    return init, params, norms


def test_deterministic_mode_is_bitwise_repeatable_and_close_to_default():
    init, a, na = _run(True)
    assert not _native.deterministic()  # closing the engine switches the mode off again
    _, b, nb = _run(True)
    assert na == nb
    for n in a:
        assert torch.equal(a[n], b[n]), n
    _, c, nc = _run(False)
    for x, y in zip(na, nc):
        assert abs(x - y) <= 2e-2 * abs(y), (na, nc)
    # Adam normalises every coordinate, so compare each parameter's update: a wrong
    # reduction gives O(1) differences, rounding order gives small ones.
    for n in a:
        upd = (c[n] - init[n]).norm().item()
        err = (a[n] - c[n]).norm().item()
        assert err <= 0.05 * max(upd, 1e-12), (n, err, upd)
