from collections import Counter

import numpy as np
import pytest

from packbalance_b200.config import DataConfig
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.packer import build_packs, pack_stats, split_documents
from packbalance_b200.data.store import TokenStore


def _covered_once(packs, cfg) -> None:
    seen: Counter = Counter()
    for p in packs:
        used = 0
        for s in p.segments:
            used += s.length
            for t in range(s.start, s.start + s.length):
                seen[(s.doc_id, t)] += 1
        assert used <= (cfg.seq_len * p.rows if p.kind == "padded" else cfg.seq_len)
    assert seen and all(v == 1 for v in seen.values())


@pytest.mark.parametrize("mode", ["pad", "pack_random", "pack_ffd", "isoflop"])
def test_packs_are_valid(store: TokenStore, flop_model: FlopModel, data_cfg: DataConfig, mode: str) -> None:
    cfg = DataConfig(**{**data_cfg.__dict__, "mode": mode})
    packs = build_packs(store, cfg, flop_model, split="train")
    _covered_once(packs, cfg)
    stats = pack_stats(packs, flop_model)
    # pad mode wastes whatever the longest row of a batch leaves; packed modes ~nothing
    assert 0.0 <= stats["padding_waste"] < (0.8 if mode == "pad" else 0.1)
    assert stats["cv"] >= 0.0
    assert [p.pack_id for p in packs] == list(range(len(packs)))


def test_document_splitting(store: TokenStore, flop_model: FlopModel, data_cfg: DataConfig) -> None:
    segs = split_documents(store, data_cfg, flop_model, np.arange(store.num_docs))
    assert segs and all(s.length <= data_cfg.max_doc_len for s in segs)
    assert all(s.length >= data_cfg.min_doc_len for s in segs)
    total = sum(s.length for s in segs)
    assert 0 < total <= int(store.doc_lengths.sum())


def test_isoflop_has_low_cost_variance(store: TokenStore, flop_model: FlopModel, data_cfg: DataConfig) -> None:
    packs = build_packs(store, DataConfig(**{**data_cfg.__dict__, "mode": "isoflop"}), flop_model)
    stats = pack_stats(packs, flop_model)
    assert stats["cv"] < 0.35 and stats["padding_waste"] < 0.05


def test_ffd_wastes_less_than_pad(store: TokenStore, flop_model: FlopModel, data_cfg: DataConfig) -> None:
    ffd = pack_stats(build_packs(store, DataConfig(**{**data_cfg.__dict__, "mode": "pack_ffd"}), flop_model), flop_model)
    pad = pack_stats(build_packs(store, DataConfig(**{**data_cfg.__dict__, "mode": "pad"}), flop_model), flop_model)
    assert ffd["padding_waste"] < pad["padding_waste"]


def test_val_split_is_disjoint(store: TokenStore, flop_model: FlopModel, data_cfg: DataConfig) -> None:
    tr = {s.doc_id for p in build_packs(store, data_cfg, flop_model, split="train") for s in p.segments}
    va = {s.doc_id for p in build_packs(store, data_cfg, flop_model, split="val") for s in p.segments}
    assert tr and va and not (tr & va)


@pytest.mark.parametrize("mode", ["pack_random", "pack_ffd", "isoflop"])
def test_boundary_lengths(edge_store: TokenStore, flop_model: FlopModel, data_cfg: DataConfig, mode: str) -> None:
    """1-token documents, documents of exactly seq_len and seq_len + 1 tokens, and one
    three packs long: every token lands in exactly one pack, long documents are cut into
    seq_len windows, and no pack overflows."""
    cfg = DataConfig(**{**data_cfg.__dict__, "mode": mode, "min_doc_len": 1, "val_fraction": 0.0})
    packs = build_packs(edge_store, cfg, flop_model, split="train")
    _covered_once(packs, cfg)
    covered = sum(s.length for p in packs for s in p.segments)
    assert covered == int(edge_store.doc_lengths.sum())
    seg_lengths = Counter(s.length for p in packs for s in p.segments)
    assert seg_lengths[cfg.seq_len] >= 1 + 1 + 3  # the SEQ doc, the SEQ+1 doc's head, the 3*SEQ doc
    assert seg_lengths[1] >= 2                      # the 1-token doc and the SEQ+1 doc's tail
