import numpy as np
import torch

from packbalance_b200.config import DataConfig
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.dataset import PackedDataset, concat_packs, doc_starts_from_ids
from packbalance_b200.data.packer import build_packs
from packbalance_b200.data.store import TokenStore


def _multi_doc(packs):
    return next(p for p in packs if p.kind != "padded" and len(p.segments) >= 2)


def test_packed_example_is_well_formed(store: TokenStore, data_cfg: DataConfig, flop_model: FlopModel) -> None:
    pack = _multi_doc(build_packs(store, data_cfg, flop_model))
    item = PackedDataset(store, [pack], data_cfg)[0]
    ids, labels = item["input_ids"].numpy(), item["labels"].numpy()
    pos, docs, starts = item["position_ids"].numpy(), item["doc_ids"].numpy(), item["doc_start"].numpy()
    assert ids.shape == (data_cfg.seq_len,)
    off = 0
    for k, seg in enumerate(pack.segments):
        toks = store.read(seg.start, seg.length)
        n = seg.length
        np.testing.assert_array_equal(ids[off : off + n], toks)
        np.testing.assert_array_equal(labels[off : off + n - 1], toks[1:])
        assert labels[off + n - 1] == -100
        np.testing.assert_array_equal(pos[off : off + n], np.arange(n))
        np.testing.assert_array_equal(docs[off : off + n], k)
        np.testing.assert_array_equal(starts[off : off + n], off)
        off += n
    assert np.all(labels[off:] == -100) and np.all(docs[off:] == -1)


def test_padded_example_is_well_formed(store: TokenStore, data_cfg: DataConfig, flop_model: FlopModel) -> None:
    cfg = DataConfig(**{**data_cfg.__dict__, "mode": "pad"})
    pack = build_packs(store, cfg, flop_model)[0]
    item = PackedDataset(store, [pack], cfg)[0]
    assert item["input_ids"].shape == (cfg.seq_len * pack.rows,)
    for row, seg in enumerate(pack.segments):
        base = row * cfg.seq_len
        assert np.array_equal(item["input_ids"][base : base + seg.length].numpy(), store.read(seg.start, seg.length))
        assert item["labels"][base + seg.length - 1].item() == -100
        assert torch.all(item["doc_ids"][base : base + cfg.seq_len] == row)
        assert torch.all(item["doc_start"][base : base + cfg.seq_len] == base)


def test_doc_starts() -> None:
    np.testing.assert_array_equal(doc_starts_from_ids(np.array([0, 0, 1, 1, 1, -1, -1])), [0, 0, 2, 2, 2, 5, 5])


def test_concat_packs_keeps_documents_apart(store: TokenStore, data_cfg: DataConfig, flop_model: FlopModel) -> None:
    packs = build_packs(store, data_cfg, flop_model)[:3]
    ds = PackedDataset(store, packs, data_cfg)
    items = [ds[i] for i in range(3)]
    cat = concat_packs(items)
    s = data_cfg.seq_len
    assert cat["input_ids"].shape == (3 * s,)
    assert cat["useful_tokens"] == sum(p.tokens for p in packs)
    for i, it in enumerate(items):
        np.testing.assert_array_equal(cat["doc_start"][i * s : (i + 1) * s].numpy(), it["doc_start"].numpy() + i * s)
    real = cat["doc_ids"][cat["doc_ids"] >= 0]
    n_docs = sum(len(p.segments) for p in packs)
    assert len(torch.unique(real)) == n_docs


def test_one_token_documents_have_no_label(edge_store: TokenStore, data_cfg: DataConfig,
                                           flop_model: FlopModel) -> None:
    """A 1-token document contributes an input but no target, sits in its own
    document (its own doc_start), and does not leak attention into its neighbours."""
    cfg = DataConfig(**{**data_cfg.__dict__, "mode": "pack_ffd", "min_doc_len": 1, "val_fraction": 0.0})
    packs = build_packs(edge_store, cfg, flop_model)
    ds = PackedDataset(edge_store, packs, cfg)
    singles = 0
    for i, p in enumerate(packs):
        item = ds[i]
        starts, labels = item["doc_start"].numpy(), item["labels"].numpy()
        off = 0
        for seg in p.segments:
            if seg.length == 1:
                singles += 1
                assert labels[off] == -100 and starts[off] == off
                if off + 1 < cfg.seq_len:
                    assert starts[off + 1] == off + 1
            off += seg.length
        assert item["useful_tokens"] == p.tokens
    assert singles >= 2
