"""Shared pytest set-up.

Markers: ``gpu`` (needs a B200 and the native extension; skipped where CUDA is
absent) and ``slow``.

Fixtures build a small model and corpus that keep the CPU suite fast but still
exercise what the packer, scheduler and kernels care about:

* GQA with a head dimension of 8 (3 query heads per KV head) and an odd vocabulary,
  so no size is a power of two by accident;
* a lognormal corpus whose tail is longer than ``max_doc_len`` (documents get split)
  and whose head reaches below the split length;
* ``edge_store``: a hand-written corpus with a 1-token document, documents of exactly
  ``seq_len`` and ``seq_len + 1`` tokens and a run of very short documents, for the
  boundary cases of packing, labels and the document-start table.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from packbalance_b200.config import DataConfig, ModelConfig
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.prepare import prepare_synthetic, write_corpus
from packbalance_b200.data.store import TokenStore

SEQ = 80        # pack length of the fixtures
VOCAB = 203     # odd on purpose


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the native extension")
    config.addinivalue_line("markers", "slow: long-running integration test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    no_gpu = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(no_gpu)


@pytest.fixture
def model_cfg() -> ModelConfig:
    """2-layer GQA decoder: d 48, 6 query heads over 2 KV heads (head_dim 8)."""
    return ModelConfig(
        vocab_size=VOCAB,
        d_model=48,
        n_layers=2,
        n_heads=6,
        n_kv_heads=2,
        d_ff=88,
        max_seq_len=SEQ,
        tie_embeddings=True,
        attention_backend="eager",
        compile_attention=False,
        use_fused_ce=False,
        ce_chunk_size=24,
    )


@pytest.fixture
def data_cfg(tmp_path: Path) -> DataConfig:
    """Lognormal corpus (median ~e^3.4 = 30 tokens) with a tail past ``max_doc_len``."""
    return DataConfig(
        dataset="synthetic",
        data_dir=str(tmp_path / "corpus"),
        seq_len=SEQ,
        mode="isoflop",
        pad_batch_size=3,
        max_doc_len=SEQ,
        min_doc_len=3,
        synthetic_num_docs=260,
        synthetic_mu=3.4,
        synthetic_sigma=0.9,
        synthetic_min_len=5,
        synthetic_max_len=170,
        synthetic_vocab_size=VOCAB,
        num_workers=0,
        prefetch_factor=1,
        val_fraction=0.15,
        seed=11,
    )


@pytest.fixture
def store(data_cfg: DataConfig) -> TokenStore:
    prepare_synthetic(data_cfg, Path(data_cfg.data_dir))
    return TokenStore.open(data_cfg.data_dir)


@pytest.fixture
def edge_store(tmp_path: Path) -> TokenStore:
    """Corpus with the boundary lengths: 1, SEQ, SEQ + 1, and a run of 2-token docs."""
    rng = np.random.default_rng(5)
    lengths = [1, SEQ, SEQ + 1, 17] + [2] * 9 + [SEQ // 2, 3 * SEQ]
    docs = [rng.integers(1, VOCAB, size=n, dtype=np.int64) for n in lengths]
    root = tmp_path / "edge_corpus"
    write_corpus(root, docs, {"source": "edge-fixture", "vocab_size": VOCAB})
    return TokenStore.open(root)


@pytest.fixture
def flop_model(model_cfg: ModelConfig) -> FlopModel:
    return FlopModel.from_config(model_cfg)
