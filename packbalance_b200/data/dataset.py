"""Pack metadata -> model-ready tensors, and the per-rank loader.

Batch dict of one pack (reference ``data/dataset.py:67-76``): ``input_ids``,
``labels`` (next token inside each document; the last token of a document and all
padding are -100), ``position_ids`` (restart at 0 per document), ``doc_ids``
(segment index, padding -1; a padded pack is flattened to ``rows * seq_len`` tokens
and every slot of row ``r`` has doc id ``r``), ``pack_id``, ``useful_tokens``,
``compute_tokens``, ``cost``.  One key is added: ``doc_start`` (int32), the index of
the first token of the attention document that contains each token; the sm100
attention kernel masks with it (``doc_start[q] <= k <= q``) instead of a block mask.

:func:`concat_packs` joins a rank's ``grad_accum`` packs into one token stream with
globally unique document ids, which is how the trainer runs the microbatches of a
step as one forward/backward.
"""

from __future__ import annotations

from collections.abc import Iterator
from typing import Any

import numpy as np
import torch
from torch.utils.data import DataLoader, Dataset, Sampler

from packbalance_b200.config import DataConfig
from packbalance_b200.data.packer import Pack
from packbalance_b200.data.store import TokenStore


def doc_starts_from_ids(doc_ids: np.ndarray) -> np.ndarray:
    """First index of the run of equal ``doc_ids`` containing each position."""
    n = doc_ids.shape[0]
    if n == 0:
        return np.zeros(0, dtype=np.int32)
    new_run = np.ones(n, dtype=bool)
    new_run[1:] = doc_ids[1:] != doc_ids[:-1]
    starts = np.where(new_run, np.arange(n), 0)
    return np.maximum.accumulate(starts).astype(np.int32)


class PackedDataset(Dataset):
    def __init__(self, store: TokenStore, packs: list[Pack], cfg: DataConfig) -> None:
        self.store = store
        self.packs = packs
        self.seq_len = cfg.seq_len
        self.pad_token_id = cfg.pad_token_id

    def __len__(self) -> int:
        return len(self.packs)

    def _fill(self, buf: dict[str, np.ndarray], at: int, seg_tokens: np.ndarray) -> int:
        n = seg_tokens.shape[0]
        buf["input_ids"][at : at + n] = seg_tokens
        if n > 1:
            buf["labels"][at : at + n - 1] = seg_tokens[1:]
        buf["position_ids"][at : at + n] = np.arange(n)
        return n

    def __getitem__(self, index: int) -> dict[str, Any]:
        pack = self.packs[index]
        padded = pack.kind == "padded"
        total = pack.rows * self.seq_len if padded else self.seq_len
        buf = {
            "input_ids": np.full(total, self.pad_token_id, dtype=np.int64),
            "labels": np.full(total, -100, dtype=np.int64),
            "position_ids": np.zeros(total, dtype=np.int64),
            "doc_ids": np.full(total, -1, dtype=np.int64),
        }
        at = 0
        for k, seg in enumerate(pack.segments):
            toks = self.store.read(seg.start, seg.length)
            if padded:
                row0 = k * self.seq_len
                self._fill(buf, row0, toks)
                buf["doc_ids"][row0 : row0 + self.seq_len] = k
            else:
                n = self._fill(buf, at, toks)
                buf["doc_ids"][at : at + n] = k
                at += n
        if not padded and at > self.seq_len:
            raise ValueError(f"pack {pack.pack_id} overflows seq_len: {at}")
        out: dict[str, Any] = {k: torch.from_numpy(v) for k, v in buf.items()}
        out["doc_start"] = torch.from_numpy(doc_starts_from_ids(buf["doc_ids"]))
        out.update(
            pack_id=pack.pack_id,
            useful_tokens=pack.tokens,
            compute_tokens=pack.compute_tokens,
            cost=pack.cost,
        )
        return out


def concat_packs(batches: list[dict[str, Any]]) -> dict[str, Any]:
    """Concatenate pack batches; document ids and ``doc_start`` stay per-document."""
    if len(batches) == 1:
        return batches[0]
    doc_ids, starts = [], []
    base_tok = 0
    base_doc = 0
    for b in batches:
        d = b["doc_ids"]
        shifted = torch.where(d >= 0, d + base_doc, d)
        doc_ids.append(shifted)
        starts.append(b["doc_start"] + base_tok)
        base_doc += int(d.max()) + 1 if d.numel() and int(d.max()) >= 0 else 0
        base_tok += d.numel()
    out: dict[str, Any] = {
        key: torch.cat([b[key] for b in batches]) for key in ("input_ids", "labels", "position_ids")
    }
    out["doc_ids"] = torch.cat(doc_ids)
    out["doc_start"] = torch.cat(starts)
    out["pack_id"] = [b.get("pack_id") for b in batches]
    for key in ("useful_tokens", "compute_tokens", "cost"):
        if all(key in b for b in batches):
            out[key] = sum(b[key] for b in batches)
    out["num_packs"] = len(batches)
    return out


class ListSampler(Sampler[int]):
    def __init__(self, indices: list[int]) -> None:
        self.indices = indices

    def __iter__(self) -> Iterator[int]:
        return iter(self.indices)

    def __len__(self) -> int:
        return len(self.indices)


def _worker_init(worker_id: int) -> None:
    np.random.seed(torch.initial_seed() % (2**32 - 1) + worker_id)


def build_dataloader(
    store: TokenStore, packs: list[Pack], cfg: DataConfig, indices: list[int]
) -> DataLoader:
    kwargs: dict[str, Any] = dict(
        dataset=PackedDataset(store, packs, cfg),
        batch_size=None,
        sampler=ListSampler(indices),
        num_workers=cfg.num_workers,
        pin_memory=cfg.pin_memory and torch.cuda.is_available(),
        persistent_workers=cfg.persistent_workers and cfg.num_workers > 0,
        worker_init_fn=_worker_init,
    )
    if cfg.num_workers > 0:
        kwargs["prefetch_factor"] = cfg.prefetch_factor
    return DataLoader(**kwargs)


def to_device(batch: dict[str, Any], device: torch.device) -> dict[str, Any]:
    return {
        k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v)
        for k, v in batch.items()
    }


def batch_tensor_bytes(batch: dict[str, Any]) -> int:
    """Bytes of the tensors a host->device copy of the batch moves (nested dicts, such as
    the attention plan, included)."""
    total = 0
    for v in batch.values():
        if isinstance(v, torch.Tensor):
            total += v.numel() * v.element_size()
        elif isinstance(v, dict):
            total += batch_tensor_bytes(v)
    return total
