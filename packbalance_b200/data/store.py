"""Read-only memory-mapped token corpus.

On-disk format (identical to the reference, ``data/prepare.py:20-56`` and
``data/store.py:20-43``): ``tokens.bin`` raw token ids (``meta["dtype"]``, uint32 by
default), ``doc_offsets.npy`` / ``doc_lengths.npy`` int64 arrays, ``meta.json``.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np


@dataclass
class TokenStore:
    data_dir: Path
    tokens: np.memmap
    doc_offsets: np.ndarray
    doc_lengths: np.ndarray
    meta: dict

    @classmethod
    def open(cls, data_dir: str | Path) -> TokenStore:
        root = Path(data_dir)
        meta_file = root / "meta.json"
        if not meta_file.exists():
            raise FileNotFoundError(
                f"{meta_file} not found; build the corpus first with "
                "`python -m packbalance_b200.data.prepare --config ...`"
            )
        meta = json.loads(meta_file.read_text(encoding="utf-8"))
        tokens = np.memmap(root / "tokens.bin", dtype=np.dtype(meta.get("dtype", "uint32")), mode="r")
        offsets = np.load(root / "doc_offsets.npy")
        lengths = np.load(root / "doc_lengths.npy")
        if offsets.shape != lengths.shape:
            raise ValueError("doc_offsets.npy and doc_lengths.npy disagree")
        if tokens.shape[0] != int(meta["num_tokens"]):
            raise ValueError(f"tokens.bin has {tokens.shape[0]} tokens, meta says {meta['num_tokens']}")
        return cls(root, tokens, offsets, lengths, meta)

    @property
    def num_docs(self) -> int:
        return int(self.doc_lengths.shape[0])

    @property
    def num_tokens(self) -> int:
        return int(self.tokens.shape[0])

    def read(self, start: int, length: int) -> np.ndarray:
        return np.asarray(self.tokens[start : start + length], dtype=np.int64)

    def read_many(self, starts: np.ndarray, lengths: np.ndarray) -> list[np.ndarray]:
        return [self.read(int(s), int(n)) for s, n in zip(starts, lengths, strict=False)]
