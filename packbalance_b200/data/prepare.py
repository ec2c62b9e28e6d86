"""Build a memory-mappable token corpus (synthetic or TinyStories).

Output format and meta keys follow the reference (``data/prepare.py:20-56``).  The
synthetic generator reproduces the reference corpus exactly for the reference's
knobs (same RNG stream: lengths first, then one ``integers`` draw per document, last
token overwritten by EOS, ``prepare.py:59-87``) and adds the knobs the B200
benchmark configs need: a median parametrisation, Zipf token ids, a minimum id,
appended EOS and a fraction of full-context single documents.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import numpy as np

from packbalance_b200.config import DataConfig, load_config


def write_corpus(data_dir: Path, docs: list[np.ndarray], meta: dict, token_dtype: str = "uint32") -> None:
    data_dir.mkdir(parents=True, exist_ok=True)
    lengths = np.fromiter((d.shape[0] for d in docs), dtype=np.int64, count=len(docs))
    offsets = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int64) if len(docs) else lengths
    flat = np.concatenate(docs).astype(np.dtype(token_dtype)) if docs else np.empty(0, token_dtype)
    flat.tofile(data_dir / "tokens.bin")
    np.save(data_dir / "doc_offsets.npy", offsets)
    np.save(data_dir / "doc_lengths.npy", lengths)
    full = dict(meta)
    full.update(
        num_docs=len(docs),
        num_tokens=int(lengths.sum()),
        dtype=token_dtype,
        min_doc_len=int(lengths.min()) if len(docs) else 0,
        max_doc_len=int(lengths.max()) if len(docs) else 0,
        mean_doc_len=float(lengths.mean()) if len(docs) else 0.0,
    )
    (data_dir / "meta.json").write_text(json.dumps(full, indent=2), encoding="utf-8")
    print(
        f"wrote {len(docs):,} docs / {int(lengths.sum()):,} tokens to {data_dir} "
        f"(mean length {full['mean_doc_len']:.1f})",
        flush=True,
    )


class _ZipfSampler:
    """Bounded Zipf(s) over ranks 1..n by inverse CDF (rank 1 is the most frequent)."""

    def __init__(self, n: int, s: float) -> None:
        weights = np.arange(1, n + 1, dtype=np.float64) ** (-s)
        self.cdf = np.cumsum(weights)
        self.cdf /= self.cdf[-1]

    def __call__(self, rng: np.random.Generator, size: int) -> np.ndarray:
        u = rng.random(size)
        return np.searchsorted(self.cdf, u, side="right").astype(np.int64)  # 0-based rank


def synthetic_documents(cfg: DataConfig) -> list[np.ndarray]:
    rng = np.random.default_rng(cfg.seed)
    n = cfg.synthetic_num_docs
    lengths = rng.lognormal(mean=cfg.lognormal_mu, sigma=cfg.synthetic_sigma, size=n).astype(np.int64)
    lengths = np.clip(lengths, cfg.synthetic_min_len, cfg.synthetic_max_len)
    if cfg.synthetic_long_doc_frac > 0:
        n_long = int(round(cfg.synthetic_long_doc_frac * n))
        body = cfg.seq_len - (1 if cfg.synthetic_append_eos else 0)
        lengths[rng.permutation(n)[:n_long]] = body
    vocab = int(cfg.synthetic_vocab_size)
    lo = int(cfg.synthetic_token_min)
    if not 0 <= lo < vocab:
        raise ValueError("synthetic_token_min must be in [0, synthetic_vocab_size)")
    zipf = _ZipfSampler(vocab - lo, cfg.synthetic_zipf_s) if cfg.synthetic_token_dist == "zipf" else None
    docs: list[np.ndarray] = []
    for length in lengths:
        length = int(length)
        if zipf is None:
            ids = rng.integers(lo, vocab, size=length, dtype=np.int64)
        else:
            ids = zipf(rng, length) + lo
        if cfg.synthetic_append_eos:
            ids = np.append(ids, np.int64(cfg.eos_token_id))
        else:
            ids[-1] = cfg.eos_token_id
        docs.append(ids)
    return docs


def prepare_synthetic(cfg: DataConfig, data_dir: Path) -> None:
    docs = synthetic_documents(cfg)
    meta = {
        "source": "synthetic",
        "seed": cfg.seed,
        "tokenizer": None,
        "vocab_size": int(cfg.synthetic_vocab_size),
        "eos_token_id": cfg.eos_token_id,
        "pad_token_id": cfg.pad_token_id,
        "distribution": {
            "name": "lognormal",
            "mu": cfg.lognormal_mu,
            "sigma": cfg.synthetic_sigma,
            "min": cfg.synthetic_min_len,
            "max": cfg.synthetic_max_len,
            "token_dist": cfg.synthetic_token_dist,
            "zipf_s": cfg.synthetic_zipf_s,
            "token_min": cfg.synthetic_token_min,
            "append_eos": cfg.synthetic_append_eos,
            "long_doc_frac": cfg.synthetic_long_doc_frac,
        },
    }
    write_corpus(Path(data_dir), docs, meta)


def prepare_tinystories(cfg: DataConfig, data_dir: Path, max_tokens: int | None = None) -> None:
    """Tokenise TinyStories (needs ``datasets`` + ``transformers`` and network)."""
    try:
        from datasets import load_dataset
        from transformers import AutoTokenizer
    except ImportError as exc:
        raise SystemExit("TinyStories preparation needs `datasets` and `transformers`") from exc
    tok = AutoTokenizer.from_pretrained(cfg.tokenizer, use_fast=True)
    if tok.eos_token_id is None:
        raise ValueError(f"tokenizer {cfg.tokenizer} has no eos token")
    eos = int(tok.eos_token_id)
    pad = int(tok.pad_token_id if tok.pad_token_id is not None else eos)
    stream = iter(load_dataset("roneneldan/TinyStories", split="train", streaming=True))
    docs: list[np.ndarray] = []
    total = 0
    seen = 0
    while cfg.max_docs is None or seen < cfg.max_docs:
        try:
            text = next(stream)["text"]
        except StopIteration:
            break
        seen += 1
        ids = tok(text, add_special_tokens=False)["input_ids"]
        if len(ids) < cfg.min_doc_len:
            continue
        docs.append(np.asarray(ids + [eos], dtype=np.int64))
        total += len(ids) + 1
        if max_tokens is not None and total >= max_tokens:
            break
    meta = {
        "source": "roneneldan/TinyStories",
        "seed": cfg.seed,
        "tokenizer": cfg.tokenizer,
        "vocab_size": int(tok.vocab_size),
        "eos_token_id": eos,
        "pad_token_id": pad,
    }
    write_corpus(Path(data_dir), docs, meta)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--config", required=True, help="YAML config with a data section")
    ap.add_argument("--dataset", choices=["synthetic", "tinystories"], default=None)
    ap.add_argument("--out", default=None, help="override data.data_dir")
    ap.add_argument("--max-docs", type=int, default=None)
    ap.add_argument("--max-tokens", type=int, default=None)
    args = ap.parse_args()
    cfg = load_config(args.config).data
    if args.dataset is not None:
        cfg.dataset = args.dataset
    if args.max_docs is not None:
        cfg.max_docs = args.max_docs
    out = Path(args.out or cfg.data_dir)
    if cfg.dataset == "synthetic":
        prepare_synthetic(cfg, out)
    elif cfg.dataset == "tinystories":
        prepare_tinystories(cfg, out, max_tokens=args.max_tokens)
    else:
        raise ValueError(f"unknown dataset {cfg.dataset}")


if __name__ == "__main__":
    main()
