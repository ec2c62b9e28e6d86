"""Document splitting and the four packing modes.

The packer decides which documents share a sequence; the scheduler
(:mod:`packbalance_b200.data.sampler`) decides which sequences share a step and a
rank.  Modes (reference ``data/packer.py:256-318``):

* ``pad``         random groups of ``pad_batch_size`` documents, one padded row each;
* ``pack_random`` best-fit bin packing in a seeded random order;
* ``pack_ffd``    best-fit decreasing by length;
* ``isoflop``     cost-aware: each segment, most expensive first, goes to the
                  cheapest pack that still has room, then a few local moves from the
                  most to the least expensive pack.

The selection rules (best-fit tie order, cheapest-bin choice, rebalance move rule,
RNG call order) are kept identical to the reference so both frameworks build the
same packs from the same corpus; the data structures are this module's own.
"""

from __future__ import annotations

import bisect
import heapq
import itertools
from dataclasses import dataclass

import numpy as np

from packbalance_b200.config import DataConfig
from packbalance_b200.data.cost import FlopModel, cost_stats
from packbalance_b200.data.store import TokenStore


@dataclass(frozen=True)
class Segment:
    doc_id: int
    start: int
    length: int
    cost: float


@dataclass
class Pack:
    pack_id: int
    segments: list[Segment]
    tokens: int
    compute_tokens: int
    cost: float
    kind: str = "packed"
    rows: int = 1

    @property
    def useful_tokens(self) -> int:
        return self.tokens

    @property
    def utilization(self) -> float:
        return self.tokens / self.compute_tokens if self.compute_tokens else 0.0

    @property
    def lengths(self) -> list[int]:
        return [s.length for s in self.segments]


def split_documents(
    store: TokenStore, cfg: DataConfig, flop_model: FlopModel, doc_ids: np.ndarray
) -> list[Segment]:
    """Cut documents into windows of at most ``min(max_doc_len, seq_len)`` tokens.

    Each window becomes its own attention document.  Windows (or whole documents)
    shorter than ``min_doc_len`` are dropped.
    """
    window = min(cfg.max_doc_len, cfg.seq_len)
    out: list[Segment] = []
    offsets = store.doc_offsets
    lengths = store.doc_lengths
    for raw in doc_ids:
        doc = int(raw)
        base = int(offsets[doc])
        total = int(lengths[doc])
        for lo in range(0, total, window):
            n = min(window, total - lo)
            if n >= cfg.min_doc_len:
                out.append(Segment(doc, base + lo, n, float(flop_model.doc_cost(n))))
    if not out:
        raise ValueError("no usable documents after filtering; lower min_doc_len")
    return out


def _as_packs(bins: list[list[Segment]], seq_len: int) -> list[Pack]:
    packs = []
    for i, segs in enumerate(bins):
        packs.append(
            Pack(
                pack_id=i,
                segments=segs,
                tokens=sum(s.length for s in segs),
                compute_tokens=seq_len,
                cost=float(sum(s.cost for s in segs)),
            )
        )
    return packs


def _pack_best_fit(
    segments: list[Segment],
    seq_len: int,
    flop_model: FlopModel,
    *,
    order: str = "length",
    seed: int = 0,
) -> list[Pack]:
    """Best-fit: each segment goes to the open bin with the least room that fits it.

    Open bins are kept in a list sorted by ``(room, -stamp)`` where ``stamp`` is the
    time the bin's room last changed, so among equally tight bins the most recently
    touched one wins.
    """
    if order == "length":
        seq = sorted(segments, key=lambda s: (-s.length, s.doc_id))
    elif order == "cost":
        seq = sorted(segments, key=lambda s: (-s.cost, -s.length, s.doc_id))
    elif order == "random":
        perm = np.random.default_rng(seed).permutation(len(segments))
        seq = [segments[int(i)] for i in perm]
    else:
        raise ValueError(f"unknown pack order {order}")

    bins: list[list[Segment]] = []
    open_bins: list[tuple[int, int, int]] = []  # (room, -stamp, bin index), ascending
    clock = itertools.count()
    for seg in seq:
        pos = bisect.bisect_left(open_bins, (seg.length, -(1 << 62), -1))
        if pos == len(open_bins):
            idx = len(bins)
            bins.append([seg])
            room = seq_len - seg.length
        else:
            room, _, idx = open_bins.pop(pos)
            bins[idx].append(seg)
            room -= seg.length
        bisect.insort(open_bins, (room, -next(clock), idx))
    return _as_packs(bins, seq_len)


def _pack_cost_aware(segments: list[Segment], seq_len: int, flop_model: FlopModel) -> list[Pack]:
    """Most expensive segment first, into the cheapest pack (by summed cost, ties by
    pack index) that still has room; a new pack when none has room."""
    seq = sorted(segments, key=lambda s: (-s.cost, -s.length, s.doc_id))
    if seq and seq[0].length > seq_len:
        raise ValueError(f"segment length {seq[0].length} exceeds seq_len {seq_len}")
    shortest = min(s.length for s in seq)
    bins: list[list[Segment]] = []
    used: list[int] = []
    cost: list[float] = []
    heap: list[tuple[float, int]] = []
    for seg in seq:
        if seg.length > seq_len:
            raise ValueError(f"segment length {seg.length} exceeds seq_len {seq_len}")
        skipped: list[tuple[float, int]] = []
        target = -1
        while heap:
            item = heapq.heappop(heap)
            if used[item[1]] + seg.length <= seq_len:
                target = item[1]
                break
            # A pack with less room than the shortest segment can never be chosen
            # again, so it leaves the candidate set for good.
            if seq_len - used[item[1]] >= shortest:
                skipped.append(item)
        for item in skipped:
            heapq.heappush(heap, item)
        if target < 0:
            target = len(bins)
            bins.append([])
            used.append(0)
            cost.append(0.0)
        bins[target].append(seg)
        used[target] += seg.length
        cost[target] += seg.cost
        heapq.heappush(heap, (cost[target], target))
    return _as_packs(bins, seq_len)


def _rebalance_packs(packs: list[Pack], seq_len: int, iterations: int) -> list[Pack]:
    """Up to ``iterations`` moves: one segment from the most expensive pack to the
    cheapest, choosing the fitting segment that leaves the smallest cost gap."""
    if len(packs) < 2:
        return packs
    for _ in range(max(0, iterations)):
        ranked = sorted(range(len(packs)), key=lambda i: packs[i].cost, reverse=True)
        hi, lo = packs[ranked[0]], packs[ranked[-1]]
        if hi.cost - lo.cost <= 1e-9:
            break
        pick = None
        pick_gap = 0.0
        for seg in hi.segments:
            if lo.tokens + seg.length > seq_len:
                continue
            new_hi, new_lo = hi.cost - seg.cost, lo.cost + seg.cost
            helps = max(new_hi, new_lo) < max(hi.cost, lo.cost) or (
                new_hi - new_lo < hi.cost - lo.cost
            )
            if not helps:
                continue
            gap = abs(new_hi - new_lo)
            if pick is None or gap < pick_gap:
                pick, pick_gap = seg, gap
        if pick is None:
            break
        hi.segments.remove(pick)
        lo.segments.append(pick)
        hi.tokens -= pick.length
        lo.tokens += pick.length
        hi.cost -= pick.cost
        lo.cost += pick.cost
    return packs


def _renumber(packs: list[Pack]) -> list[Pack]:
    for i, p in enumerate(packs):
        p.pack_id = i
    return packs


def _split_doc_ids(n: int, cfg: DataConfig, split: str) -> np.ndarray:
    if not 0.0 <= cfg.val_fraction < 1.0:
        raise ValueError("val_fraction must be in [0, 1)")
    n_val = int(round(n * cfg.val_fraction))
    cut = max(0, n - n_val)
    ids = np.arange(cut, n, dtype=np.int64) if split == "val" else np.arange(0, cut, dtype=np.int64)
    if ids.size == 0:
        raise ValueError(f"empty {split} split (docs={n}, val_fraction={cfg.val_fraction})")
    if cfg.max_docs is not None:
        ids = ids[: cfg.max_docs]
    return ids


def build_packs(
    store: TokenStore, cfg: DataConfig, flop_model: FlopModel, *, split: str = "train"
) -> list[Pack]:
    """Split documents of ``split`` and pack them with ``cfg.mode``."""
    segments = split_documents(store, cfg, flop_model, _split_doc_ids(store.num_docs, cfg, split))
    rng = np.random.default_rng(cfg.seed + (0 if split == "train" else 1))
    if cfg.mode == "pad":
        order = rng.permutation(len(segments))
        packs = []
        for k, lo in enumerate(range(0, len(segments), cfg.pad_batch_size)):
            segs = [segments[int(i)] for i in order[lo : lo + cfg.pad_batch_size]]
            lens = [s.length for s in segs]
            packs.append(
                Pack(
                    pack_id=k,
                    segments=segs,
                    tokens=int(sum(lens)),
                    compute_tokens=cfg.seq_len * len(segs),
                    cost=flop_model.padded_batch_cost(lens, cfg.seq_len),
                    kind="padded",
                    rows=len(segs),
                )
            )
    elif cfg.mode == "pack_random":
        packs = _pack_best_fit(segments, cfg.seq_len, flop_model, order="random", seed=cfg.seed)
    elif cfg.mode == "pack_ffd":
        packs = _pack_best_fit(segments, cfg.seq_len, flop_model, order="length")
    elif cfg.mode == "isoflop":
        packs = _pack_cost_aware(segments, cfg.seq_len, flop_model)
        packs = _rebalance_packs(packs, cfg.seq_len, cfg.isoflop_iterations)
    else:
        raise ValueError(f"unknown packing mode {cfg.mode}")
    packs = _renumber(packs)
    if split == "train":
        perm = rng.permutation(len(packs))
        packs = _renumber([packs[int(i)] for i in perm])
    return packs


def pack_stats(packs: list[Pack], flop_model: FlopModel) -> dict[str, float]:
    useful = sum(p.useful_tokens for p in packs)
    compute = sum(p.compute_tokens for p in packs)
    docs = sum(len(p.segments) for p in packs)
    stats = cost_stats([p.cost for p in packs])
    stats.update(
        num_packs=len(packs),
        num_docs=docs,
        useful_tokens=useful,
        compute_tokens=compute,
        padding_waste=1.0 - useful / compute if compute else 0.0,
        mean_docs_per_pack=docs / len(packs) if packs else 0.0,
        mean_utilization=float(np.mean([p.utilization for p in packs])) if packs else 0.0,
    )
    return stats
