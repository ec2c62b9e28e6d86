"""Gradient bucket planning of the data-parallel engine (CPU, no process group)."""

from __future__ import annotations

from dataclasses import replace

import pytest

from packbalance_b200.config import ModelConfig
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.parallel.distributed import DataParallel
from packbalance_b200.parallel.flat import FlatParameters


def _dp(model_cfg: ModelConfig, cap_mb: float, wire: str) -> tuple[DataParallel, FlatParameters]:
    cfg = replace(model_cfg, n_layers=3)
    flat = FlatParameters(LlamaForCausalLM(cfg))
    return DataParallel(flat, bucket_cap_mb=cap_mb, wire=wire), flat


@pytest.mark.parametrize("wire", ["fp32", "bf16"])
@pytest.mark.parametrize("cap_mb", [25.0, 0.004])
def test_buckets_cover_the_buffer_backwards_with_aligned_starts(model_cfg: ModelConfig, wire: str, cap_mb: float):
    dp, flat = _dp(model_cfg, cap_mb, wire)
    assert dp.align == (8 if wire == "bf16" else 4)
    b = dp.buckets
    # contiguous, last parameters first, the whole buffer
    assert b[0][1] == flat.numel and b[-1][0] == 0
    for (lo, hi), (lo2, hi2) in zip(b, b[1:]):
        assert hi2 == lo and lo2 < hi2
    # every start but the buffer's own is a 16-byte boundary in the wire type
    assert all(lo % dp.align == 0 for lo, _ in b)
    # a decoder layer's first parameter starts a bucket (one bucket per layer at the
    # default cap; more with a cap below a layer's size)
    starts = {lo for lo, _ in b}
    for s in flat.slots:
        if s.name.endswith("input_layernorm.weight") and s.offset % dp.align == 0:
            assert s.offset in starts
    if cap_mb < 1:
        assert len(b) > 3 + 1
        cap = dp.cap
        # only buckets holding a single parameter larger than the cap exceed it
        for lo, hi in b:
            if hi - lo > cap:
                assert sum(1 for s in flat.slots if lo <= s.offset < hi) == 1


def test_tail_offset_is_the_first_layers_second_norm(model_cfg: ModelConfig):
    dp, flat = _dp(model_cfg, 25.0, "fp32")
    off = next(s.offset for s in flat.slots if s.name == "model.layers.0.post_attention_layernorm.weight")
    assert dp.tail_offset == off
    # buckets below it (the first layer's and the embedding's) go out on the wide launch
    assert any(lo < dp.tail_offset for lo, _ in dp.buckets)
