"""Fused gradient all-reduce over NVSwitch peer memory.

:class:`FusedAllReduce` moves the flat fp32 gradient buffer of
:class:`~packbalance_b200.parallel.flat.FlatParameters` into symmetric memory
(``torch.distributed._symmetric_memory``: one allocation per rank, mapped into every
peer, plus a per-rank signal pad) and averages contiguous ranges of it with the native
``fused_allreduce`` kernel (``csrc/comm.cu``): reduce-scatter with the 1/W scale and the
squared-norm partial fused in, then all-gather, synchronised by per-CTA flags in the
peers' signal pads with bounded waits.  The rendezvous and the process group come from
``torch.distributed`` (NCCL); the data never goes through NCCL.

The squared norm of the averaged gradient accumulates in a device scalar across the
buckets of a step, which gives gradient clipping its global norm without a separate
reduction pass or a scalar all-reduce.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from packbalance_b200.ops import _native


class FusedAllReduce:
    CTAS = 32

    def __init__(self, grad: torch.Tensor, group: dist.ProcessGroup | None = None, flat=None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        if not grad.is_cuda or grad.dtype != torch.float32:
            raise ValueError("fused all-reduce needs an fp32 CUDA gradient buffer")
        self.group = group if group is not None else dist.group.WORLD
        buf = symm_mem.empty(grad.numel(), dtype=torch.float32, device=grad.device)
        buf.copy_(grad)
        self.handle = symm_mem.rendezvous(buf, self.group)
        self.buf = buf
        self.rank = self.handle.rank
        self.world = self.handle.world_size
        self.pad_words = self.handle.signal_pad_size // 4
        self.ctas = min(self.CTAS, self.pad_words // (3 * self.world))
        if self.ctas < 1:
            raise RuntimeError("signal pad too small for the fused all-reduce")
        self.epoch = 0
        self.sumsq = torch.zeros((), device=grad.device, dtype=torch.float32)
        if flat is not None:
            flat.rebind_grad(buf)
        _native.module().fused_allreduce  # fail loudly if the extension lacks the kernel

    def start_step(self) -> None:
        self.sumsq.zero_()

    def all_reduce_mean(self, lo: int, hi: int) -> torch.Tensor:
        """Average elements [lo, hi) of the gradient over all ranks (current stream)."""
        self.epoch += 1
        _native.module().fused_allreduce(
            self.handle.buffer_ptrs_dev, self.handle.signal_pad_ptrs_dev, self.pad_words, lo, hi, self.rank,
            self.world, self.epoch, 1.0 / self.world, self.sumsq, self.ctas,
        )
        return self.sumsq

    def check(self) -> None:
        _native.check_status(self.buf.device)

    def close(self) -> None:
        self.handle = None
