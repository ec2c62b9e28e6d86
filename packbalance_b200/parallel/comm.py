"""Fused gradient all-reduce over NVSwitch peer memory.

:class:`FusedAllReduce` moves the flat fp32 gradient buffer of
:class:`~packbalance_b200.parallel.flat.FlatParameters` into symmetric memory
(``torch.distributed._symmetric_memory``: one allocation per rank, mapped into every
peer) and averages contiguous ranges (buckets) of it with native kernels
(``csrc/comm.cu``):

* ``nvls_allreduce`` when the driver binds an NVLink multicast object over the
  buffers: ``multimem.ld_reduce`` (the NVSwitch sums the ranks' values) and
  ``multimem.st`` (the switch writes the result into every rank), the 1/W scale and the
  squared norm fused in;
* ``fused_allreduce`` otherwise: two-shot reduce-scatter / all-gather with peer loads.

Both synchronise through per-CTA flags in a symmetric sync buffer (release/acquire at
system scope, bounded waits).  Barrier epochs come from a device counter bumped once
per step (:meth:`start_step`) plus the launch's index within the step, so a captured
CUDA graph replays with fresh epochs.  The kernels use small CTAs that fit beside the
backward pass's GEMM and attention CTAs on the same SMs.  The rendezvous and the
process group come from ``torch.distributed`` (NCCL); the data never goes through NCCL.

The squared norm of the averaged gradient accumulates in a device scalar across the
buckets of a step, which gives gradient clipping its global norm without a separate
reduction pass or a scalar all-reduce.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from packbalance_b200.ops import _native


class FusedAllReduce:
    """``mode``: "nvls" (multimem through the NVSwitch; default when the multicast
    object is available), "p2p" (two-shot over peer loads) or "auto"."""

    # Launch widths (CTAs of 128 threads, csrc/comm_common.cuh).  A bucket reduced while
    # the backward pass still runs gets a narrow launch: a collective with a CTA on every
    # SM keeps the ~225 KB GEMM and attention CTAs from being scheduled until it ends
    # (measured: a GEMM beside 148 resident collective CTAs waits for them, beside 16 it
    # runs at full speed), and a few dozen CTAs with eight loads in flight per thread move
    # a bucket well within one layer's backward.  A bucket with nothing left to overlap
    # (the last one of the step) gets the whole GPU.
    CTAS_OVERLAP = 40  # measured at W = 2: 16 -> 11.94, 24 -> 10.62, 40 -> 10.52 ms per step
    CTAS_TAIL = 4 * 148
    SYNC_WORDS = 16384

    def __init__(self, grad: torch.Tensor, group: dist.ProcessGroup | None = None, flat=None, mode: str | None = None,
                 wire: str = "fp32") -> None:
        import os

        import torch.distributed._symmetric_memory as symm_mem

        if not grad.is_cuda or grad.dtype != torch.float32:
            raise ValueError("fused all-reduce needs an fp32 CUDA gradient buffer")
        self.group = group if group is not None else dist.group.WORLD
        n = grad.numel()
        # 16 trailing floats: the step's squared-norm accumulator (written via multicast).
        full = symm_mem.empty(n + 16, dtype=torch.float32, device=grad.device)
        full.zero_()
        self.handle = symm_mem.rendezvous(full, self.group)
        self.full = full
        # per-CTA barrier slots: a symmetric buffer of our own (the default signal pad
        # is too small for one CTA per SM at W = 8)
        self.sync = symm_mem.empty(self.SYNC_WORDS, dtype=torch.int32, device=grad.device)
        self.sync.zero_()
        self.h_sync = symm_mem.rendezvous(self.sync, self.group)
        buf = full[:n]
        buf.copy_(grad)
        self.buf = buf
        self.rank = self.handle.rank
        self.world = self.handle.world_size
        if not 2 <= self.world <= 8:
            raise RuntimeError("fused all-reduce covers 2..8 ranks of one node")
        self.pad_words = self.SYNC_WORDS
        cap = self.pad_words // (3 * self.world)
        self.ctas = min(int(os.environ.get("PB_COMM_CTAS", self.CTAS_OVERLAP)), cap)
        self.ctas_tail = min(self.CTAS_TAIL, cap)
        if self.ctas < 1:
            raise RuntimeError("signal pad too small for the fused all-reduce")
        # Barrier epochs: a device base bumped by EPOCH_STRIDE at every step start plus the
        # launch's index within the step, so a captured graph replays with fresh epochs.
        self.epoch_base = torch.zeros(1, dtype=torch.int32, device=grad.device)
        self._k = 0
        mode = mode or os.environ.get("PB_ALLREDUCE", "auto")
        if int(getattr(self.handle, "offset", 0)) != 0:
            raise RuntimeError("symmetric buffer must start at its allocation base")
        mc = int(self.handle.multicast_ptr or 0)
        self.mode = "nvls" if mode in ("auto", "nvls") and mc else "p2p"
        if mode == "nvls" and self.mode != "nvls":
            raise RuntimeError("NVLink multicast is not available for this group")
        self.mc = mc
        # Tail buckets (nothing left to overlap) take the faster kernel for the width: at two
        # ranks the two-shot peer-load kernel moves less over NVLink than multimem (each GPU
        # also reads its own copy through the switch) and measured faster (98 MB: 0.24 vs
        # 0.31 ms); from four ranks on, the in-switch reduction moves less.
        tail_env = os.environ.get("PB_ALLREDUCE_TAIL")
        self.tail_mode = tail_env if tail_env in ("p2p", "nvls") else ("p2p" if self.world == 2 else self.mode)
        if self.tail_mode == "nvls" and not mc:
            self.tail_mode = "p2p"
        # one norm accumulator for both kernels: in the symmetric buffer, where the multimem
        # kernel adds every rank's part and the peer-load kernel adds the whole bucket's
        self.sumsq = full[n]
        # bf16 wire: a symmetric bf16 copy of the gradient crosses NVLink instead of the
        # fp32 values (the two-shot kernel; sums in fp32, result rounded to bf16 on every
        # rank alike); bucket starts must then be multiples of 8 elements.
        if wire not in ("fp32", "bf16"):
            raise ValueError("wire must be fp32 or bf16")
        self.wire = wire
        self.h_wire = None
        if wire == "bf16":
            self.wire_buf = symm_mem.empty(n + 8, dtype=torch.bfloat16, device=grad.device)
            self.h_wire = symm_mem.rendezvous(self.wire_buf, self.group)
            self.mode = self.tail_mode = "p2p"
        if flat is not None:
            flat.rebind_grad(buf)
        _native.module().fused_allreduce  # fail loudly if the extension lacks the kernel

    @property
    def align(self) -> int:
        """Required multiple (in elements) of a bucket's start."""
        return 8 if self.wire == "bf16" else 4

    EPOCH_STRIDE = 64  # launches per step, at most

    def start_step(self) -> None:
        """Stream-ordered start of a step's reductions (zero the norm, new epoch base)."""
        self.sumsq.zero_()
        _native.module().epoch_bump(self.epoch_base, self.EPOCH_STRIDE)
        self._k = 0

    def all_reduce_mean(self, lo: int, hi: int, tail: bool = False) -> torch.Tensor:
        """Average elements [lo, hi) of the gradient over all ranks (current stream).
        ``tail``: nothing else runs meanwhile, launch over the whole GPU (every rank must
        pass the same value for the same bucket)."""
        ctas = self.ctas_tail if tail else self.ctas
        mode = self.tail_mode if tail else self.mode
        self._k += 1
        if self._k >= self.EPOCH_STRIDE:
            raise RuntimeError("more all-reduce launches in one step than the epoch stride allows")
        C = _native.module()
        base = self.epoch_base.data_ptr()
        if self.wire == "bf16":
            C.fused_allreduce_bf16(
                self.handle.buffer_ptrs_dev, self.h_wire.buffer_ptrs_dev, self.h_sync.buffer_ptrs_dev, self.pad_words,
                lo, hi, self.rank, self.world, self._k, 1.0 / self.world, self.sumsq, ctas, base,
            )
        elif mode == "nvls":
            n = self.buf.numel()
            C.nvls_allreduce(
                self.handle.buffer_ptrs_dev, self.h_sync.buffer_ptrs_dev, self.pad_words, self.mc,
                self.mc + 4 * n, lo, hi, self.rank, self.world, self._k, 1.0 / self.world, self.sumsq, ctas, base,
            )
        else:
            C.fused_allreduce(
                self.handle.buffer_ptrs_dev, self.h_sync.buffer_ptrs_dev, self.pad_words, lo, hi, self.rank,
                self.world, self._k, 1.0 / self.world, self.sumsq, ctas, base,
            )
        return self.sumsq

    def check(self) -> None:
        _native.check_status(self.buf.device)

    def close(self) -> None:
        self.handle = None
        self.h_sync = None
        self.h_wire = None
