"""Process-group setup and the data-parallel gradient engine.

``init_distributed`` follows the reference (``train/distributed.py:16-30``): NCCL when
CUDA is present, gloo otherwise, one process per GPU from torchrun's environment,
plus a configurable timeout so a dead rank ends its peers' next collective with an
error rather than a hang.

:class:`DataParallel` replaces ``torch.nn.parallel.DistributedDataParallel``.  It
owns no hooks inside autograd; gradients live in the flat buffer of
:class:`~packbalance_b200.parallel.flat.FlatParameters` and are averaged bucket by
bucket over contiguous ranges of that buffer:

* CUDA + peer memory available: the fused all-reduce kernels
  (:mod:`packbalance_b200.parallel.comm`: NVLS multimem or peer loads), which sum in
  fp32, scale by 1/W and also return the squared L2 norm of the result for gradient
  clipping;
* otherwise ``torch.distributed.all_reduce`` (NCCL on GPU, gloo on CPU).

Buckets are issued in reverse layer order as soon as the backward pass has written
the layer (``notify_ready``), on a side stream, so communication overlaps the rest
of the backward pass.
"""

from __future__ import annotations

import contextlib
import datetime
import os

import torch
import torch.distributed as dist

from packbalance_b200.parallel.flat import FlatParameters
from packbalance_b200.utils import get_local_rank, get_world_size


def init_distributed(device_override: str | None = None, timeout_s: float = 300.0) -> torch.device:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        if not dist.is_initialized():
            cuda = torch.cuda.is_available() and (device_override is None or device_override.startswith("cuda"))
            if cuda:
                torch.cuda.set_device(get_local_rank())
            dist.init_process_group(
                backend="nccl" if cuda else "gloo",
                timeout=datetime.timedelta(seconds=timeout_s),
                device_id=torch.device("cuda", get_local_rank()) if cuda else None,
            )
        if dist.get_backend() == "nccl":
            return torch.device("cuda", get_local_rank())
        return torch.device("cpu")
    if device_override is not None:
        return torch.device(device_override)
    return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")


def cleanup_distributed() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()


@contextlib.contextmanager
def no_sync(model: torch.nn.Module, enabled: bool):
    """Reference-compatible context manager; :class:`DataParallel` only reduces when
    :meth:`DataParallel.reduce` is called, so nothing needs suppressing here."""
    fn = getattr(model, "no_sync", None)
    if not enabled or fn is None:
        yield
        return
    with fn():
        yield


def unwrap_model(model: torch.nn.Module) -> torch.nn.Module:
    inner = getattr(model, "module", model)
    return getattr(inner, "_orig_mod", inner)


class DataParallel:
    """Bucketed gradient averaging over the flat gradient buffer."""

    def __init__(
        self,
        flat: FlatParameters,
        bucket_cap_mb: float = 25.0,
        backend: str = "auto",
        group: dist.ProcessGroup | None = None,
        overlap: bool | None = None,
        deterministic: bool = False,
        wire: str = "fp32",
    ) -> None:
        self.flat = flat
        self.wire = wire
        self.align = 8 if wire == "bf16" else 4  # bucket starts: 16-byte vectors of the wire type
        # deterministic mode: the peer-load kernel (sums in rank order) and a norm taken
        # afterwards in a fixed order (the fused partial norms are added atomically)
        self.deterministic = deterministic
        # Issue buckets during the backward pass (overlap) or all at once after it.
        env = os.environ.get("PB_COMM_OVERLAP")
        self.overlap = (env != "0") if overlap is None and env is not None else (True if overlap is None else overlap)
        self.group = group
        self.world = get_world_size() if dist.is_initialized() else 1
        self.cap = max(1, int(bucket_cap_mb * 1024 * 1024 // 4))
        self.buckets = self._make_buckets()
        self.fused = None
        self.stream = None
        if self.world > 1 and flat.grad.is_cuda and backend in ("auto", "fused"):
            from packbalance_b200.parallel.comm import FusedAllReduce

            try:
                self.fused = FusedAllReduce(flat.grad, group=group, flat=flat,
                                            mode="p2p" if deterministic else None, wire=wire)
                if deterministic:
                    self.fused.tail_mode = "p2p"
            except Exception as exc:  # peer memory unavailable
                if backend == "fused":
                    raise
                print(f"[comm] fused all-reduce unavailable, using NCCL: {exc}", flush=True)
        if flat.grad.is_cuda and self.world > 1:
            self.stream = torch.cuda.Stream(priority=-1)
        self._issued: list[bool] = [False] * len(self.buckets)
        self._norm_parts: list[torch.Tensor] = []
        self.hold = False  # set while a non-final microbatch runs its backward pass
        # Buckets below this offset are reduced once the backward pass has (almost) ended:
        # those of the first decoder layer (only the embedding's backward follows them) and
        # the embedding's.  They take the wide launch.
        self.tail_offset = self._tail_offset()

    def _tail_offset(self) -> int:
        for name in ("model.layers.0.post_attention_layernorm.weight", "model.layers.1.input_layernorm.weight"):
            for s in self.flat.slots:
                if s.name == name:
                    return s.offset
        return 1  # no decoder layers found: only the bucket at offset 0

    # Buckets start at a decoder layer's first parameter, so a layer's gradient goes out as
    # one bucket when its backward ends and is reduced beside the next layer's MLP GEMMs.
    # (Measured at W = 2: splitting a layer at its MLP half, reduced beside the attention
    # backward, made the step slower, 11.74 against 10.61 ms: the attention backward's
    # CTAs fill the register file and the collective's share of it.)
    READY_POINTS = ("input_layernorm.weight",)

    def _make_buckets(self) -> list[tuple[int, int]]:
        """Contiguous ranges of whole parameters, last parameters first (backward order):
        a new bucket starts at every ready point (a decoder layer's first parameter) and
        wherever a bucket would exceed the size cap.  Bucket starts are 16-byte aligned
        in the wire type (cuts only at offsets that are multiples of ``align``)."""
        buckets: list[tuple[int, int]] = []
        hi = self.flat.numel
        lo = hi
        for s in reversed(self.flat.slots):
            if hi - s.offset > self.cap and lo < hi and lo % self.align == 0:
                buckets.append((lo, hi))
                hi = lo
            lo = s.offset
            if s.name.endswith(self.READY_POINTS) and lo % self.align == 0 and lo < hi:
                buckets.append((lo, hi))
                hi = lo
        if lo < hi:
            buckets.append((lo, hi))
        return buckets

    def start_step(self) -> None:
        self._issued = [False] * len(self.buckets)
        self._norm_parts = []
        if self.fused is not None:
            self.fused.start_step()

    def notify_ready(self, offset: int, streams: tuple = ()) -> None:
        """Every gradient at flat offset >= ``offset`` is final for this step once the
        current stream and ``streams`` (e.g. the weight-gradient stream) reach this point:
        issue the buckets that lie entirely above it."""
        if self.world <= 1 or not self.overlap or self.hold:
            return
        for i, (lo, hi) in enumerate(self.buckets):
            if not self._issued[i] and lo >= offset:
                self._issue(i, streams=streams)

    def _issue(self, i: int, tail: bool = False, streams: tuple = ()) -> None:
        lo, hi = self.buckets[i]
        # Buckets of the first decoder layer and the embedding (written by the last kernels
        # of the backward pass) and buckets issued after the backward have nothing to overlap.
        tail = tail or lo < self.tail_offset
        self._issued[i] = True
        view = self.flat.grad[lo:hi]
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream())
            for st in streams:
                self.stream.wait_stream(st)
            ctx = torch.cuda.stream(self.stream)
        else:
            ctx = contextlib.nullcontext()
        with ctx:
            if self.fused is not None:
                self.fused.all_reduce_mean(lo, hi, tail=tail)
            elif self.wire == "bf16":
                # library path of the bf16 wire: the same rounding of the inputs, the sum
                # rounded once more by the library (identical on every rank)
                w = view.to(torch.bfloat16)
                dist.all_reduce(w, op=dist.ReduceOp.SUM, group=self.group)
                view.copy_(w).mul_(1.0 / self.world)
            else:
                dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.group)
                view.mul_(1.0 / self.world)

    def reduce(self) -> torch.Tensor | None:
        """Finish averaging (issuing whatever is left) and wait for it on the current
        stream.  Returns the squared global gradient norm when the fused path computed
        it, else ``None``."""
        if self.world <= 1:
            return None
        for i in range(len(self.buckets)):
            if not self._issued[i]:
                self._issue(i, tail=True)
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)
        if self.fused is not None and not self.deterministic:
            return self.fused.sumsq
        return None

    def check(self) -> None:
        """Raise if a fused all-reduce recorded a timeout (host synchronisation)."""
        if self.fused is not None:
            self.fused.check()

    def close(self) -> None:
        if self.fused is not None:
            self.fused.close()
            self.fused = None
