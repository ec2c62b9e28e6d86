"""Flat parameter / gradient / bf16-shadow buffers.

Every trainable parameter of a module becomes a view into one fp32 buffer, its
``.grad`` a view into one fp32 gradient buffer, and (on CUDA) a bf16 shadow view
feeds the tensor-core kernels.  Parameters are laid out in registration order
without padding, so the weights a fused GEMM needs side by side (q|k|v, gate|up)
are already one contiguous ``[N, K]`` matrix in every buffer.

Consequences the rest of the framework relies on:

* the optimizer is one elementwise kernel over the flat buffers (no per-tensor
  launches) and it refreshes the bf16 shadow in the same pass;
* gradient buckets for the all-reduce are contiguous ranges of the flat grad
  buffer, so a bucket needs no packing copy;
* the native backward writes weight gradients directly into the flat grad views
  (first writer of a step overwrites, later writers accumulate), so autograd's
  per-parameter accumulation never runs on the CUDA path.

State-dict keys are unchanged (the parameters are still the module's own
``nn.Parameter`` objects), which keeps the reference checkpoint format.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn


@dataclass
class Slot:
    name: str
    param: nn.Parameter
    offset: int
    numel: int
    shape: torch.Size


class GradWindow:
    """First-writer-overwrites protocol of one accumulation window.

    Kernels that produce a weight gradient call :meth:`claim` first: the first writer of
    a window overwrites the gradient memory (no zeroing pass), later writers (the second
    use of a tied weight, the next microbatch) accumulate."""

    _fresh: set[int]

    def begin_window(self) -> None:
        """New window without clearing memory (every slot is overwritten first)."""
        self._fresh.clear()

    def claim(self, *params: nn.Parameter) -> bool:
        """Return True if the caller must accumulate (an earlier writer this window)."""
        key = id(params[0])
        if key in self._fresh:
            return True
        for p in params:
            self._fresh.add(id(p))
        return False

    def backward_begin(self, *params: nn.Parameter) -> None:
        """A decoder layer's backward pass starts (``params``: its weights).  Replicated
        weights need nothing; the sharded engine prefetches the previous layer here."""

    def prezero(self, *params: nn.Parameter) -> None:
        """Zero the gradients of ``params`` that no writer has claimed yet this window, with
        one fill per contiguous run of them, and claim them: their writers then add into
        zeros.  A layer's split-K weight-gradient GEMMs (which add partial products) need
        zeroed memory; one fill per layer replaces one per GEMM."""
        slots = sorted((self.by_param[id(p)] for p in params if id(p) not in self._fresh), key=lambda s: s.offset)
        runs: list[list[int]] = []
        for s in slots:
            if runs and runs[-1][1] == s.offset:
                runs[-1][1] = s.offset + s.numel
            else:
                runs.append([s.offset, s.offset + s.numel])
        for lo, hi in runs:
            self.grad[lo:hi].zero_()
        for s in slots:
            self._fresh.add(id(s.param))


class FlatParameters(GradWindow):
    def __init__(self, module: nn.Module, *, with_shadow: bool | None = None) -> None:
        seen: set[int] = set()
        slots: list[Slot] = []
        offset = 0
        for name, p in module.named_parameters():
            if id(p) in seen or not p.requires_grad:
                continue
            seen.add(id(p))
            slots.append(Slot(name, p, offset, p.numel(), p.shape))
            offset += p.numel()
        if not slots:
            raise ValueError("module has no trainable parameters")
        self.slots = slots
        self.by_param = {id(s.param): s for s in slots}
        self.numel = offset
        first = slots[0].param
        self.device = first.device
        self.data = torch.empty(offset, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(offset, dtype=torch.float32, device=self.device)
        for s in slots:
            self.data[s.offset : s.offset + s.numel].copy_(s.param.detach().reshape(-1).float())
            s.param.data = self.data[s.offset : s.offset + s.numel].view(s.shape)
            s.param.grad = self.grad[s.offset : s.offset + s.numel].view(s.shape)
        use_shadow = self.device.type == "cuda" if with_shadow is None else with_shadow
        self.shadow = torch.empty(offset, dtype=torch.bfloat16, device=self.device) if use_shadow else None
        self._shadow_version = -1
        self._fresh: set[int] = set()
        self.ready_hook = None
        self.refresh_shadow()

    # ---- bf16 shadow --------------------------------------------------------------
    def refresh_shadow(self, force: bool = False) -> None:
        """Recast the fp32 master weights into the bf16 shadow if they changed.

        In-place updates through PyTorch bump ``data._version``; the native AdamW
        writes the shadow itself and calls :meth:`mark_shadow_fresh`.
        """
        if self.shadow is None:
            return
        if force or self._shadow_version != self.data._version:
            self.shadow.copy_(self.data)
            self._shadow_version = self.data._version

    def mark_shadow_fresh(self) -> None:
        self._shadow_version = self.data._version

    def shadow_of(self, *params: nn.Parameter) -> torch.Tensor:
        """bf16 view covering ``params`` (must be adjacent, in order) as one matrix
        ``[sum(rows), cols]``."""
        assert self.shadow is not None, "bf16 shadow only exists on CUDA"
        return self._span(self.shadow, params)

    def grad_of(self, *params: nn.Parameter) -> torch.Tensor:
        return self._span(self.grad, params)

    def _span(self, buf: torch.Tensor, params) -> torch.Tensor:
        slots = [self.by_param[id(p)] for p in params]
        for a, b in zip(slots, slots[1:], strict=False):
            if a.offset + a.numel != b.offset:
                raise ValueError(f"parameters {a.name} and {b.name} are not adjacent")
        cols = slots[0].shape[-1]
        rows = sum(s.numel for s in slots) // cols
        return buf[slots[0].offset : slots[0].offset + rows * cols].view(rows, cols)

    def slot(self, p: nn.Parameter) -> Slot:
        return self.by_param[id(p)]

    def rebind_grad(self, buf: torch.Tensor) -> None:
        """Move the flat gradient into ``buf`` (e.g. symmetric memory) and re-point every
        parameter's ``.grad`` view at it."""
        if buf.numel() != self.numel or buf.dtype != self.grad.dtype:
            raise ValueError("replacement gradient buffer has the wrong size or dtype")
        buf.copy_(self.grad)
        self.grad = buf
        for s in self.slots:
            s.param.grad = buf[s.offset : s.offset + s.numel].view(s.shape)

    # ---- gradient write protocol -----------------------------------------------
    def zero_grad(self) -> None:
        """Start a new accumulation window: the next writer of each slot overwrites."""
        self._fresh.clear()
        self.grad.zero_()

    def finish_window(self) -> None:
        """Zero the gradient of every slot no writer claimed this window (a slot that
        is not written must not keep last step's values)."""
        for s in self.slots:
            if id(s.param) not in self._fresh:
                self.grad[s.offset : s.offset + s.numel].zero_()
                self._fresh.add(id(s.param))

    def ready(self, offset: int, streams: tuple = ()) -> None:
        """Gradients at flat offsets >= ``offset`` are final for this step once the
        current stream and ``streams`` reach this point."""
        if self.ready_hook is not None:
            self.ready_hook(offset, streams)

    def ready_all(self) -> None:
        self.ready(0)

    def ready_after(self, p: nn.Parameter, streams: tuple = ()) -> None:
        """The gradients of ``p`` and of every parameter registered after it are final
        (the backward pass runs in reverse registration order)."""
        self.ready(self.slot(p).offset, streams)

    # ---- hooks the sharded layout overrides ------------------------------------
    def gather_spec(self, *params: nn.Parameter) -> list[int] | None:
        """Fused all-gather spec for the GEMM that first reads ``params`` (none here:
        every weight is local)."""
        return None

    def embedding(self, ids: torch.Tensor, weight: nn.Parameter) -> torch.Tensor:
        from packbalance_b200.ops import _native

        return _native.module().embedding_fwd(ids, weight)
