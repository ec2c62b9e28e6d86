"""AdamW over the flat parameter buffer, with gradient clipping folded in.

Math is ``torch.optim.AdamW`` (decoupled weight decay on every parameter, as the
reference's single param group does, ``train/train.py:58-69``).  On CUDA one native
kernel updates the fp32 master weights, both moments and the bf16 shadow in a
single pass, scaling the gradient by ``min(1, max_norm / (norm + 1e-6))`` read from
device memory, and skipping the update when the norm is not finite.  On CPU the
same math runs as torch ops over the flat buffers.

``state_dict()`` has the ``torch.optim.AdamW`` layout (per-parameter ``step``,
``exp_avg``, ``exp_avg_sq``; ``param_groups`` with ``initial_lr`` once an LR scheduler
is attached) so checkpoints load in either framework.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from packbalance_b200.parallel.flat import FlatParameters


class FlatAdamW(torch.optim.Optimizer):
    def __init__(
        self,
        flat: FlatParameters,
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
    ) -> None:
        params = [s.param for s in flat.slots]
        defaults = dict(
            lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=False,
            maximize=False, foreach=None, capturable=False, differentiable=False, fused=None,
        )
        super().__init__(params, defaults)
        self.flat = flat
        self.exp_avg = torch.zeros_like(flat.data)
        self.exp_avg_sq = torch.zeros_like(flat.data)
        self.step_count = 0
        self.last_skipped = torch.zeros((), dtype=torch.int32, device=flat.device)
        self._bind_state()

    def _bind_state(self) -> None:
        # one shared CPU scalar for every parameter's "step" entry, updated in place
        self._step_t = torch.tensor(float(self.step_count))
        for s in self.flat.slots:
            self.state[s.param] = {
                "step": self._step_t,
                "exp_avg": self.exp_avg[s.offset : s.offset + s.numel].view(s.shape),
                "exp_avg_sq": self.exp_avg_sq[s.offset : s.offset + s.numel].view(s.shape),
            }

    def load_state_dict(self, state_dict: dict[str, Any]) -> None:
        groups = state_dict["param_groups"]
        if len(groups) != 1:
            raise ValueError("FlatAdamW expects a single parameter group")
        saved_ids = groups[0]["params"]
        if len(saved_ids) != len(self.flat.slots):
            raise ValueError(f"optimizer state has {len(saved_ids)} params, model has {len(self.flat.slots)}")
        for key, value in groups[0].items():
            if key != "params":
                self.param_groups[0][key] = value
        steps = []
        for pid, s in zip(saved_ids, self.flat.slots, strict=True):
            st = state_dict["state"].get(pid)
            if st is None:
                continue
            self.exp_avg[s.offset : s.offset + s.numel].copy_(st["exp_avg"].reshape(-1))
            self.exp_avg_sq[s.offset : s.offset + s.numel].copy_(st["exp_avg_sq"].reshape(-1))
            steps.append(float(st["step"]))
        self.step_count = int(max(steps)) if steps else 0
        self._bind_state()

    @torch.no_grad()
    def step(self, closure=None, grad_norm: torch.Tensor | None = None, max_norm: float = 0.0,
             hparams: torch.Tensor | None = None):
        """One update.  ``grad_norm`` (device scalar) enables clipping to ``max_norm``
        and the non-finite skip; without it gradients are used as they are.  ``hparams``
        (CUDA, fp32 [3]): lr and the two bias corrections read on the device, for
        captured CUDA graphs (the caller keeps them current)."""
        loss = closure() if closure is not None else None
        group = self.param_groups[0]
        lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
        self.step_count += 1
        t = self.step_count
        bc1 = 1.0 - b1**t
        bc2 = 1.0 - b2**t
        flat = self.flat
        if flat.data.is_cuda:
            from packbalance_b200.ops import _native

            norm = grad_norm if grad_norm is not None else torch.zeros((), device=flat.device)
            _native.module().adamw_step(
                flat.data, flat.grad, self.exp_avg, self.exp_avg_sq,
                flat.shadow if flat.shadow is not None else flat.data,
                norm, self.last_skipped,
                float(lr), float(b1), float(b2), float(eps), float(wd),
                float(bc1), float(bc2), float(max_norm if grad_norm is not None else 0.0),
                flat.shadow is not None, hparams,
            )
            flat.mark_shadow_fresh()
        else:
            g = flat.grad
            if grad_norm is not None:
                if not torch.isfinite(grad_norm):
                    self.last_skipped.fill_(1)
                    self.step_count -= 1
                    return loss
                if max_norm > 0:
                    coef = min(1.0, max_norm / (float(grad_norm) + 1e-6))
                    if coef < 1.0:
                        g = g * coef
            self.last_skipped.fill_(0)
            flat.data.mul_(1.0 - lr * wd)
            self.exp_avg.lerp_(g, 1.0 - b1)
            self.exp_avg_sq.mul_(b2).addcmul_(g, g, value=1.0 - b2)
            denom = (self.exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
            flat.data.addcdiv_(self.exp_avg, denom, value=-lr / bc1)
        self._step_t.fill_(float(self.step_count))
        return loss


    # ---- CUDA-graph support --------------------------------------------------------
    def launch(self, grad_norm: torch.Tensor, max_norm: float, hparams: torch.Tensor) -> None:
        """The update kernel alone, with lr and bias corrections read from ``hparams`` on
        the device (captured into a CUDA graph); the host-side step count is advanced
        by the caller (see :meth:`sync_step_state`)."""
        from packbalance_b200.ops import _native

        group = self.param_groups[0]
        flat = self.flat
        b1, b2 = group["betas"]
        _native.module().adamw_step(
            flat.data, flat.grad, self.exp_avg, self.exp_avg_sq,
            flat.shadow if flat.shadow is not None else flat.data, grad_norm, self.last_skipped,
            0.0, float(b1), float(b2), float(group["eps"]), float(group["weight_decay"]), 1.0, 1.0,
            float(max_norm), flat.shadow is not None, hparams,
        )
        flat.mark_shadow_fresh()

    def sync_step_state(self) -> None:
        """Refresh the per-parameter ``step`` entries after a replayed update."""
        self._step_t.fill_(float(self.step_count))

    def state_dict(self) -> dict[str, Any]:
        sd = super().state_dict()
        for st in sd["state"].values():  # independent step tensors, as torch.optim.AdamW has
            st["step"] = st["step"].clone()
        return sd


def global_grad_norm(flat: FlatParameters) -> torch.Tensor:
    """L2 norm of the flat gradient as a device scalar (no host sync)."""
    if flat.grad.is_cuda:
        from packbalance_b200.ops import _native

        return _native.module().l2_norm(flat.grad)
    return torch.linalg.vector_norm(flat.grad)
