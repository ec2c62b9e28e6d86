"""One training step: the public API the trainer, the benches and users drive.

:class:`TrainEngine` owns the model, the flat parameter buffers, the data-parallel
gradient engine, the optimizer and the LR schedule.  ``engine.step(packs,
step_tokens)`` runs one optimizer step on this rank's packs and returns device
scalars (no host synchronisation):

1. the packs are concatenated (``fuse_microbatches``) or looped over (the
   reference's ``no_sync`` microbatch loop) - both give the reference's gradient;
2. loss = summed token CE * ``world_size / step_tokens`` (the reference's exact
   global-token normalisation, ``train/train.py:320-345``);
3. backward writes weight gradients into the flat buffer; the data-parallel engine
   averages them bucket by bucket as layers finish;
4. global gradient norm, clipping and AdamW run as device kernels; a non-finite
   norm skips the update.
"""

from __future__ import annotations

import contextlib
import math
from typing import Any

import torch
import torch.distributed as dist
from torch.profiler import record_function

from packbalance_b200.config import PackBalanceConfig
from packbalance_b200.data.dataset import concat_packs
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.parallel.distributed import DataParallel
from packbalance_b200.parallel.flat import FlatParameters
from packbalance_b200.parallel.optim import FlatAdamW, global_grad_norm
from packbalance_b200.utils import get_autocast_dtype, get_world_size


def make_lr_lambda(cfg: PackBalanceConfig):
    """Linear warmup from 0, then cosine to ``min_lr`` (reference ``train/train.py:72-83``)."""
    warm = max(1, cfg.train.warmup_steps)
    total = max(1, cfg.train.max_steps)
    floor = cfg.train.min_lr / cfg.train.lr if cfg.train.lr else 0.0

    def lr_lambda(step: int) -> float:
        if step < warm:
            return step / warm
        frac = min(1.0, (step - warm) / max(1, total - warm))
        return floor + (1.0 - floor) * 0.5 * (1.0 + math.cos(math.pi * frac))

    return lr_lambda


def to_device_batch(batch: dict[str, Any], device: torch.device) -> dict[str, Any]:
    return {k: (v.to(device, non_blocking=True) if isinstance(v, torch.Tensor) else v) for k, v in batch.items()}


class TrainEngine:
    def __init__(
        self,
        cfg: PackBalanceConfig,
        device: torch.device,
        model: LlamaForCausalLM | None = None,
        *,
        start_step: int = 0,
    ) -> None:
        self.cfg = cfg
        self.device = device
        self.world = get_world_size() if dist.is_initialized() else 1
        self.model = model if model is not None else LlamaForCausalLM(cfg.model).to(device)
        if cfg.model.gradient_checkpointing:
            self.model.gradient_checkpointing_enable()
        self.model.train()
        self.fsdp = bool(cfg.train.fsdp) and self.world > 1
        self.sharded = None
        native_ok = device.type == "cuda" and self.model.uses_native_path(torch.empty(0, device=device))
        if self.fsdp and native_ok:
            # Native sharded path: per-unit shards in symmetric memory, all-gather fused
            # into the consuming GEMMs, reduce-scatter fused with the sharded AdamW.
            from packbalance_b200.parallel.sharded import ShardedAdamW, ShardedParameters

            self.sharded = ShardedParameters(self.model)
            self.model.flat = self.sharded
            self.flat = self.sharded
            self.dp = None
            self.optimizer = ShardedAdamW(
                self.sharded,
                lr=cfg.train.lr,
                betas=(cfg.train.beta1, cfg.train.beta2),
                weight_decay=cfg.train.weight_decay,
            )
        elif self.fsdp:
            # CPU (gloo) or eager path: torch FSDP2 over the module graph (per-layer
            # units, then the root), AdamW on the DTensor shards, DCP checkpoints.
            from torch.distributed.fsdp import fully_shard

            self.model.native = False
            for layer in self.model.model.layers:
                fully_shard(layer)
            fully_shard(self.model)
            self.flat = None
            self.dp = None
            self.optimizer = torch.optim.AdamW(
                self.model.parameters(),
                lr=cfg.train.lr,
                betas=(cfg.train.beta1, cfg.train.beta2),
                weight_decay=cfg.train.weight_decay,
                fused=device.type == "cuda",
            )
        else:
            self.flat = FlatParameters(self.model)
            self.model.flat = self.flat
            self.dp = DataParallel(self.flat, cfg.train.bucket_cap_mb, cfg.train.comm_backend)
            self.flat.ready_hook = self.dp.notify_ready
            self.optimizer = FlatAdamW(
                self.flat,
                lr=cfg.train.lr,
                betas=(cfg.train.beta1, cfg.train.beta2),
                weight_decay=cfg.train.weight_decay,
            )
        self.scheduler = self.make_scheduler(start_step)
        self.native = self.model.uses_native_path(torch.empty(0, device=device))
        amp = get_autocast_dtype(cfg.train.dtype) if device.type == "cuda" and not self.native else None
        self.autocast = (lambda: torch.autocast("cuda", dtype=amp)) if amp is not None else contextlib.nullcontext

    def make_scheduler(self, start_step: int):
        return torch.optim.lr_scheduler.LambdaLR(
            self.optimizer, make_lr_lambda(self.cfg), last_epoch=start_step - 1
        )

    def rebuild_scheduler(self, start_step: int) -> None:
        for g in self.optimizer.param_groups:
            g.setdefault("initial_lr", self.cfg.train.lr)
        self.scheduler = self.make_scheduler(start_step)

    def _forward_backward(self, batch: dict[str, Any], loss_scale: float) -> torch.Tensor:
        with record_function("packbalance/forward"), self.autocast():
            out = self.model(
                batch["input_ids"].unsqueeze(0),
                labels=batch["labels"].unsqueeze(0),
                position_ids=batch["position_ids"].unsqueeze(0),
                doc_ids=batch["doc_ids"].unsqueeze(0),
                doc_start=batch.get("doc_start"),
            )
        loss = out.loss
        with record_function("packbalance/backward"):
            (loss * loss_scale).backward()
        return loss.detach().float()

    def step(self, packs: list[dict[str, Any]], step_tokens: int) -> dict[str, torch.Tensor]:
        """One optimizer step on this rank's packs (host or device tensors)."""
        if step_tokens <= 0:
            raise RuntimeError("step has no useful tokens")
        loss_scale = self.world / step_tokens
        if self.sharded is not None:
            return self._sharded_step(packs, loss_scale)
        if self.fsdp:
            return self._fsdp_step(packs, loss_scale)
        if self.native:
            self.flat.begin_window()
        else:
            self.flat.zero_grad()
        self.dp.start_step()
        groups = [concat_packs(packs)] if self.cfg.train.fuse_microbatches else packs
        local = torch.zeros((), device=self.device, dtype=torch.float32)
        for i, batch in enumerate(groups):
            # gradients are final only in the last microbatch's backward pass
            self.dp.hold = i < len(groups) - 1
            local += self._forward_backward(to_device_batch(batch, self.device), loss_scale)
        self.dp.hold = False
        if self.native:
            self.flat.finish_window()
        with record_function("packbalance/optimizer"):
            sq = self.dp.reduce()
            if not self.native:
                self.flat.ready_all()
            norm = sq.sqrt() if sq is not None else global_grad_norm(self.flat)
            self.optimizer.step(grad_norm=norm, max_norm=self.cfg.train.grad_clip)
            self.scheduler.step()
        return {"loss_sum": local, "grad_norm": norm}

    def _sharded_step(self, packs: list[dict[str, Any]], loss_scale: float) -> dict[str, torch.Tensor]:
        sp = self.sharded
        sp.begin_window()
        sp.start_step()
        groups = [concat_packs(packs)] if self.cfg.train.fuse_microbatches else packs
        local = torch.zeros((), device=self.device, dtype=torch.float32)
        for i, batch in enumerate(groups):
            # earlier microbatches only accumulate: no unit is final before the last one
            sp.hold_ready = i < len(groups) - 1
            local += self._forward_backward(to_device_batch(batch, self.device), loss_scale)
        sp.hold_ready = False
        with record_function("packbalance/optimizer"):
            self.optimizer.step(max_norm=self.cfg.train.grad_clip)
            self.scheduler.step()
        return {"loss_sum": local, "grad_norm": sp.norm_out}

    def _fsdp_step(self, packs: list[dict[str, Any]], loss_scale: float) -> dict[str, torch.Tensor]:
        self.optimizer.zero_grad(set_to_none=True)
        groups = [concat_packs(packs)] if self.cfg.train.fuse_microbatches else packs
        local = torch.zeros((), device=self.device, dtype=torch.float32)
        for i, batch in enumerate(groups):
            self.model.set_requires_gradient_sync(i == len(groups) - 1)
            local += self._forward_backward(to_device_batch(batch, self.device), loss_scale)
        with record_function("packbalance/optimizer"):
            norm = torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.train.grad_clip)
            if hasattr(norm, "full_tensor"):
                norm = norm.full_tensor()
            self.optimizer.step()
            self.scheduler.step()
        return {"loss_sum": local, "grad_norm": norm}

    def global_loss(self, local_loss_sum: torch.Tensor, step_tokens: int) -> torch.Tensor:
        with record_function("packbalance/comm"):
            t = local_loss_sum.detach().clone()
            if dist.is_initialized():
                dist.all_reduce(t, op=dist.ReduceOp.SUM)
            return t / step_tokens

    def close(self) -> None:
        if self.dp is not None:
            self.dp.close()
