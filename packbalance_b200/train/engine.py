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

On the native CUDA path without sharding, the whole step (forward, backward, the
gradient all-reduce launches on their side stream, norm and AdamW) is captured once
in a CUDA graph per input signature and replayed: the step's inputs are copied into
the graph's static buffers, and the per-step scalars (loss scale, learning rate, bias
corrections) live in device memory, so one launch replaces several hundred and the
host no longer paces the GPU.
"""

from __future__ import annotations

import contextlib
import math
import os
from typing import Any

import torch
import torch.distributed as dist
from torch.profiler import record_function

from packbalance_b200.config import PackBalanceConfig
from packbalance_b200.data.dataset import concat_packs
from packbalance_b200.models.llama import LlamaForCausalLM
from packbalance_b200.ops.attention import PLAN_CTAS, attention_plan_host, plan_to_device
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


def _signature(batch: dict[str, Any]) -> tuple:
    sig = []
    for k in sorted(batch):
        v = batch[k]
        if isinstance(v, torch.Tensor):
            sig.append((k, tuple(v.shape), v.dtype))
        elif isinstance(v, dict):
            sig.append((k, _signature(v)))
    return tuple(sig)


def _copy_into(dst: dict[str, Any], src: dict[str, Any]) -> None:
    for k, v in dst.items():
        if isinstance(v, torch.Tensor):
            v.copy_(src[k], non_blocking=True)
        elif isinstance(v, dict):
            _copy_into(v, src[k])


def _pin(tree: dict[str, Any]) -> dict[str, Any]:
    return {k: (_pin(v) if isinstance(v, dict) else v.pin_memory() if isinstance(v, torch.Tensor) else v)
            for k, v in tree.items()}


class HostScalars:
    """Device scalars (losses, norms) read back to the host without stalling the launch
    queue: :meth:`push` starts a non-blocking copy into pinned memory and returns the
    value pushed ``lag`` calls earlier (``None`` until there is one), so the host
    prepares and launches step i+1 while step i runs; :meth:`drain` returns the rest.
    Every pushed value reaches the host."""

    def __init__(self, lag: int = 1) -> None:
        self.lag = lag
        self._pending: list[tuple[torch.Tensor, Any]] = []

    def push(self, value: torch.Tensor) -> float | None:
        value = value.detach().reshape(())
        if value.is_cuda:
            buf = torch.empty((), dtype=value.dtype, pin_memory=True)
            buf.copy_(value, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
        else:
            buf, ev = value.clone(), None
        self._pending.append((buf, ev))
        if len(self._pending) > self.lag:
            return self._pop()
        return None

    def _pop(self) -> float:
        buf, ev = self._pending.pop(0)
        if ev is not None:
            ev.synchronize()
        return float(buf)

    def drain(self) -> list[float]:
        out = []
        while self._pending:
            out.append(self._pop())
        return out


def _clone_tensors(batch: dict[str, Any]) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            out[k] = v.clone()
        elif isinstance(v, dict):
            out[k] = _clone_tensors(v)
    return out


class _GraphedStep:
    """One captured native step with static input buffers (see the module docstring)."""

    HP_RING = 4

    def __init__(self, engine: "TrainEngine", batch: dict[str, Any]) -> None:
        dev = engine.device
        self.static = _clone_tensors(batch)
        self.loss_scale = torch.ones((), device=dev, dtype=torch.float32)
        self.hp = torch.zeros(3, device=dev, dtype=torch.float32)  # lr, bias corrections 1 and 2
        # A ring of pinned staging buffers for ``hp``: the host may run several steps
        # ahead of the device, and a buffer is rewritten only after its copy ran.
        self.hp_host = [torch.zeros(3, dtype=torch.float32).pin_memory() for _ in range(self.HP_RING)]
        self.hp_done = [torch.cuda.Event() for _ in range(self.HP_RING)]
        self.hp_next = 0
        engine.flat.refresh_shadow()
        torch.cuda.synchronize(dev)
        from packbalance_b200.models import fused

        self.graph = torch.cuda.CUDAGraph()
        fused.ASYNC_WGRAD = True  # weight gradients on a parallel branch of the graph
        try:
            # thread-local capture: a data-loader thread pinning host memory meanwhile
            # (cudaHostAlloc) must not invalidate this thread's capture
            with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
                self.out = engine._native_body([self.static], self.loss_scale, self.hp)
        finally:
            fused.ASYNC_WGRAD = False

    def run(self, batch: dict[str, Any], loss_scale: float, hp: tuple[float, float, float]) -> dict[str, torch.Tensor]:
        _copy_into(self.static, batch)
        self.loss_scale.fill_(loss_scale)
        k = self.hp_next
        self.hp_next = (k + 1) % self.HP_RING
        self.hp_done[k].synchronize()  # the copy that last used this buffer has run
        buf = self.hp_host[k]
        buf[0], buf[1], buf[2] = hp
        self.hp.copy_(buf, non_blocking=True)
        self.hp_done[k].record()
        self.graph.replay()
        return {k: v.clone() for k, v in self.out.items()}


def to_device_batch(batch: dict[str, Any], device: torch.device) -> dict[str, Any]:
    out: dict[str, Any] = {}
    for k, v in batch.items():
        if isinstance(v, torch.Tensor):
            out[k] = v.to(device, non_blocking=True)
        elif k == "attn_plan" and isinstance(v, dict):
            out[k] = plan_to_device(v, device)
        else:
            out[k] = v
    return out


class TrainEngine:
    # Captured step graphs kept (each holds its own activation memory pool); inputs of
    # other shapes run eagerly.
    MAX_GRAPHS = 4

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
        # the reference's train.deterministic: fixed-order reductions in the native kernels
        # (ops/_native.set_deterministic), eager steps (no CUDA graphs), peer-load
        # all-reduce summed in rank order
        self.deterministic = bool(cfg.train.deterministic) and native_ok
        if self.deterministic:
            from packbalance_b200.ops import _native

            _native.set_deterministic(True)
        if self.fsdp and native_ok:
            # Native sharded path: per-unit shards in symmetric memory, all-gather fused
            # into the consuming GEMMs, reduce-scatter fused with the sharded AdamW.
            from packbalance_b200.parallel.sharded import ShardedAdamW, ShardedParameters, auto_weight_windows

            ww = cfg.train.fsdp_weight_windows
            if ww < 0:
                n_params = sum(p.numel() for p in self.model.parameters())
                ww = auto_weight_windows(n_params, torch.cuda.get_device_properties(device).total_memory)
            # rotating gradient windows need one backward per step (the microbatch loop
            # keeps every unit's gradient until the optimizer step)
            self.sharded = ShardedParameters(self.model, grad_windows=None if cfg.train.fuse_microbatches else 0,
                                             weight_windows=ww)
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
            self.dp = DataParallel(self.flat, cfg.train.bucket_cap_mb, cfg.train.comm_backend,
                                   deterministic=self.deterministic, wire=cfg.train.grad_reduce_dtype)
            self.flat.ready_hook = self.dp.notify_ready
            self.optimizer = FlatAdamW(
                self.flat,
                lr=cfg.train.lr,
                betas=(cfg.train.beta1, cfg.train.beta2),
                weight_decay=cfg.train.weight_decay,
            )
        self.scheduler = self.make_scheduler(start_step)
        self.native = self.model.uses_native_path(torch.empty(0, device=device))
        self._graphs: dict[tuple, _GraphedStep] = {}
        self._eager_seen: dict[tuple, int] = {}
        env = os.environ.get("PB_CUDA_GRAPHS")
        self.use_graphs = (
            cfg.train.cuda_graphs and (env != "0") and self.native and self.sharded is None and not self.fsdp
            and not self.deterministic
            and device.type == "cuda" and (self.world == 1 or (self.dp is not None and self.dp.fused is not None))
        )
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

    def prepare_batch(self, batch: dict[str, Any]) -> dict[str, Any]:
        """Host-side preprocessing of a (concatenated) batch: on the native path, the
        attention work lists are built on the host from ``doc_start`` and travel with
        the batch's host->device copy."""
        if self.native and "attn_plan" not in batch and isinstance(batch.get("doc_start"), torch.Tensor) \
                and not batch["doc_start"].is_cuda:
            batch = dict(batch)
            ctas = PLAN_CTAS
            if self.device.type == "cuda":
                from packbalance_b200.ops.gemm import sm_count

                ctas = sm_count(self.device)
            plan = attention_plan_host(batch["doc_start"], self.cfg.model.n_heads, ctas)
            if self.device.type == "cuda":
                # pinned (torch's caching host allocator), so the copy to the device is
                # asynchronous and the host can prepare the next step meanwhile
                plan = _pin(plan)
            batch["attn_plan"] = plan
        return batch

    def _forward_backward(self, batch: dict[str, Any], loss_scale: float) -> torch.Tensor:
        with record_function("packbalance/forward"), self.autocast():
            out = self.model(
                batch["input_ids"].unsqueeze(0),
                labels=batch["labels"].unsqueeze(0),
                position_ids=batch["position_ids"].unsqueeze(0),
                doc_ids=batch["doc_ids"].unsqueeze(0),
                doc_start=batch.get("doc_start"),
                attn_plan=batch.get("attn_plan"),
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
        groups = [concat_packs(packs)] if self.cfg.train.fuse_microbatches else packs
        if self.use_graphs and len(groups) == 1:
            batch = self.prepare_batch(groups[0])
            sig = _signature(batch)
            g = self._graphs.get(sig)
            if g is None and self._eager_seen.get(sig, 0) >= 2 and len(self._graphs) < self.MAX_GRAPHS:
                # warmed up (allocator pools, kernel attributes, lazy buffers): capture
                g = self._graphs[sig] = _GraphedStep(self, to_device_batch(batch, self.device))
            if g is not None:
                opt = self.optimizer
                grp = opt.param_groups[0]
                b1, b2 = grp["betas"]
                opt.step_count += 1
                t = opt.step_count
                out = g.run(batch, loss_scale, (float(grp["lr"]), 1.0 - b1**t, 1.0 - b2**t))
                opt.sync_step_state()
                self.scheduler.step()
                return out
            self._eager_seen[sig] = self._eager_seen.get(sig, 0) + 1
            groups = [batch]
        out = self._native_body([to_device_batch(self.prepare_batch(b), self.device) for b in groups], loss_scale)
        self.scheduler.step()
        return out

    def _native_body(self, batches: list[dict[str, Any]], loss_scale, hparams: torch.Tensor | None = None
                     ) -> dict[str, torch.Tensor]:
        """Forward + backward of this rank's batches (device), gradient averaging, norm,
        clipping and AdamW.  ``loss_scale`` and ``hparams`` may be device tensors (graph
        capture); with ``hparams`` the optimizer's host-side step count is left alone."""
        if self.native:
            self.flat.begin_window()
        else:
            self.flat.zero_grad()
        self.dp.start_step()
        local = torch.zeros((), device=self.device, dtype=torch.float32)
        for i, batch in enumerate(batches):
            # gradients are final only in the last microbatch's backward pass
            self.dp.hold = i < len(batches) - 1
            local += self._forward_backward(batch, loss_scale)
        self.dp.hold = False
        if self.native:
            self.flat.finish_window()
        with record_function("packbalance/optimizer"):
            sq = self.dp.reduce()
            if not self.native:
                self.flat.ready_all()
            norm = sq.sqrt() if sq is not None else global_grad_norm(self.flat)
            if hparams is None:
                self.optimizer.step(grad_norm=norm, max_norm=self.cfg.train.grad_clip)
            else:
                self.optimizer.launch(norm, self.cfg.train.grad_clip, hparams)
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
            local += self._forward_backward(to_device_batch(self.prepare_batch(batch), self.device), loss_scale)
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
        if self.deterministic:
            from packbalance_b200.ops import _native

            _native.set_deterministic(False)
