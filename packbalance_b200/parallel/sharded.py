"""Fully-sharded data parallelism over NVSwitch peer memory (native FSDP engine).

Replaces the reference's FSDP2 wrapping (``train/distributed.py:42-51``: ``fully_shard``
per decoder layer, then the root) for the native CUDA path.  Same sharding units (one
per decoder layer, one for the embedding, one for an untied LM head); the collectives
are this framework's own kernels:

* **all-gather fused into the consuming GEMM.**  Rank p owns the p-th of W equal chunks
  of every unit and keeps the bf16 copy of its chunks in a symmetric "owned" buffer
  (written by its optimizer step).  A unit is used from this rank's bf16 gathered
  storage: its own place (embedding, head, and every unit when the weights persist), or
  one of ``weight_windows`` rotating windows (decoder layers).  The first GEMM that
  reads a unit's weights (the QKV GEMM for q|k|v|o, the gate|up GEMM for gate|up|down,
  the LM-head GEMM for the head) carries copy warps that fetch the chunks over NVLink
  while its MMAs run on the tiles already copied (``csrc/ag_copy.cuh``).  With windows,
  a layer's weights are fetched again for its backward pass: a narrow all-gather on a
  side stream, issued when the next layer's backward starts (one layer ahead), like the
  reference's FSDP2 resharding after forward with prefetch.  The embedding lookup reads
  its rows straight from the owners' fp32 master shards.
* **reduce-scatter as each unit's backward finishes**, on a communication stream: rank
  r sums chunk r of the unit's gradient over all ranks, scales by 1/W and keeps only
  that chunk (fp32), plus its squared norm.
* **reduce-scatter fused with the sharded AdamW**: the embedding unit, finished last,
  is reduced by the optimizer kernel itself, which then exchanges the shards' squared
  norms through peer memory, clips, runs AdamW on the fp32 master shard and writes
  the bf16 copy of its chunk into the gathered buffer for the next step's fetches
  (``csrc/fsdp.cu``).

Memory per rank (B200 has 180 GB), P parameters, W ranks, layer = the largest decoder
layer's parameters, E = embedding + head parameters:

* sharded state: 18 B/param / W (fp32 master, moments and reduced gradient, bf16 owned);
* fp32 gradients: 4 B x E plus ``grad_windows`` (3) x 4 B x layer;
* bf16 weights: 2 B x P persistent (``weight_windows`` = 0: the backward pass needs no
  second all-gather), or 2 B x E plus ``weight_windows`` (2) x 2 B x layer.

RMSNorm weights (a few KB per layer) stay replicated in fp32; their gradient is averaged
with the fused all-reduce.

Checkpoints use the reference's FSDP layout (``torch.distributed.checkpoint`` with
``model.<name>`` and AdamW ``optimizer.state.<i>.*`` keys, full tensors).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from packbalance_b200.ops import _native
from packbalance_b200.parallel.flat import GradWindow, Slot

ALIGN = 64  # elements; chunk boundaries stay 16-byte aligned in bf16 and fp32
SYNC_WORDS = 16384  # per-CTA barrier slots (uint32) in the symmetric sync buffer
PIECE_SHIFT = 12  # all-gather piece = 4096 bf16 = 8 KB (one round of a warp's loads)
BLOCK_SHIFT = 18  # readiness is tracked per block of 256 Ki elements


@dataclass
class Unit:
    name: str
    slots: list[Slot]
    unit0: int = 0  # first element in gathered/gradient coordinates
    cs: int = 0  # chunk size per rank
    soff: int = 0  # offset of this rank's chunk in the shard buffers
    order: int = 0  # position in model order (embedding 0, layers 1..L, head L+1)
    span: int = 0  # elements of parameters (the rest up to W * cs is padding)
    segments: list[tuple[int, int]] = field(default_factory=list)  # gather ranges (element lo, hi)
    # where this unit's gradient lives: in the fixed buffer (norms, embedding, head) or in
    # a rotating window (decoder layers), at element ``goff`` of that buffer
    gwin: int = -1  # window index, -1: fixed buffer
    goff: int = 0
    # where its gathered bf16 weights live: own place or a rotating window, at ``woff``
    wwin: int = -1
    woff: int = 0


def _units_of(model) -> tuple[list[Slot], list[Unit]]:
    """Replicated RMSNorm weights and the sharded units, in model order."""
    m = model.model
    norms: list[nn.Parameter] = []
    units: list[tuple[str, list[nn.Parameter]]] = [("embed", [m.embed_tokens.weight])]
    for i, layer in enumerate(m.layers):
        a, mlp = layer.self_attn, layer.mlp
        norms += [layer.input_layernorm.weight, layer.post_attention_layernorm.weight]
        units.append((f"layer{i}", [a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.o_proj.weight,
                                    mlp.gate_proj.weight, mlp.up_proj.weight, mlp.down_proj.weight]))
    norms.append(m.norm.weight)
    if model.lm_head is not None:
        units.append(("head", [model.lm_head.weight]))
    names = {id(p): n for n, p in model.named_parameters()}
    covered = {id(p) for p in norms} | {id(p) for _, ps in units for p in ps}
    missing = [n for n, p in model.named_parameters() if p.requires_grad and id(p) not in covered]
    if missing:
        raise ValueError(f"sharded layout does not cover parameters: {missing}")
    rep = [Slot(names[id(p)], p, 0, p.numel(), p.shape) for p in norms]
    out = [Unit(n, [Slot(names[id(p)], p, 0, p.numel(), p.shape) for p in ps], order=i) for i, (n, ps) in enumerate(units)]
    return rep, out


@dataclass
class Layout:
    rep: list[Slot]  # replicated RMSNorm weights (fp32), at the front
    units: list[Unit]
    rep_n: int  # elements of the replicated region (padded)
    numel: int  # gathered / gradient buffer elements
    shard_numel: int  # elements of one rank's shard


def plan_layout(model, world: int) -> Layout:
    """Element layout of the gathered and gradient buffers: the replicated norms, then
    every unit padded to a multiple of ``world * ALIGN`` and cut into ``world`` equal
    chunks (rank p owns chunk p; its shard holds its chunks of all units in order)."""
    rep, units = _units_of(model)
    off = 0
    for s in rep:
        s.offset = off
        off += s.numel
    rep_n = -(-off // ALIGN) * ALIGN
    off = rep_n
    soff = 0
    for u in units:
        u.unit0 = off
        for s in u.slots:
            s.offset = off
            off += s.numel
        u.span = off - u.unit0
        padded = -(-u.span // (world * ALIGN)) * world * ALIGN
        u.cs = padded // world
        u.soff = soff
        soff += u.cs
        off = u.unit0 + padded
        # gather segments: q..o and gate..down of a layer (the QKV and gate|up GEMMs fetch
        # them), the whole unit otherwise
        if u.name.startswith("layer"):
            q, o, g, d = u.slots[0], u.slots[3], u.slots[4], u.slots[6]
            u.segments = [(q.offset, o.offset + o.numel), (g.offset, d.offset + d.numel)]
        else:
            u.segments = [(u.unit0, u.unit0 + u.span)]
    return Layout(rep, units, rep_n, off, soff)


@dataclass
class GradStorage:
    fixed_numel: int  # norms (at their layout offsets), then the non-layer units
    win_numel: int  # one window (the largest layer unit, W * cs elements)
    windows: int  # 0: every unit in the fixed buffer (no rotation)


def plan_grad_storage(layout: Layout, world: int, windows: int) -> GradStorage:
    """Physical placement of the gradients.  With ``windows`` = K > 0 the decoder layers'
    gradients rotate through K windows of the largest layer's size, in backward order
    (the last layer takes window 0): a layer's window is written again K layers later,
    after its reduce-scatter has finished on every rank.  The norms, the embedding and an
    untied head keep their own storage (the embedding is reduced by the optimizer kernel
    at the end of the step).  With K = 0 every unit keeps its own storage, as a full
    gradient buffer."""
    off = layout.rep_n
    layers = [u for u in layout.units if u.name.startswith("layer")]
    if windows == 1:
        raise ValueError("gradient windows: 0 (no rotation) or at least 2")
    rotate = windows > 0 and len(layers) > 0
    for u in layout.units:
        if rotate and u.name.startswith("layer"):
            continue
        u.gwin, u.goff = -1, off
        off += world * u.cs
    win_numel = 0
    if rotate:
        win_numel = max(world * u.cs for u in layers)
        for pos, u in enumerate(reversed(layers)):
            u.gwin = pos % windows
            u.goff = u.gwin * win_numel
    return GradStorage(off, win_numel, windows if rotate else 0)


def auto_weight_windows(n_params: int, device_bytes: int, share: float = 0.25) -> int:
    """Weight windows for ``fsdp_weight_windows: -1``: persistent gathered bf16 weights
    (0) while they take at most ``share`` of the device's memory, else two windows."""
    return 0 if 2 * n_params <= share * device_bytes else 2


@dataclass
class WeightStorage:
    fixed_numel: int  # the non-layer units (all units without windows), then the windows
    win_numel: int
    windows: int
    numel: int  # whole gathered storage


def plan_weight_storage(layout: Layout, world: int, windows: int) -> WeightStorage:
    """Physical placement of the gathered bf16 weights.  With ``windows`` = K > 0 the
    decoder layers take K rotating windows of the largest layer's size (layer i in window
    i % K): the forward pass gathers layer i while layers i-1 .. i-K+1 stay resident, the
    backward pass gathers layer i-1 while layer i runs.  The embedding and an untied head
    keep their own place.  With K = 0 every unit keeps its own place."""
    layers = [u for u in layout.units if u.name.startswith("layer")]
    if windows == 1:
        raise ValueError("weight windows: 0 (persistent weights) or at least 2")
    rotate = windows > 0 and len(layers) > 0
    off = 0
    for u in layout.units:
        if rotate and u.name.startswith("layer"):
            continue
        u.wwin, u.woff = -1, off
        off += world * u.cs
    fixed = off
    win_numel = 0
    if rotate:
        win_numel = max(world * u.cs for u in layers)
        for i, u in enumerate(layers):
            u.wwin = i % windows
            u.woff = fixed + u.wwin * win_numel
        off = fixed + windows * win_numel
    return WeightStorage(fixed, win_numel, windows if rotate else 0, max(off, 8))


class ShardedParameters(GradWindow):
    """Sharded parameter/gradient/optimizer-state buffers of one model (CUDA, W >= 2)."""

    # Reduce-scatter launch widths: narrow while the backward pass still runs beside it
    # (a collective with a CTA on every SM keeps the GEMM / attention CTAs from being
    # scheduled until it ends), the whole GPU once nothing is left to overlap.
    RS_CTAS_OVERLAP = 24
    RS_CTAS_TAIL = 4 * 148

    # Decoder-layer gradients rotate through this many windows (0: a full gradient buffer).
    GRAD_WINDOWS = 3
    # Width of the backward pass's weight prefetch (beside the running layer's kernels).
    AG_CTAS_PREFETCH = 24

    def __init__(self, model, group: dist.ProcessGroup | None = None, rs_ctas: int | None = None,
                 grad_windows: int | None = None, weight_windows: int = 0) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if not 2 <= self.world <= 8:
            raise RuntimeError("the sharded engine covers 2..8 GPUs of one node")
        first = next(model.parameters())
        self.device = first.device
        if self.device.type != "cuda":
            raise RuntimeError("the sharded engine needs CUDA tensors")
        self.model = model
        W = self.world
        layout = plan_layout(model, W)
        self.rep_n, self.numel, self.shard_numel = layout.rep_n, layout.numel, layout.shard_numel
        rep, units = layout.rep, layout.units
        self.gstore = plan_grad_storage(layout, W, self.GRAD_WINDOWS if grad_windows is None else grad_windows)
        self.wstore = plan_weight_storage(layout, W, weight_windows)
        self.rep_slots = rep
        self.units = units
        self.embed_unit = units[0]
        self.slots = rep + [s for u in units for s in u.slots]
        self.by_param = {id(s.param): s for s in self.slots}
        self.unit_of = {id(s.param): u for u in units for s in u.slots}
        # norms (and, for the ready protocol, their layer's unit order)
        self.rep_order = {}
        # a layer's unit is only final at its input norm: the half-way point (the norm in
        # front of the MLP) releases nothing here
        self.mid_layer: set[int] = set()
        for i, layer in enumerate(model.model.layers):
            self.rep_order[id(layer.input_layernorm.weight)] = i + 1
            self.rep_order[id(layer.post_attention_layernorm.weight)] = i + 1
            self.mid_layer.add(id(layer.post_attention_layernorm.weight))
        self.rep_order[id(model.model.norm.weight)] = len(model.model.layers) + 1

        # ---- buffers -------------------------------------------------------------------
        dev = self.device
        # bf16 weights: this rank's chunks (read by the peers' fetches) and the local
        # gathered storage (plan_weight_storage)
        self.owned = symm_mem.empty(max(self.shard_numel, 8), dtype=torch.bfloat16, device=dev)
        self.gathered = torch.empty(self.wstore.numel, dtype=torch.bfloat16, device=dev)
        # gradients: norms and non-layer units in ``grad``; decoder layers in the rotating
        # windows of ``grad_win`` (plan_grad_storage)
        self.grad = symm_mem.empty(self.gstore.fixed_numel, dtype=torch.float32, device=dev)
        K = self.gstore.windows
        self.grad_win = symm_mem.empty(max(K * self.gstore.win_numel, 4), dtype=torch.float32, device=dev)
        self.master = symm_mem.empty(max(self.shard_numel, 4), dtype=torch.float32, device=dev)
        self.sync = symm_mem.empty(SYNC_WORDS + 64, dtype=torch.int32, device=dev)
        self.grad.zero_()
        self.grad_win.zero_()
        self.master.zero_()
        self.sync.zero_()
        self.h_owned = symm_mem.rendezvous(self.owned, self.group)
        self.h_grad = symm_mem.rendezvous(self.grad, self.group)
        self.h_win = symm_mem.rendezvous(self.grad_win, self.group)
        self.h_master = symm_mem.rendezvous(self.master, self.group)
        self.h_sync = symm_mem.rendezvous(self.sync, self.group)
        for h in (self.h_owned, self.h_grad, self.h_win, self.h_master, self.h_sync):
            if int(getattr(h, "offset", 0)) != 0:
                raise RuntimeError("symmetric buffers must start at their allocation base")
        # NVLS: reduce-scatter with multimem.ld_reduce when the driver bound a multicast
        # object over the gradient buffers (PB_ALLREDUCE=p2p forces peer loads)
        use_mc = os.environ.get("PB_ALLREDUCE", "auto") in ("auto", "nvls")
        self.grad_mc = int(self.h_grad.multicast_ptr or 0) if use_mc else 0
        self.win_mc = int(self.h_win.multicast_ptr or 0) if use_mc else 0
        if not (self.grad_mc and self.win_mc):
            self.grad_mc = self.win_mc = 0  # one kernel kind for every unit
        self.mode = "nvls" if self.grad_mc else "p2p"
        # window w may be written again once this event (recorded on the communication
        # stream after a later reduce-scatter, whose first barrier every rank passes only
        # after finishing the reduce-scatter that read window w) has completed
        self._win_free = [torch.cuda.Event() for _ in range(K)]
        self._last_win_unit: Unit | None = None
        self.xchg_ptrs = torch.tensor([int(p) + 4 * SYNC_WORDS for p in self.h_sync.buffer_ptrs], dtype=torch.int64,
                                      device=dev)
        self.exp_avg = torch.zeros(max(self.shard_numel, 4), dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self.shard_grad = torch.zeros_like(self.exp_avg)
        self.rep_data = torch.zeros(self.rep_n, dtype=torch.float32, device=dev)
        self.rep_m = torch.zeros_like(self.rep_data)
        self.rep_v = torch.zeros_like(self.rep_data)
        self.sumsq = torch.zeros((), dtype=torch.float32, device=dev)
        self.rep_sumsq = torch.zeros((), dtype=torch.float32, device=dev)
        self.norm_out = torch.zeros((), dtype=torch.float32, device=dev)
        self.skipped = torch.zeros((), dtype=torch.int32, device=dev)
        self.arrive = torch.zeros(1, dtype=torch.int32, device=dev)
        self.go = torch.zeros(1, dtype=torch.int32, device=dev)
        max_blocks = max(((hi - lo) >> BLOCK_SHIFT) + 2 for u in units for lo, hi in u.segments)
        self.ag_counters = torch.zeros(max_blocks + 1, dtype=torch.int32, device=dev)
        # fetch sources: owner p's element e of unit u sits at owned_p[soff + e - unit0 - p cs];
        # row u holds the W bases that make that ``src[p] + e`` (bf16 elements)
        src = [[int(self.h_owned.buffer_ptrs[p]) + 2 * (u.soff - u.unit0 - p * u.cs) for p in range(W)]
               for u in units]
        self.ag_src = torch.tensor(src, dtype=torch.int64, device=dev)
        # backward-pass prefetch of the next layer's weights (side stream, own counters)
        self.ag_stream = torch.cuda.Stream(device=dev, priority=-1)
        self.ag_counters_pf = torch.zeros_like(self.ag_counters)
        self.ag_ctas_prefetch = self.AG_CTAS_PREFETCH
        Kw = self.wstore.windows
        self._resident: list[Unit | None] = [None] * Kw  # unit gathered in each window
        self._pending: list[torch.cuda.Event | None] = [None] * Kw  # prefetch not yet waited on
        self._epoch = 0  # barrier epochs (sync pads), one per collective launch
        self._arrive_total = 0
        cap = SYNC_WORDS // (3 * W)
        self.rs_ctas = min(rs_ctas or self.RS_CTAS_OVERLAP, cap)
        self.rs_ctas_tail = min(rs_ctas or self.RS_CTAS_TAIL, cap)
        C = _native.module()
        self.final_ctas = int(min(C.fsdp_adamw_max_ctas(W), SYNC_WORDS // (3 * W)))
        self.comm = torch.cuda.Stream(device=dev, priority=-1)

        # ---- initial values (every rank holds the same full init) ------------------
        with torch.no_grad():
            for s in rep:
                self.rep_data[s.offset : s.offset + s.numel].copy_(s.param.detach().reshape(-1))
            for u in units:
                full = self._unit_from_params(u)
                lo = self.rank * u.cs
                self.master[u.soff : u.soff + u.cs].copy_(full[lo : lo + u.cs])
                self.owned[u.soff : u.soff + u.cs].copy_(full[lo : lo + u.cs])
                if u.wwin < 0:
                    self.gathered[u.woff : u.woff + W * u.cs].copy_(full)
        # parameters become views: norms -> replicated fp32, sharded -> gathered bf16 (a
        # windowed layer's view shows its weights only while the layer is resident)
        for s in rep:
            s.param.data = self.rep_data[s.offset : s.offset + s.numel].view(s.shape)
            s.param.grad = self.grad[s.offset : s.offset + s.numel].view(s.shape)
        for u in units:
            for s in u.slots:
                s.param.grad = None
                o = u.woff + s.offset - u.unit0
                s.param.data = self.gathered[o : o + s.numel].view(s.shape)
        self._segs = self._build_segments()
        self._fresh: set[int] = set()
        self._gathered_segs: set[tuple[int, int]] = {seg for u in units if u.wwin < 0 for seg in u.segments}
        self._issued: set[int] = set()
        self.ready_hook = None
        self.hold_ready = False  # set while a non-final microbatch runs its backward pass
        # the first fetches read the peers' owned chunks written above
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    # ---- construction helpers ---------------------------------------------------------
    def _unit_from_params(self, u: Unit) -> torch.Tensor:
        full = torch.zeros(self.world * u.cs, dtype=torch.float32, device=self.device)
        for s in u.slots:
            o = s.offset - u.unit0
            full[o : o + s.numel].copy_(s.param.detach().reshape(-1).float())
        return full

    def _build_segments(self) -> torch.Tensor:
        rows = []
        base = self.owned.data_ptr()
        for u in self.units:
            rows.append([
                self.master.data_ptr() + 4 * u.soff, self.exp_avg.data_ptr() + 4 * u.soff,
                self.exp_avg_sq.data_ptr() + 4 * u.soff, self.shard_grad.data_ptr() + 4 * u.soff,
                base + 2 * u.soff, u.cs,
            ])
        rows.append([self.rep_data.data_ptr(), self.rep_m.data_ptr(), self.rep_v.data_ptr(),
                     self.grad.data_ptr(), 0, self.rep_n])
        return torch.tensor(rows, dtype=torch.int64, device=self.device)

    # ---- views the fused model code uses -----------------------------------------------
    def slot(self, p: nn.Parameter) -> Slot:
        return self.by_param[id(p)]

    def _span(self, params) -> torch.Tensor:
        """[rows, cols] view of adjacent ``params`` in the gathered storage."""
        slots = [self.by_param[id(p)] for p in params]
        for a, b in zip(slots, slots[1:], strict=False):
            if a.offset + a.numel != b.offset:
                raise ValueError(f"parameters {a.name} and {b.name} are not adjacent")
        cols = slots[0].shape[-1]
        rows = sum(s.numel for s in slots) // cols
        u = self.unit_of[id(params[0])]
        o = u.woff + slots[0].offset - u.unit0
        return self.gathered[o : o + rows * cols].view(rows, cols)

    def _segment(self, p: nn.Parameter) -> tuple[Unit, tuple[int, int]]:
        u = self.unit_of[id(p)]
        off = self.by_param[id(p)].offset
        for seg in u.segments:
            if seg[0] <= off < seg[1]:
                return u, seg
        raise AssertionError("parameter outside its unit's segments")

    def _ag_spec(self, u: Unit, seg: tuple[int, int], b0: int, split: int = 0, counters: torch.Tensor | None = None
                 ) -> list[int]:
        # sources: the owners' ``owned`` buffers (row u of ag_src); destination: the unit's
        # place in the gathered storage, both addressed by gathered-coordinate elements
        return [
            self.ag_src[u.order].data_ptr(), self.gathered.data_ptr() + 2 * (u.woff - u.unit0), seg[0],
            -(-seg[1] // 8) * 8, u.unit0, u.cs, b0, split, self.rank, self.world, PIECE_SHIFT, BLOCK_SHIFT,
            (self.ag_counters if counters is None else counters).data_ptr(), 1,
        ]

    def _make_resident(self, u: Unit) -> None:
        """Bookkeeping before ``u`` is gathered: its window's previous unit is evicted."""
        if u.wwin < 0:
            return
        prev = self._resident[u.wwin]
        if prev is not None and prev is not u:
            for seg in prev.segments:
                self._gathered_segs.discard(seg)
        self._resident[u.wwin] = u

    def _use(self, u: Unit) -> None:
        """The current stream is about to read ``u``'s gathered weights: wait for a
        prefetch that filled its window."""
        if u.wwin >= 0 and self._pending[u.wwin] is not None:
            torch.cuda.current_stream(self.device).wait_event(self._pending[u.wwin])
            self._pending[u.wwin] = None

    def gather_spec(self, *params: nn.Parameter) -> list[int] | None:
        """Spec of the fused all-gather for the GEMM that reads ``params`` as its B
        operand, or None when that segment is already local this step."""
        if id(params[0]) not in self.unit_of:
            return None
        u, seg = self._segment(params[0])
        if seg in self._gathered_segs:
            self._use(u)
            return None
        self._make_resident(u)
        self._use(u)
        self._gathered_segs.add(seg)
        # gate|up: the two matrices are copied interleaved, in the order SwiGLU tiles read them
        split = params[0].numel() if len(params) == 2 and params[0].shape == params[1].shape else 0
        return self._ag_spec(u, seg, self.by_param[id(params[0])].offset, split)

    def _ensure_gathered(self, params) -> None:
        for p in params:
            if id(p) not in self.unit_of:
                continue
            u, seg = self._segment(p)
            if seg not in self._gathered_segs:
                self._make_resident(u)
                self._use(u)
                self._gathered_segs.add(seg)
                _native.module().fsdp_all_gather(self._ag_spec(u, seg, seg[0]), 2 * _sms(self.device))
            else:
                self._use(u)

    def shadow_of(self, *params: nn.Parameter) -> torch.Tensor:
        self._ensure_gathered(params)
        return self._span(params)

    def backward_begin(self, *params: nn.Parameter) -> None:
        """A decoder layer's backward pass starts (``params``: its weights).  With weight
        windows, fetch the previous layer's weights into its window on the prefetch stream,
        beside this layer's kernels; the window's last reader (the layer ``windows``
        positions later) was enqueued on the current stream before this point."""
        u = self.unit_of.get(id(params[0]))
        if u is None or u.wwin < 0:
            return
        prev = next((v for v in self.units if v.order == u.order - 1), None)
        if prev is None or prev.wwin < 0 or all(seg in self._gathered_segs for seg in prev.segments):
            return
        cur = torch.cuda.current_stream(self.device)
        self.ag_stream.wait_stream(cur)
        self._make_resident(prev)
        with torch.cuda.stream(self.ag_stream):
            for seg in prev.segments:
                if seg not in self._gathered_segs:
                    self._gathered_segs.add(seg)
                    _native.module().fsdp_all_gather(
                        self._ag_spec(prev, seg, seg[0], counters=self.ag_counters_pf), self.ag_ctas_prefetch)
            ev = torch.cuda.Event()
            ev.record(self.ag_stream)
        self._pending[prev.wwin] = ev

    def _unit_grad(self, u: Unit) -> torch.Tensor:
        """The unit's gradient (its W * cs elements, unit layout) where it lives now."""
        buf = self.grad_win if u.gwin >= 0 else self.grad
        return buf[u.goff : u.goff + self.world * u.cs]

    def _slot_grad(self, s: Slot) -> torch.Tensor:
        u = self.unit_of.get(id(s.param))
        if u is None:  # replicated norm: fixed buffer at its layout offset
            return self.grad[s.offset : s.offset + s.numel]
        return self._unit_grad(u)[s.offset - u.unit0 : s.offset - u.unit0 + s.numel]

    def grad_of(self, *params: nn.Parameter) -> torch.Tensor:
        slots = [self.by_param[id(p)] for p in params]
        for a, b in zip(slots, slots[1:], strict=False):
            if a.offset + a.numel != b.offset:
                raise ValueError(f"parameters {a.name} and {b.name} are not adjacent")
        cols = slots[0].shape[-1]
        rows = sum(x.numel for x in slots) // cols
        u = self.unit_of.get(id(params[0]))
        if u is None:
            return self.grad[slots[0].offset : slots[0].offset + rows * cols].view(rows, cols)
        lo = slots[0].offset - u.unit0
        return self._unit_grad(u)[lo : lo + rows * cols].view(rows, cols)

    def prezero(self, *params: nn.Parameter) -> None:
        """GradWindow.prezero over this layout: a decoder layer's window is zeroed (once
        the window is free on every rank) in one fill of its claimed range."""
        fresh = [p for p in params if id(p) not in self._fresh]
        by_unit: dict[int, list[Slot]] = {}
        for p in fresh:
            u = self.unit_of.get(id(p))
            by_unit.setdefault(id(u) if u is not None else 0, []).append(self.by_param[id(p)])
        for key, slots in by_unit.items():
            u = self.unit_of.get(id(slots[0].param))
            if u is not None and u.gwin >= 0:
                torch.cuda.current_stream(self.device).wait_event(self._win_free[u.gwin])
            slots.sort(key=lambda x: x.offset)
            runs: list[list[Slot]] = []
            for x in slots:
                if runs and runs[-1][-1].offset + runs[-1][-1].numel == x.offset:
                    runs[-1].append(x)
                else:
                    runs.append([x])
            for run in runs:
                first, last = run[0], run[-1]
                if u is None:
                    self.grad[first.offset : last.offset + last.numel].zero_()
                else:
                    self._unit_grad(u)[first.offset - u.unit0 : last.offset - u.unit0 + last.numel].zero_()
            for x in slots:
                self._fresh.add(id(x.param))

    def embedding(self, ids: torch.Tensor, weight: nn.Parameter) -> torch.Tensor:
        u = self.unit_of[id(weight)]
        s = self.by_param[id(weight)]
        return _native.module().fsdp_embedding_fwd(
            ids, int(self.h_master.buffer_ptrs_dev), s.offset, u.unit0, u.cs, u.soff, s.shape[1], s.shape[0]
        )

    def refresh_shadow(self, force: bool = False) -> None:
        """The gathered buffer is maintained by the fetches and the optimizer."""

    # ---- gradient protocol -------------------------------------------------------------
    def finish_window(self) -> None:
        """Zero the gradients no writer claimed this window: the norms, and the units whose
        reduce-scatter has not been issued yet (issued ones were finished just before)."""
        for s in self.rep_slots:
            if id(s.param) not in self._fresh:
                self.grad[s.offset : s.offset + s.numel].zero_()
                self._fresh.add(id(s.param))
        for u in self.units:
            if u.order not in self._issued:
                self._finish_unit(u)

    def zero_grad(self) -> None:
        self._fresh.clear()
        self.grad.zero_()
        self.grad_win.zero_()

    def start_step(self) -> None:
        """Called before the step's first backward: clears the norm accumulator."""
        self._issued.clear()
        self.sumsq.zero_()

    def ready(self, offset: int, streams: tuple = ()) -> None:  # FlatParameters-compatible entry (unused)
        pass

    def ready_after(self, p: nn.Parameter, streams: tuple = ()) -> None:
        """``p``'s unit and every later unit (model order) have final gradients: reduce-
        scatter them now, except the embedding unit, which the optimizer kernel reduces.
        (The callers join the weight-gradient stream before a unit's last ready point.)"""
        if self.hold_ready or id(p) in self.mid_layer:
            return
        order = self.unit_of[id(p)].order if id(p) in self.unit_of else self.rep_order[id(p)]
        for u in self.units:
            if u.order >= order and u.order not in self._issued and u is not self.embed_unit:
                self._issue_rs(u)

    def _finish_unit(self, u: Unit) -> None:
        for s in u.slots:
            if id(s.param) not in self._fresh:
                if u.gwin >= 0:
                    torch.cuda.current_stream(self.device).wait_event(self._win_free[u.gwin])
                self._slot_grad(s).zero_()
                self._fresh.add(id(s.param))

    def _issue_rs(self, u: Unit, tail: bool = False) -> None:
        self._issued.add(u.order)
        self._finish_unit(u)
        self.comm.wait_stream(torch.cuda.current_stream(self.device))
        win = u.gwin >= 0
        with torch.cuda.stream(self.comm):
            self._epoch += 1
            lo = u.goff + self.rank * u.cs
            h = self.h_win if win else self.h_grad
            _native.module().fsdp_reduce_scatter(
                int(h.buffer_ptrs_dev), int(self.h_sync.buffer_ptrs_dev), SYNC_WORDS, lo, lo + u.cs,
                self.shard_grad.data_ptr() + 4 * u.soff, self.rank, self.world, self._epoch, 1.0 / self.world,
                self.sumsq, self.rs_ctas_tail if tail else self.rs_ctas, self.win_mc if win else self.grad_mc,
            )
            # this launch's first barrier means every rank finished the reduce-scatter of
            # the previous windowed unit: that window is free once this launch completes
            if win:
                if self._last_win_unit is not None:
                    self._win_free[self._last_win_unit.gwin].record(self.comm)
                self._last_win_unit = u

    # ---- optimizer step -----------------------------------------------------------------
    def optimizer_step(self, lr: float, b1: float, b2: float, eps: float, wd: float, bc1: float, bc2: float,
                       max_norm: float) -> None:
        """Finish the reduce-scatters, then the fused reduce-scatter + AdamW kernel.
        Leaves the global gradient norm in ``norm_out`` and the skip flag in ``skipped``."""
        C = _native.module()
        self.finish_window()
        # every prefetch of this step has finished before the optimizer kernel's first
        # barrier (after it the owners overwrite the chunks the prefetches read)
        cur = torch.cuda.current_stream(self.device)
        for w, ev in enumerate(self._pending):
            if ev is not None:
                cur.wait_event(ev)
                self._pending[w] = None
        for u in self.units:
            if u.order not in self._issued and u is not self.embed_unit:
                self._issue_rs(u, tail=True)
        self.comm.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.comm):
            self.rep_sumsq.zero_()
            self._epoch += 1
            C.fused_allreduce(
                int(self.h_grad.buffer_ptrs_dev), int(self.h_sync.buffer_ptrs_dev), SYNC_WORDS, 0, self.rep_n,
                self.rank, self.world, self._epoch, 1.0 / self.world, self.rep_sumsq, min(16, self.rs_ctas), 0,
            )
            self._epoch += 1
            self._arrive_total += self.final_ctas
            e = self.embed_unit
            lo = e.goff + self.rank * e.cs
            C.fsdp_adamw(
                [int(self.h_grad.buffer_ptrs_dev), int(self.h_sync.buffer_ptrs_dev), SYNC_WORDS, self.rank,
                 self.world, self._epoch, lo, lo + e.cs, self.shard_grad.data_ptr() + 4 * e.soff,
                 self.rep_sumsq.data_ptr(), self.xchg_ptrs.data_ptr(), self.arrive.data_ptr(),
                 self._arrive_total & 0xFFFFFFFF, self.go.data_ptr(), self._segs.data_ptr(), self._segs.shape[0],
                 self.final_ctas, self.grad_mc],
                [1.0 / self.world, lr, b1, b2, eps, wd, bc1, bc2, max_norm],
                self.sumsq, self.norm_out, self.skipped,
            )
            # the optimizer kernel's barriers follow every reduce-scatter of the step:
            # after it, every window is free on every rank
            for ev in self._win_free:
                ev.record(self.comm)
        self._last_win_unit = None
        torch.cuda.current_stream(self.device).wait_stream(self.comm)
        self._issued.add(e.order)
        self._invalidate_gathered()

    def _invalidate_gathered(self) -> None:
        """The owned chunks changed: every unit is fetched again before its next use."""
        self._gathered_segs.clear()
        self._resident = [None] * self.wstore.windows
        cur = torch.cuda.current_stream(self.device)
        for w, ev in enumerate(self._pending):
            if ev is not None:
                cur.wait_event(ev)
                self._pending[w] = None

    def check(self) -> None:
        _native.check_status(self.device)

    # ---- full (unsharded) state for checkpoints ------------------------------------------
    def _gather_unit(self, buf: torch.Tensor, u: Unit) -> torch.Tensor:
        out = torch.empty(self.world * u.cs, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(out, buf[u.soff : u.soff + u.cs].contiguous(), group=self.group)
        return out

    def full_tensors(self, which: str = "param", owner_only: bool = False) -> dict[str, torch.Tensor]:
        """Full fp32 CPU tensors keyed by parameter name (``which``: param, exp_avg,
        exp_avg_sq).  Collective.  With ``owner_only`` a rank keeps only the tensors of
        the parameters whose index i satisfies i % W == rank."""
        shard = {"param": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq}[which]
        rep = {"param": self.rep_data, "exp_avg": self.rep_m, "exp_avg_sq": self.rep_v}[which]
        index = {s.name: i for i, s in enumerate(self.model_order())}
        keep = (lambda n: index[n] % self.world == self.rank) if owner_only else (lambda n: True)
        out: dict[str, torch.Tensor] = {}
        for s in self.rep_slots:
            if keep(s.name):
                out[s.name] = rep[s.offset : s.offset + s.numel].view(s.shape).cpu()
        for u in self.units:
            full = self._gather_unit(shard, u)
            for s in u.slots:
                if keep(s.name):
                    o = s.offset - u.unit0
                    out[s.name] = full[o : o + s.numel].view(s.shape).cpu()
        return out

    def load_full_tensors(self, tensors: dict[str, torch.Tensor], which: str = "param") -> None:
        """Inverse of :meth:`full_tensors` (every rank passes full tensors of the
        parameters it wants to set)."""
        shard = {"param": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq}[which]
        rep = {"param": self.rep_data, "exp_avg": self.rep_m, "exp_avg_sq": self.rep_v}[which]
        with torch.no_grad():
            for s in self.rep_slots:
                if s.name in tensors:
                    rep[s.offset : s.offset + s.numel].copy_(tensors[s.name].reshape(-1))
            for u in self.units:
                c0, c1 = u.unit0 + self.rank * u.cs, u.unit0 + (self.rank + 1) * u.cs
                for s in u.slots:
                    if s.name not in tensors:
                        continue
                    t = tensors[s.name].reshape(-1).to(self.device, torch.float32)
                    lo, hi = max(s.offset, c0), min(s.offset + s.numel, c1)
                    if lo < hi:
                        shard[u.soff + lo - c0 : u.soff + hi - c0].copy_(t[lo - s.offset : hi - s.offset])
            if which == "param":
                for u in self.units:
                    self.owned[u.soff : u.soff + u.cs].copy_(self.master[u.soff : u.soff + u.cs])
        if which == "param":
            # the peers fetch these owned chunks in the next step: every rank has written its
            # own before any rank reads
            self._invalidate_gathered()
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)

    def model_order(self) -> list[Slot]:
        """Slots in ``model.named_parameters()`` order (the optimizer's param indices)."""
        by_name = {s.name: s for s in self.slots}
        return [by_name[n] for n, p in self.model.named_parameters() if n in by_name]


def _sms(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


class ShardedAdamW(torch.optim.Optimizer):
    """AdamW over :class:`ShardedParameters` (torch.optim.AdamW math and param groups;
    the update itself is the fused reduce-scatter + AdamW kernel)."""

    def __init__(self, sp: ShardedParameters, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2) -> None:
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=False, maximize=False,
                        foreach=None, capturable=False, differentiable=False, fused=None)
        super().__init__([s.param for s in sp.model_order()], defaults)
        self.sp = sp
        self.step_count = 0
        self.last_skipped = sp.skipped

    @torch.no_grad()
    def step(self, closure=None, grad_norm: torch.Tensor | None = None, max_norm: float = 0.0):
        loss = closure() if closure is not None else None
        g = self.param_groups[0]
        b1, b2 = g["betas"]
        self.step_count += 1
        t = self.step_count
        self.sp.optimizer_step(float(g["lr"]), b1, b2, g["eps"], g["weight_decay"], 1.0 - b1**t, 1.0 - b2**t,
                               float(max_norm))
        return loss

    @property
    def grad_norm(self) -> torch.Tensor:
        return self.sp.norm_out

    # Checkpoint format: torch.optim.AdamW's (full tensors).  Collective.
    def full_state_dict(self, owner_only: bool = False) -> dict[str, Any]:
        m = self.sp.full_tensors("exp_avg", owner_only)
        v = self.sp.full_tensors("exp_avg_sq", owner_only)
        state = {}
        for i, s in enumerate(self.sp.model_order()):
            if s.name in m:
                state[i] = {"step": torch.tensor(float(self.step_count)), "exp_avg": m[s.name],
                            "exp_avg_sq": v[s.name]}
        groups = [{k: v for k, v in self.param_groups[0].items() if k != "params"}]
        groups[0]["params"] = list(range(len(self.sp.model_order())))
        return {"state": state, "param_groups": groups}

    def load_full_state_dict(self, sd: dict[str, Any]) -> None:
        order = self.sp.model_order()
        m, v, steps = {}, {}, []
        for i, st in sd.get("state", {}).items():
            name = order[int(i)].name
            m[name], v[name] = st["exp_avg"], st["exp_avg_sq"]
            steps.append(float(st["step"]))
        self.sp.load_full_tensors(m, "exp_avg")
        self.sp.load_full_tensors(v, "exp_avg_sq")
        if steps:
            self.step_count = int(max(steps))
        for k, val in sd.get("param_groups", [{}])[0].items():
            if k != "params":
                self.param_groups[0][k] = val

