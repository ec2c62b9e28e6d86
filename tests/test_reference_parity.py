"""Benchmark config #1 against the reference itself (CPU, gloo, world size 2, fp32).

Both frameworks read the same corpus; the test checks that the packs and the balanced
schedule are identical, starts both models from the same weights (the reference's
initial state dict, loaded through the shared parameter names) and compares the global
loss of 10 training steps: the reference's step body (DDP + AdamW + clipping, its own
modules) against ``TrainEngine.step``.  Skipped when the reference cannot be found
(``packbalance_b200.utils.reference.locate_reference``).
"""

import json
import os
import socket
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

from packbalance_b200.utils.reference import locate_reference

ROOT = Path(__file__).resolve().parents[1]
REF, _TRIED = locate_reference(ROOT)

pytestmark = pytest.mark.skipif(REF is None, reason="reference not found: " + "; ".join(_TRIED))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


WORKER = textwrap.dedent(
    """
    import json, os, sys
    from dataclasses import replace
    from pathlib import Path
    import torch, torch.distributed as dist
    sys.path.insert(0, os.environ["PB_ROOT"])
    sys.path.insert(1, os.environ["PB_REF"])
    torch.set_num_threads(1)
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cpu")

    from packbalance_b200.config import load_config
    from packbalance_b200.data.cost import FlopModel
    from packbalance_b200.data.dataset import PackedDataset
    from packbalance_b200.data.packer import build_packs
    from packbalance_b200.data.prepare import prepare_synthetic
    from packbalance_b200.data.sampler import build_schedule
    from packbalance_b200.data.store import TokenStore
    from packbalance_b200.models.llama import LlamaForCausalLM
    from packbalance_b200.train.engine import TrainEngine

    from packbalance.config import DataConfig as RData, ModelConfig as RModel, PackBalanceConfig as RCfg
    from packbalance.config import TrainConfig as RTrain
    from packbalance.data.cost import FlopModel as RFlop
    from packbalance.data.dataset import PackedDataset as RDataset
    from packbalance.data.packer import build_packs as rbuild_packs
    from packbalance.data.sampler import build_schedule as rbuild_schedule
    from packbalance.data.store import TokenStore as RStore
    from packbalance.model.llama import LlamaForCausalLM as RModelCls
    from packbalance.train import train as rtrain
    from packbalance.train.distributed import no_sync, wrap_model

    cfg = load_config(Path(os.environ["PB_ROOT"]) / "configs" / "b1_tiny_cpu.yaml")
    tmp = Path(os.environ["PB_TMP"])
    cfg = replace(cfg, data=replace(cfg.data, data_dir=str(tmp / "data")),
                  train=replace(cfg.train, output_dir=str(tmp / "out")))
    if rank == 0:
        prepare_synthetic(cfg.data, Path(cfg.data.data_dir))
    dist.barrier()
    m, d, t = cfg.model, cfg.data, cfg.train
    rcfg = RCfg(
        model=RModel(vocab_size=m.vocab_size, d_model=m.d_model, n_layers=m.n_layers, n_heads=m.n_heads,
                     n_kv_heads=m.n_kv_heads, d_ff=m.d_ff, max_seq_len=m.max_seq_len, tie_embeddings=m.tie_embeddings,
                     attention_backend="eager", use_fused_ce=False, ce_chunk_size=m.ce_chunk_size),
        data=RData(dataset="synthetic", data_dir=d.data_dir, seq_len=d.seq_len, mode=d.mode, schedule=d.schedule,
                   max_doc_len=d.max_doc_len, min_doc_len=d.min_doc_len, val_fraction=0.0, seed=d.seed, num_workers=0),
        train=RTrain(grad_accum=t.grad_accum, lr=t.lr, min_lr=t.min_lr, warmup_steps=t.warmup_steps, dtype="fp32",
                     max_steps=t.max_steps, grad_clip=t.grad_clip, weight_decay=t.weight_decay),
    )
    A = t.grad_accum
    store, rstore = TokenStore.open(d.data_dir), RStore.open(d.data_dir)
    packs = build_packs(store, d, FlopModel.from_config(m), split="train")
    rpacks = rbuild_packs(rstore, rcfg.data, RFlop.from_config(rcfg.model), split="train")
    key = lambda ps: [[(s.doc_id, s.start, s.length) for s in p.segments] for p in ps]
    assert key(packs) == key(rpacks), "packs differ"
    sched = build_schedule(packs, world, A, seed=d.seed, mode=d.schedule)
    rsched = rbuild_schedule(rpacks, world, A, seed=d.seed, mode=d.schedule)
    assert [s.rank_packs for s in sched.steps] == [s.rank_packs for s in rsched.steps], "schedules differ"

    torch.manual_seed(0)
    rmodel = RModelCls(rcfg.model)
    ours = LlamaForCausalLM(m)
    ours.load_state_dict(rmodel.state_dict())
    rmodel = wrap_model(rmodel, rcfg.train, dev)
    ropt = rtrain._make_optimizer(rmodel, rcfg)
    rlr = rtrain._make_scheduler(ropt, rcfg)
    engine = TrainEngine(cfg, dev, model=ours)
    ds, rds = PackedDataset(store, packs, d), RDataset(rstore, rpacks, rcfg.data)
    losses = []
    for step in range(t.max_steps):
        plan = sched.steps[step]
        ids = plan.rank_packs[rank]
        # reference step body (train/train.py:318-362) on its own modules
        ropt.zero_grad(set_to_none=True)
        local = torch.zeros(())
        for micro, i in enumerate(ids):
            with no_sync(rmodel, enabled=micro != A - 1):
                out = rtrain._forward_microbatch(rmodel, rds[i], dev, rcfg, need_block_mask=False)
                (out.loss * (world / plan.step_tokens)).backward()
            local += out.loss.detach()
        rtrain._clip_grads(rmodel, rcfg.train.grad_clip)
        ropt.step()
        rlr.step()
        ref_loss = float(rtrain._all_reduce_sum(local) / plan.step_tokens)
        o = engine.step([ds[i] for i in ids], plan.step_tokens)
        our_loss = float(engine.global_loss(o["loss_sum"], plan.step_tokens))
        losses.append((ref_loss, our_loss))
    if rank == 0:
        print("LOSSES " + json.dumps(losses), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    """
)


def test_config1_matches_reference_losses(tmp_path: Path) -> None:
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    port = str(_free_port())
    env = {**os.environ, "PB_ROOT": str(ROOT), "PB_REF": str(REF), "PB_TMP": str(tmp_path),
           "CUDA_VISIBLE_DEVICES": "", "OMP_NUM_THREADS": "1"}
    r = subprocess.run(
        ["timeout", "-k", "20", "280", sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
         "--master-addr=127.0.0.1", f"--master-port={port}", str(script)],
        env=env, capture_output=True, text=True, timeout=320,
    )
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-5000:]
    line = next(x for x in r.stdout.splitlines() if x.startswith("LOSSES "))
    losses = json.loads(line[len("LOSSES "):])
    assert len(losses) == 10
    for ref, ours in losses:
        assert abs(ref - ours) <= 2e-5 * abs(ref) + 1e-6, losses
    # the model trains: last loss below the first
    assert losses[-1][0] < losses[0][0]


@pytest.mark.parametrize("mode", ["pad", "pack_random", "pack_ffd", "isoflop"])
@pytest.mark.parametrize("schedule", ["random", "balanced"])
@pytest.mark.parametrize("world", [1, 4])
def test_packs_and_schedules_match_reference(tmp_path: Path, mode: str, schedule: str, world: int) -> None:
    """Every packing mode and both schedules give the reference's packs and step plans on
    a corpus with long (split) and one-token documents (no process group needed)."""
    import sys as _sys

    _sys.path.insert(1, str(REF))
    from packbalance.config import DataConfig as RData
    from packbalance.config import ModelConfig as RModel
    from packbalance.data.cost import FlopModel as RFlop
    from packbalance.data.packer import build_packs as rbuild_packs
    from packbalance.data.sampler import build_schedule as rbuild_schedule
    from packbalance.data.store import TokenStore as RStore

    from packbalance_b200.config import DataConfig, ModelConfig
    from packbalance_b200.data.cost import FlopModel
    from packbalance_b200.data.packer import build_packs
    from packbalance_b200.data.prepare import prepare_synthetic
    from packbalance_b200.data.sampler import build_schedule
    from packbalance_b200.data.store import TokenStore

    d = DataConfig(dataset="synthetic", data_dir=str(tmp_path / "c"), seq_len=96, mode=mode, schedule=schedule,
                   max_doc_len=96, min_doc_len=1, synthetic_num_docs=300, synthetic_mu=3.4, synthetic_sigma=1.1,
                   synthetic_min_len=1, synthetic_max_len=250, synthetic_vocab_size=97, num_workers=0,
                   val_fraction=0.1, seed=5, pad_batch_size=4)
    m = ModelConfig(vocab_size=97, d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=64, max_seq_len=96)
    prepare_synthetic(d, Path(d.data_dir))
    rd = RData(dataset="synthetic", data_dir=d.data_dir, seq_len=d.seq_len, mode=mode, schedule=schedule,
               max_doc_len=d.max_doc_len, min_doc_len=d.min_doc_len, val_fraction=d.val_fraction, seed=d.seed,
               num_workers=0, pad_batch_size=d.pad_batch_size)
    rm = RModel(vocab_size=m.vocab_size, d_model=m.d_model, n_layers=m.n_layers, n_heads=m.n_heads,
                n_kv_heads=m.n_kv_heads, d_ff=m.d_ff, max_seq_len=m.max_seq_len)
    key = lambda ps: [[(s.doc_id, s.start, s.length) for s in p.segments] for p in ps]  # noqa: E731
    built = {}
    for split in ("train", "val"):
        packs = build_packs(TokenStore.open(d.data_dir), d, FlopModel.from_config(m), split=split)
        rpacks = rbuild_packs(RStore.open(d.data_dir), rd, RFlop.from_config(rm), split=split)
        assert key(packs) == key(rpacks), (split, mode)
        built[split] = (packs, rpacks)
    packs, rpacks = built["train"]
    accum = 2
    sched = build_schedule(packs, world, accum, seed=d.seed, mode=schedule)
    rsched = rbuild_schedule(rpacks, world, accum, seed=d.seed, mode=schedule)
    assert len(sched.steps) > 0
    assert [s.rank_packs for s in sched.steps] == [s.rank_packs for s in rsched.steps]
    assert [s.step_tokens for s in sched.steps] == [s.step_tokens for s in rsched.steps]


def test_greedy_generation_matches_reference() -> None:
    """The KV-cache generate gives the reference's greedy continuation (which recomputes
    the whole prefix every token) from the same weights."""
    import sys as _sys

    import torch

    _sys.path.insert(1, str(REF))
    from packbalance.config import ModelConfig as RModel
    from packbalance.model.llama import LlamaForCausalLM as RModelCls

    from packbalance_b200.config import ModelConfig
    from packbalance_b200.models.llama import LlamaForCausalLM

    kw = dict(vocab_size=113, d_model=48, n_layers=2, n_heads=6, n_kv_heads=2, d_ff=80, max_seq_len=40)
    torch.manual_seed(4)
    ref = RModelCls(RModel(**kw, attention_backend="eager", use_fused_ce=False))
    ours = LlamaForCausalLM(ModelConfig(**kw, attention_backend="eager", use_fused_ce=False))
    ours.load_state_dict(ref.state_dict())
    prompt = torch.randint(1, 113, (2, 7), generator=torch.Generator().manual_seed(9))
    with torch.no_grad():
        a = ref.generate(prompt, max_new_tokens=20)
        b = ours.generate(prompt, max_new_tokens=20)
    assert torch.equal(a, b)
    # stops at max_seq_len like the reference
    with torch.no_grad():
        assert torch.equal(ref.generate(prompt, max_new_tokens=50), ours.generate(prompt, max_new_tokens=50))
