"""Checkpoints move between the reference and this framework in both directions.

Two gloo ranks on CPU (fp32).  The same starting weights and the same batch on both
sides:

* ``state.pt`` (DDP / single process): the reference trains one step with its own model
  and ``torch.optim.AdamW`` and writes the file with its own ``save_checkpoint``; this
  framework's ``load_checkpoint`` restores it into a ``TrainEngine``; both take one more
  identical step and end at the same weights.  Then the reverse: ``TrainEngine`` writes,
  the reference's ``load_checkpoint`` reads, weights and Adam moments agree.
* DCP directory (FSDP): the same round trip between the reference's FSDP2 model and a
  ``TrainEngine`` with ``train.fsdp`` on.

Skipped when the reference cannot be found
(``packbalance_b200.utils.reference.locate_reference``).
"""

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
    import os, sys
    from pathlib import Path
    import torch, torch.distributed as dist
    sys.path.insert(0, os.environ["PB_ROOT"])
    sys.path.insert(1, os.environ["PB_REF"])
    torch.set_num_threads(1)
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    cpu = torch.device("cpu")
    FSDP = os.environ["PB_FSDP"] == "1"
    TMP = Path(os.environ["PB_TMP"])

    from packbalance_b200.config import DataConfig, ModelConfig, PackBalanceConfig, TrainConfig
    from packbalance_b200.models.llama import LlamaForCausalLM
    from packbalance_b200.train.checkpoint import load_checkpoint, save_checkpoint
    from packbalance_b200.train.engine import TrainEngine

    from packbalance.config import ModelConfig as RModel, PackBalanceConfig as RCfg, TrainConfig as RTrain
    from packbalance.model.llama import LlamaForCausalLM as RModelCls
    from packbalance.train import train as rtrain
    from packbalance.train.checkpoint import load_checkpoint as rload, save_checkpoint as rsave
    from packbalance.train.distributed import wrap_model

    mk = dict(vocab_size=97, d_model=32, n_layers=2, n_heads=4, n_kv_heads=2, d_ff=56, max_seq_len=40,
              attention_backend="eager", use_fused_ce=False, ce_chunk_size=16)
    tk = dict(lr=2e-3, min_lr=2e-3, warmup_steps=0, max_steps=50, weight_decay=0.05, grad_clip=1.0, dtype="fp32",
              fsdp=FSDP, grad_accum=1)
    cfg = PackBalanceConfig(model=ModelConfig(**mk), data=DataConfig(seq_len=40), train=TrainConfig(**tk))
    rcfg = RCfg(model=RModel(**mk), train=RTrain(**tk))

    # one fixed batch, identical on both ranks: 3 documents in a 40-token pack
    g = torch.Generator().manual_seed(5)
    lens = [13, 19, 8]
    ids = torch.randint(1, 97, (40,), generator=g)
    doc = torch.cat([torch.full((n,), i) for i, n in enumerate(lens)])
    pos = torch.cat([torch.arange(n) for n in lens])
    labels = torch.cat([ids[1:], torch.tensor([-100])])
    ends = torch.cumsum(torch.tensor(lens), 0) - 1
    labels[ends] = -100
    batch = dict(input_ids=ids, labels=labels, position_ids=pos, doc_ids=doc)
    useful = int((labels != -100).sum())
    step_tokens = world * useful

    def ref_step(model, opt):
        opt.zero_grad(set_to_none=True)
        out = model(ids[None], labels=labels[None], position_ids=pos[None], doc_ids=doc[None])
        (out.loss * (world / step_tokens)).backward()
        rtrain._clip_grads(model, 1.0)
        opt.step()

    def full(t):
        return t.full_tensor() if hasattr(t, "full_tensor") else t

    def params(model):
        raw = getattr(model, "module", model)  # the reference's DDP wrapper
        return {k: full(v).detach().clone() for k, v in raw.state_dict().items()}

    def close(a, b, tol):
        assert a.keys() == b.keys(), (sorted(a)[:3], sorted(b)[:3])
        for k in a:
            torch.testing.assert_close(a[k], b[k], atol=tol, rtol=tol, msg=k)

    torch.manual_seed(0)
    init = RModelCls(rcfg.model).state_dict()

    # ---- reference writes, we read --------------------------------------------
    rmodel = RModelCls(rcfg.model)
    rmodel.load_state_dict(init)
    rmodel = wrap_model(rmodel, rcfg.train, cpu)
    ropt = rtrain._make_optimizer(rmodel, rcfg)
    rtrain._make_scheduler(ropt, rcfg)  # as the reference trainer does (adds initial_lr)
    ref_step(rmodel, ropt)
    d_ref = TMP / ("ref_fsdp" if FSDP else "ref_ddp")
    rsave(rmodel, ropt, 3, d_ref, fsdp=FSDP)
    dist.barrier()

    ours = LlamaForCausalLM(cfg.model)
    eng = TrainEngine(cfg, cpu, model=ours)
    meta = load_checkpoint(d_ref / "step_0000003", eng.model, eng.optimizer, fsdp=eng.fsdp, device=cpu)
    assert meta["step"] == 3, meta
    close(params(eng.model), params(rmodel), 0.0)
    # one more identical step on both sides
    ref_step(rmodel, ropt)
    eng.step([dict(batch)], step_tokens)
    close(params(eng.model), params(rmodel), 2e-5)

    # ---- we write, reference reads --------------------------------------------
    d_ours = TMP / ("ours_fsdp" if FSDP else "ours_ddp")
    save_checkpoint(eng.model, eng.optimizer, 5, d_ours, fsdp=eng.fsdp)
    dist.barrier()
    rmodel2 = RModelCls(rcfg.model)
    rmodel2 = wrap_model(rmodel2, rcfg.train, cpu)
    ropt2 = rtrain._make_optimizer(rmodel2, rcfg)
    # the reference's loader fills the optimizer's existing state in place, so its
    # AdamW state must exist first
    ref_step(rmodel2, ropt2)
    rmeta = rload(d_ours / "step_0000005", rmodel2, ropt2, fsdp=FSDP, device=cpu)
    assert int(rmeta["step"]) == 5, rmeta
    close(params(rmodel2), params(eng.model), 0.0)
    # the Adam moments came across too: one more step on both sides stays together
    ref_step(rmodel2, ropt2)
    eng.step([dict(batch)], step_tokens)
    close(params(rmodel2), params(eng.model), 2e-5)
    dist.barrier()
    if rank == 0:
        print("INTEROP OK", flush=True)
    dist.destroy_process_group()
    """
)


@pytest.mark.parametrize("fsdp", [False, True])
def test_checkpoints_cross_between_frameworks(tmp_path: Path, fsdp: bool) -> None:
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = {**os.environ, "PB_ROOT": str(ROOT), "PB_REF": str(REF), "PB_TMP": str(tmp_path),
           "PB_FSDP": "1" if fsdp else "0", "CUDA_VISIBLE_DEVICES": "", "OMP_NUM_THREADS": "1"}
    r = subprocess.run(
        ["timeout", "-k", "20", "280", sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
         "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(script)],
        env=env, capture_output=True, text=True, timeout=320,
    )
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-5000:]
    assert "INTEROP OK" in r.stdout
