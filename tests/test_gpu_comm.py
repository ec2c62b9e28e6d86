"""Fused peer-memory all-reduce: numerics against NCCL on 2+ GPUs, and the bounded
barrier wait on one GPU (a peer that never arrives -> error status, no hang)."""

import os
import socket
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


WORKER = textwrap.dedent(
    """
    import os, sys, datetime, torch, torch.distributed as dist
    sys.path.insert(0, os.environ["PB_ROOT"])
    from packbalance_b200.parallel.comm import FusedAllReduce
    from packbalance_b200.ops import _native
    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    n = 3 * 1000 * 1000 + 13  # ragged end: the last bucket is not a multiple of 16 bytes
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    grad = torch.randn(n, device="cuda", generator=g)
    ref = grad.clone()
    dist.all_reduce(ref)
    ref /= world
    wire = os.environ.get("PB_WIRE", "fp32")
    ar = FusedAllReduce(grad, mode=os.environ["PB_ALLREDUCE"], wire=wire)
    if rank == 0:
        print("mode", ar.mode, "tail", ar.tail_mode, "wire", ar.wire)
    # bf16 wire: each rank's input and the average are rounded to bf16 (relative error at
    # most 2^-8 each); sums are fp32.  Bound per element: 2^-8 (mean |g_p| + |average|).
    abs_mean = grad.abs()
    dist.all_reduce(abs_mean)
    abs_mean /= world
    bound = 1.01 * 2.0 ** -8 * (abs_mean + ref.abs()) + 1e-30
    for step in range(3):
        ar.buf.copy_(grad)
        ar.start_step()
        # an 8-element bucket, a bucket smaller than one CTA's share, large ones; narrow
        # (beside-compute) and wide (tail) launches, both kernels when the tail kernel differs
        cuts = [0, 8, 1000, 2_000_000, n]
        for i, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:])):
            ar.all_reduce_mean(lo, hi, tail=(i + step) % 2 == 1)
        torch.cuda.synchronize()
        _native.check_status()
        if wire == "fp32":
            err = (ar.buf - ref).abs().max().item()
            assert err < 1e-5, err
        else:
            over = ((ar.buf - ref).abs() > bound).sum().item()
            assert over == 0, (over, (ar.buf - ref).abs().max().item())
            # identical on every rank (each rank keeps the rounded average, not its fp32 sum)
            mine = ar.buf.double().sum()
            other = mine.clone()
            dist.all_reduce(other, op=dist.ReduceOp.MAX)
            assert mine.item() == other.item()
        ss = ar.sumsq.item()
        ref_ss = ar.buf.square().sum().item() if wire == "bf16" else ref.square().sum().item()
        assert abs(ss - ref_ss) < 1e-3 * ss, (ss, ref_ss)
    ar.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)  # one write: ranks do not interleave
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode,wire", [("p2p", "fp32"), ("auto", "fp32"), ("auto", "bf16")])
def test_fused_allreduce_matches_nccl(tmp_path, mode, wire):
    world = min(torch.cuda.device_count(), 8)
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = {**os.environ, "PB_ROOT": str(ROOT), "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()),
           "NCCL_NVLS_ENABLE": "0", "PB_ALLREDUCE": mode, "PB_WIRE": wire}
    r = subprocess.run(
        ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
         f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={env['MASTER_PORT']}", str(script)],
        env=env, capture_output=True, text=True, timeout=300,
    )
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("ok") == world
    print(r.stdout[:200])


def test_barrier_timeout_reports_status():
    """World of 2 on one GPU: the second 'peer' never arrives, so barrier 0 gives up
    after its bounded wait and records status 401 + 1000 * peer; the context stays usable."""
    from packbalance_b200.ops import _native

    C = _native.module()
    dev = torch.device("cuda")
    buf = torch.zeros(1024, device=dev)
    pads = torch.zeros(2, 3 * 32 * 2, device=dev, dtype=torch.int32)
    ptrs = torch.tensor([buf.data_ptr(), buf.data_ptr()], device=dev, dtype=torch.int64)
    pad_ptrs = torch.tensor([pads[0].data_ptr(), pads[1].data_ptr()], device=dev, dtype=torch.int64)
    sumsq = torch.zeros((), device=dev)
    C.status_read(dev.index or 0, True)
    C.fused_allreduce(ptrs.data_ptr(), pad_ptrs.data_ptr(), pads.shape[1], 0, 1024, 0, 2, 1, 0.5, sumsq, 4, 0)
    torch.cuda.synchronize()
    code = C.status_read(dev.index or 0, True)
    assert code == 401 + 1000 * 1, code
    # the device still works
    assert torch.ones(4, device=dev).sum().item() == 4.0


TRAIN_WORKER = textwrap.dedent(
    """
    import os, sys, datetime, json, torch, torch.distributed as dist
    from dataclasses import replace
    sys.path.insert(0, os.environ["PB_ROOT"])
    from packbalance_b200.config import ModelConfig, PackBalanceConfig, TrainConfig
    from packbalance_b200.data.dataset import doc_starts_from_ids
    from packbalance_b200.train.engine import TrainEngine
    rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    g = torch.Generator().manual_seed(10 + rank)
    lengths = [900, 400, 748]
    ids = torch.randint(1, 2048, (sum(lengths),), generator=g)
    doc = torch.cat([torch.full((n,), i) for i, n in enumerate(lengths)])
    pos = torch.cat([torch.arange(n) for n in lengths])
    labels = torch.cat([ids[1:], torch.tensor([-100])])
    labels[torch.cumsum(torch.tensor(lengths), 0) - 1] = -100
    batch = dict(input_ids=ids, labels=labels, position_ids=pos, doc_ids=doc,
                 doc_start=torch.from_numpy(doc_starts_from_ids(doc.numpy())))
    tokens = int((labels != -100).sum()) * world
    base = PackBalanceConfig(model=ModelConfig(vocab_size=2048, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2,
                                               d_ff=512, max_seq_len=2048),
                             train=TrainConfig(lr=2e-3, warmup_steps=1, max_steps=20))
    losses = {}
    for wire in ("fp32", "bf16"):
        torch.manual_seed(0)
        eng = TrainEngine(replace(base, train=replace(base.train, grad_reduce_dtype=wire)), dev)
        out = []
        for step in range(10):
            o = eng.step([batch], tokens)
            out.append(float(eng.global_loss(o["loss_sum"], tokens)))
        losses[wire] = out
        eng.close()
    if rank == 0:
        print("LOSSES " + json.dumps(losses), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_bf16_wire_training_tracks_fp32(tmp_path):
    """Ten steps with the bf16-wire all-reduce follow the fp32 run's losses."""
    import json

    world = min(torch.cuda.device_count(), 8)
    script = tmp_path / "train_worker.py"
    script.write_text(TRAIN_WORKER)
    env = {**os.environ, "PB_ROOT": str(ROOT), "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()),
           "NCCL_NVLS_ENABLE": "0"}
    r = subprocess.run(
        ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
         f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={env['MASTER_PORT']}", str(script)],
        env=env, capture_output=True, text=True, timeout=360,
    )
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = next(x for x in r.stdout.splitlines() if x.startswith("LOSSES "))
    losses = json.loads(line[len("LOSSES "):])
    for a, b in zip(losses["fp32"], losses["bf16"]):
        assert abs(a - b) <= 1e-2 * abs(a), losses
    assert losses["bf16"][-1] < losses["bf16"][0]
