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
    ar = FusedAllReduce(grad, mode=os.environ["PB_ALLREDUCE"])
    if rank == 0:
        print("mode", ar.mode, "tail", ar.tail_mode)
    for step in range(3):
        ar.buf.copy_(grad)
        ar.start_step()
        # a 4-element bucket, a bucket smaller than one CTA's share, large ones; narrow
        # (beside-compute) and wide (tail) launches, both kernels when the tail kernel differs
        cuts = [0, 4, 1000, 2_000_000, n]
        for i, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:])):
            ar.all_reduce_mean(lo, hi, tail=(i + step) % 2 == 1)
        torch.cuda.synchronize()
        _native.check_status()
        err = (ar.buf - ref).abs().max().item()
        assert err < 1e-5, err
        ss = ar.sumsq.item()
        assert abs(ss - ref.square().sum().item()) < 1e-3 * ss, (ss, ref.square().sum().item())
    ar.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank} ok", flush=True)  # one write: ranks do not interleave
    """
)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["p2p", "auto"])
def test_fused_allreduce_matches_nccl(tmp_path, mode):
    world = min(torch.cuda.device_count(), 8)
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = {**os.environ, "PB_ROOT": str(ROOT), "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()),
           "NCCL_NVLS_ENABLE": "0", "PB_ALLREDUCE": mode}
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
