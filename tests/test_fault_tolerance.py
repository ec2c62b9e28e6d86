"""Failure handling on the host (no GPU): a rank that dies ends the survivors' next
collective with an error within the process-group timeout instead of hanging them."""

import datetime
import multiprocessing as mp
import os
import socket
import time


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _worker(rank: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE="2",
                      LOCAL_RANK=str(rank), CUDA_VISIBLE_DEVICES="")
    import torch
    import torch.distributed as dist

    from packbalance_b200.parallel.distributed import init_distributed

    init_distributed("cpu", timeout_s=5.0)
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks alive: succeeds
    if rank == 1:
        os._exit(3)  # dies between steps, with nothing in flight
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        q.put(("no error", time.monotonic() - t0))
    except Exception as exc:  # noqa: BLE001 - any error type is the expected outcome
        q.put((type(exc).__name__, time.monotonic() - t0))


def test_dead_rank_ends_next_collective_with_error() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        kind, waited = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert kind != "no error"
    assert waited < 60.0, waited
