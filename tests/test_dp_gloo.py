"""Multi-process (world size 2, gloo on CPU) test of the encoder's batch
data parallelism: each rank computes logits for its shard and rank 0
receives the whole batch in order. Same code path as the NCCL run."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferc_b200 import dp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, total, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        full = torch.arange(total * 2, dtype=torch.float32).reshape(total, 2)
        s, e = dp.shard_rows(total, world, rank)
        out = dp.gather_logits(full[s:e].clone(), total)
        if rank == 0:
            result_q.put(bool(torch.equal(out, full)))
        else:
            result_q.put(out is None)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("total", [8, 7, 1])
def test_gather_logits_world2(total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, total, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert q.get(timeout=5) and q.get(timeout=5)
