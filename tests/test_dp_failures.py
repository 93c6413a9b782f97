"""Failure handling of the encoder's batch data parallelism, made on the host
with gloo ranks on CPU (no device is faulted, trapped or hung):

  - a rank that leaves between steps: the others learn it from the store
    before their next step and stop with PeerLeft;
  - a rank that dies without saying so: a short process-group timeout (or
    the closed connection) ends the survivor's next collective with an error
    instead of a hang;
  - a peer that never joins: init_process_group gives up after its timeout;
  - a mismatched batch split: every rank rejects it before any collective.

The reference has no multi-process code; errors surface there as a non-zero
exit status of the CLI (src/cli/main.cpp:365-383), which is what the worker
processes report here too."""
import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferc_b200 import dp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _step(total, world, rank):
    s, e = dp.shard_rows(total, world, rank)
    local = torch.arange(s * 2, e * 2, dtype=torch.float32).reshape(e - s, 2)
    return dp.gather_logits(local, total)


def _leaver(rank, world, port, q):
    _init(rank, world, port, 20)
    store = dist.distributed_c10d._get_default_store()
    m = dp.Membership(store, world, rank)
    try:
        for step in range(5):
            if rank == 1 and step == 2:
                m.leave()  # between steps: nothing of this rank is in flight
                q.put((rank, "left"))
                return
            if rank == 0 and step == 2:
                # learn of the departure on the host before the next launch
                store.wait([f"{m.prefix}1"], datetime.timedelta(seconds=15))
            m.check()
            _step(10, world, rank)
        q.put((rank, "finished"))
    except dp.PeerLeft as e:
        q.put((rank, f"peer-left {e.ranks}"))
    finally:
        dist.destroy_process_group()


def test_rank_leaves_between_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode == 0
    got = dict(q.get(timeout=5) for _ in range(2))
    assert got == {0: "peer-left [1]", 1: "left"}


def _dier(rank, world, port, q):
    _init(rank, world, port, 3)
    _step(8, world, rank)
    if rank == 1:
        os._exit(0)  # dies without telling anyone, between steps
    t0 = time.monotonic()
    try:
        _step(8, world, rank)
        q.put(("no error", time.monotonic() - t0))
    except Exception as e:  # gloo: connection closed or timeout
        q.put((type(e).__name__, time.monotonic() - t0))
    # os._exit skips the queue's feeder thread: flush the result first
    q.close()
    q.join_thread()
    os._exit(0)


def test_dead_peer_ends_next_collective_with_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dier, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    kind, waited = q.get(timeout=5)
    assert kind != "no error"
    assert waited < 30


def _lonely(port, q):
    t0 = time.monotonic()
    try:
        _init(0, 2, port, 2)  # rank 1 never starts
        q.put(("joined", 0.0))
    except Exception as e:
        q.put((type(e).__name__, time.monotonic() - t0))


def test_init_times_out_when_a_peer_never_joins():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    p.join(90)
    kind, waited = q.get(timeout=5)
    assert kind != "joined"
    assert waited < 60


def _mismatch(rank, world, port, q):
    _init(rank, world, port, 20)
    try:
        local = torch.zeros(3, 2)  # 10 rows over 2 ranks is 5 + 5, not 3
        dp.gather_logits(local, 10)
        q.put((rank, "accepted"))
    except ValueError as e:
        q.put((rank, "rejected" if "expected 5" in str(e) else str(e)))
    finally:
        dist.destroy_process_group()


def test_mismatched_batch_split_is_rejected_before_the_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mismatch, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode == 0
    assert dict(q.get(timeout=5) for _ in range(2)) == {0: "rejected", 1: "rejected"}


def test_shard_rows_rejects_bad_arguments():
    import pytest
    for args in [(8, 0, 0), (8, 2, 2), (8, 2, -1), (-1, 2, 0)]:
        with pytest.raises(ValueError):
            dp.shard_rows(*args)
