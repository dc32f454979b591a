"""The bench's multi-process plumbing on CPU: two gloo ranks agree on the
max-over-ranks time and on one printed line (rank 0 only)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    # Each rank's own step time; the reported time is the max over ranks.
    mine = torch.tensor([1.0 + rank], dtype=torch.float64)
    dist.all_reduce(mine, op=dist.ReduceOp.MAX)
    dist.barrier()
    q.put((rank, float(mine.item())))
    dist.destroy_process_group()


def test_max_over_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    assert got == [(0, 2.0), (1, 2.0)]


def test_reference_arm_other_ranks_exit_quietly(monkeypatch, capsys):
    import bench
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")

    class A:
        steps, warmup = 1, 3
    bench.run_reference(A())
    assert capsys.readouterr().out == ""
