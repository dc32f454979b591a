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


def test_row_blocks_cover_every_element_once():
    import bench
    for world in (1, 2, 3, 4, 8):
        blocks = [bench.row_block(world, r) for r in range(world)]
        assert blocks[0][0] == 0 and blocks[-1][1] == bench.N
        for (a, b), (c, d) in zip(blocks, blocks[1:]):
            assert b == c and a < b and a % 4096 == 0
        assert sum(b - a for a, b in blocks) == bench.N


def _rank_wait(rank, world, port, q):
    import datetime
    import time
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench
    if rank == 0:
        time.sleep(1.0)            # rank 0 "runs the pass" meanwhile
    t0 = time.monotonic()
    bench.wait_for_rank0(world, rank, "pass_done")
    dist.barrier()
    q.put((rank, time.monotonic() - t0))
    dist.destroy_process_group()


def test_other_ranks_wait_on_the_host_for_rank0():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_wait, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        assert p.exitcode == 0
    waited = dict(q.get(timeout=10) for _ in range(2))
    assert waited[1] >= 0.8          # rank 1 waited for rank 0's key
