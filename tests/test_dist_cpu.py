"""The N > 1 path of bench.py on CPU: two ranks over gloo (127.0.0.1), as
torchrun launches them.  The replicas share nothing on the data path; the
process group aligns the timed regions and reduces the per-rank device times
to the max over ranks (the job's time), and the end-to-end rate to the
slowest rank's.  The reference arm runs on rank 0 only."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import bench
    ctx = bench._Dist()
    ctx.init("gloo")
    ms = [12.5, 15.0][rank]          # per-rank device time of the timed region
    e2e = [410.0, 395.0][rank]       # per-rank end-to-end steps/s
    ctx.barrier()
    job_ms = ctx.max(ms)
    slowest = -ctx.max(-e2e)
    ctx.barrier()
    ctx.close()
    q.put((rank, job_ms, slowest))


def test_two_gloo_ranks_reduce_to_the_slowest():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[0] for r in res] == [0, 1]
    for _, job_ms, slowest in res:
        assert job_ms == 15.0          # every rank sees the max over ranks
        assert slowest == 395.0        # and the slowest rank's end-to-end rate


def test_reference_arm_is_rank0_only(monkeypatch):
    """Under torchrun the reference arm runs (and prints) on rank 0 alone; the
    other ranks return at once without work."""
    import bench
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    ctx = bench._Dist()

    class _Args:
        steps, warmup, gpus = 1, 1, 2

    called = []
    monkeypatch.setattr(bench, "cpu_step_runner", lambda *a: called.append(1))
    assert bench.run_reference_arm(_Args(), ctx) is None
    assert called == []
