"""The multi-rank path of bench.py on CPU: two gloo ranks (torchrun-style environment, 127.0.0.1) take the
same collective steps; the slowest rank's time and the whole-job rate come out the same on every rank; the
reference arm runs on rank 0 only; a rank that dies or hangs between steps ends the survivor's next collective
with an error within the process-group timeout instead of a hang."""

import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(REPO))
    import bench
    import torch.distributed as dist
    r, w, _ = bench.dist_env()
    bench.init_ranks(w, "gloo")
    ms = bench.max_over_ranks(10.0 + 5.0 * r, w)   # rank 1 is the slow one
    rate = bench.whole_job_rate(64, w, 10, ms)
    dist.barrier()
    dist.destroy_process_group()
    q.put((r, ms, rate))


def test_two_gloo_ranks_agree_on_slowest_time_and_rate():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=600) for _ in range(world))  # a cold first torch import can take a minute
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [o[1] for o in out] == [15.0, 15.0]
    assert all(abs(o[2] - 64 * 2 * 10 / 0.015) < 1e-6 for o in out)


def test_reference_arm_runs_on_rank_zero_only(capsys):
    sys.path.insert(0, str(REPO))
    import bench
    assert bench.run_reference(None, 1, 2) == 0
    assert capsys.readouterr().out == ""


def _failing_rank(rank: int, world: int, port: int, mode: str, q, start) -> None:
    """Step 1 together; then rank 1 exits ("exit") or stops answering ("hang"), and rank 0 takes step 2.  The
    ranks meet at `start` after their imports (a cold first torch import can take a minute) so that the 5 s
    process-group timeout is not spent on one rank's start-up."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, str(REPO))
    import bench
    r, w, _ = bench.dist_env()
    start.wait(timeout=600)
    bench.init_ranks(w, "gloo", timeout_s=5)
    bench.max_over_ranks(1.0, w)                 # step 1: both ranks
    if r == 1:
        if mode == "exit":
            os._exit(0)                           # dies between steps, no collective in flight
        time.sleep(60)                            # hangs between steps
        os._exit(0)
    t0 = time.perf_counter()
    try:
        bench.max_over_ranks(2.0, w)             # step 2: the peer is gone
        q.put(("no error", time.perf_counter() - t0))
    except Exception as exc:  # noqa: BLE001 - any error ends the step, which is the point
        q.put((type(exc).__name__, time.perf_counter() - t0))
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "hang"])
def test_survivor_errors_within_the_timeout_when_a_rank_dies_or_hangs(mode):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    start = ctx.Barrier(world)
    procs = [ctx.Process(target=_failing_rank, args=(r, world, port, mode, q, start)) for r in range(world)]
    for p in procs:
        p.start()
    kind, elapsed = q.get(timeout=660)
    for p in procs:
        p.join(timeout=90)
        if p.is_alive():
            p.kill()
    assert kind != "no error"
    assert elapsed < 60, elapsed                  # the 5 s timeout (plus teardown), not a hang
