"""Host-side failure detection on gloo ranks (no GPU): a rank that raises, goes silent, never joins or
leaves is reported to its peers by the store before their next launch; a short process-group timeout
ends a collective that a peer skipped with an error instead of a hang."""
import time

import pytest

from conftest import free_port, run_gloo


def _raiser(rank, world):
    import torch.distributed as dist

    from comm_opt_b200.parallel.health import RankFailure, RankMonitor

    mon = RankMonitor.from_default_group(prefix="t1", stale_s=30)
    mon.wait_joined(30)
    dist.barrier()  # every rank is past its join before the failure is posted
    if rank == 2:
        with pytest.raises(ValueError):
            with mon.guard():
                raise ValueError("bad batch")
    dist.barrier()  # the failing rank has posted its notice (host-side; a real rank would exit here)
    if rank != 2:
        with pytest.raises(RankFailure) as ei:
            mon.check()
        assert set(ei.value.problems) == {2} and "ValueError: bad batch" in ei.value.problems[2]


def test_rank_that_raises_is_reported():
    run_gloo(_raiser, 3)


def _silent(rank, world):
    import torch.distributed as dist

    from comm_opt_b200.parallel.health import RankFailure, RankMonitor

    mon = RankMonitor.from_default_group(prefix="t2", stale_s=1.0)
    mon.wait_joined(30)
    dist.barrier()
    if rank == 1:
        return  # stops beating without a notice (a hung or killed process)
    t0 = time.monotonic()
    p = {}
    while time.monotonic() - t0 < 10 and 1 not in p:
        mon.beat()
        p = mon.problems()
        time.sleep(0.05)
    assert 1 in p and "no heartbeat" in p[1], p
    assert time.monotonic() - t0 >= 1.0  # not before the stale limit


def test_silent_rank_goes_stale():
    run_gloo(_silent, 3)


def _never_joins(rank, world):
    from comm_opt_b200.parallel.health import RankFailure, RankMonitor

    mon = RankMonitor.from_default_group(prefix="t3", stale_s=30)
    if rank == 2:
        return  # never beats
    with pytest.raises(RankFailure) as ei:
        mon.wait_joined(1.0)
    assert set(ei.value.problems) == {2} and "never joined" in ei.value.problems[2]


def test_rank_that_never_joins_is_reported():
    run_gloo(_never_joins, 3)


def _leaves(rank, world):
    import torch.distributed as dist

    from comm_opt_b200.parallel.health import RankFailure, RankMonitor

    mon = RankMonitor.from_default_group(prefix="t4", stale_s=30)
    mon.wait_joined(30)
    mon.check()  # everyone healthy
    dist.barrier()
    if rank == 0:
        mon.leave()
    dist.barrier()
    if rank != 0:
        with pytest.raises(RankFailure, match="rank 0: left the group"):
            mon.check()


def test_rank_that_leaves_is_reported():
    run_gloo(_leaves, 2)


def _skipped_collective(rank, world, port, q):
    import datetime
    import os

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=2))
    try:
        if rank == world - 1:
            time.sleep(4)  # skips the collective, stays alive past the others' timeout
            q.put((rank, "skipped"))
            return
        t0 = time.monotonic()
        try:
            dist.all_reduce(torch.ones(4))
            q.put((rank, "completed"))
        except RuntimeError:
            q.put((rank, f"error after {time.monotonic() - t0:.1f} s"))
    finally:
        dist.destroy_process_group()


def test_short_pg_timeout_ends_skipped_collective_with_error():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_skipped_collective, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung in the collective"
    got = {}
    while not q.empty():
        r, what = q.get()
        got[r] = what
    assert got[2] == "skipped"
    for r in (0, 1):
        assert got[r].startswith("error after"), got
        assert float(got[r].split()[2]) < 10


def _step_sync(rank, world):
    from comm_opt_b200.parallel.health import RankFailure, RankMonitor

    mon = RankMonitor.from_default_group(prefix="t5", stale_s=30)
    mon.wait_joined(30)
    done = 0
    for step in range(5):
        if rank == world - 1 and step == 2:
            mon.leave()  # between steps, nothing in flight
            break
        try:
            mon.sync(30)
        except RankFailure as e:
            assert set(e.problems) == {world - 1} and "left" in e.problems[world - 1]
            break
        done += 1
    assert done == 2, (rank, done)  # every rank completed steps 0 and 1, no rank launched step 2


def test_step_sync_stops_every_rank_at_the_same_step():
    run_gloo(_step_sync, 3)
