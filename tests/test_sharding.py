"""Host-side multi-GPU logic on CPU: world-size-2 `gloo` ranks check that slot ranges are
disjoint and cover the job, that prefix streams do not depend on the world size, and
that the timing reduction returns the slowest rank's time on every rank."""
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from conftest import load_package
        load_package()
        from qasr_b200 import sharding
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        mine = list(sharding.slot_range(rank, world, 32))
        times = [0.5 + rank, 2.0 - rank]
        out = sharding.max_over_ranks(times, dist)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        dist.destroy_process_group()
        q.put((rank, out, gathered))
    except Exception as e:  # report instead of dying silently
        q.put((rank, repr(e), None))


def test_two_rank_slot_sharding(qasr):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=90) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out, gathered in results:
        assert gathered is not None, f"rank {rank} failed: {out}"
        assert out == [1.5, 2.0]  # max over ranks, element-wise
        flat = sorted(s for r in gathered for s in r)
        assert flat == list(range(64))
        assert set(gathered[0]).isdisjoint(gathered[1])


def test_prefix_streams_independent_of_world(qasr):
    from qasr_b200 import sharding
    assert sharding.prefix_stream(40, 2) == 40 * 65536 + 2
    assert list(sharding.slot_range(1, 8, 32)) == list(range(32, 64))
    with pytest.raises(ValueError):
        sharding.slot_range(8, 8, 32)


def _dying_worker(rank, world, port, q):
    """Rank 1 leaves between steps (an exception on the host, nothing in flight); rank 0
    then enters the post-timing MAX reduction and must get an error, not wait forever."""
    import time
    try:
        import datetime

        import torch.distributed as dist
        from conftest import load_package
        load_package()
        from qasr_b200 import sharding
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        sharding.max_over_ranks([1.0], dist)  # one good step on both ranks
        if rank == 1:
            raise RuntimeError("rank 1 failed between steps")
        t0 = time.monotonic()
        try:
            sharding.max_over_ranks([2.0], dist)
            q.put((rank, "no error", time.monotonic() - t0))
        except Exception as e:  # the peer is gone: the collective ends with an error
            q.put((rank, type(e).__name__, time.monotonic() - t0))
    except Exception as e:
        q.put((rank, "left: " + repr(e), 0.0))


def test_a_rank_that_leaves_is_an_error_on_the_others(qasr):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (what, dt)) for r, what, dt in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    assert results[1][0].startswith("left: RuntimeError")
    what, dt = results[0]
    print(f"surviving rank: {what} after {dt:.1f} s")
    assert what != "no error", results
    assert dt < 60, results  # bounded by the group's timeout, not a hang
