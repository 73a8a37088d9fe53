"""Rank failure detected on the host, with CPU processes only: a rank that
stops making progress or declares failure is named by RankHealth within its
timeout, and a collective that a dead rank never joins ends with an error at
the process group's (short) timeout instead of hanging.  Nothing here touches
a GPU."""
import os
import socket
import time

import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _paths():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen3-vl_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)


def _health_worker(rank, world, port, scenario, q):
    _paths()
    import torch.distributed as dist
    from q3vl.health import RankFailure, RankHealth
    store = dist.TCPStore("127.0.0.1", port, world, is_master=(rank == 0),
                          timeout=__import__("datetime").timedelta(seconds=30))
    h = RankHealth(store, rank, world)
    try:
        for step in range(4):
            if rank == 1 and scenario == "stall" and step == 2:
                time.sleep(4)        # stops beating (as a rank that died would)
                return
            if rank == 1 and scenario == "declare" and step == 2:
                h.fail("out of memory in step 2")
                return
            h.beat(step)
            if rank == 0:
                h.wait_for_peers(step, timeout_s=1.5)
        if rank == 0:
            q.put(("ok", None))
    except RankFailure as e:
        q.put(("failure", (e.rank, e.reason)))


def _run(scenario):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_health_worker, args=(r, 2, port, scenario, q))
             for r in range(2)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    res = q.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
    return res, time.monotonic() - t0


def test_tick_numbers_keep_growing_across_loops():
    _paths()
    from q3vl.health import RankHealth

    class Store(dict):
        def set(self, k, v):
            self[k] = v.encode()

        def get(self, k):
            return dict.__getitem__(self, k)

        def check(self, keys):
            return all(k in self for k in keys)

    h = RankHealth(Store(), 0, 1)
    assert [h.tick() for _ in range(3)] == [0, 1, 2]
    assert [h.tick() for _ in range(2)] == [3, 4]      # a second loop continues the count


def test_healthy_ranks_pass_every_step():
    res, _ = _run("none")
    assert res == ("ok", None)


def test_a_stalled_rank_is_named_within_the_timeout():
    res, elapsed = _run("stall")
    assert res[0] == "failure" and res[1][0] == 1 and "no heartbeat for step 2" in res[1][1]
    assert elapsed < 30


def test_a_declared_failure_is_reported_with_its_reason():
    res, _ = _run("declare")
    assert res[0] == "failure" and res[1] == (1, "failed: out of memory in step 2")


def _collective_worker(rank, world, port, q):
    _paths()
    import datetime
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)                    # both ranks alive
    if rank == 1:
        os._exit(0)                        # leaves between steps, without a word
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        q.put(("returned", time.monotonic() - t0))
    except Exception as e:  # the collective's timeout or a closed peer connection
        q.put(("error", time.monotonic() - t0, type(e).__name__))


def test_a_collective_with_a_departed_rank_errors_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_collective_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[0] == "error" and res[1] < 30
