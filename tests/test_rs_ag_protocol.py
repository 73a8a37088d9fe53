"""The prefill two-shot all-reduce protocol (tests/rs_ag_protocol_model.py),
with ranks as threads: exact sums on every rank over repeated calls while
ranks drift apart, and a rank that never pushes is reported by the owners
of its tiles within the wait limit instead of hanging anyone.  CPU only."""
import random
import threading

import pytest

from tests.rs_ag_protocol_model import PUSH_TIMEOUT, GATHER_TIMEOUT, TwoShot


def _run(ex, calls, seed, skip=None):
    world, rows, cols = ex.world, ex.rows, ex.cols
    outs = [[None] * calls for _ in range(world)]
    inputs = []
    g = random.Random(seed)
    for k in range(calls):
        parts = [[[g.randint(-50, 50) for _ in range(cols)] for _ in range(rows)]
                 for _ in range(world)]
        res = [[g.randint(-50, 50) for _ in range(cols)] for _ in range(rows)]
        inputs.append((parts, res))

    def rank(r):
        rng = random.Random(seed * 31 + r)
        for k in range(calls):
            if rng.random() < 0.3:
                threading.Event().wait(rng.random() * 0.004)   # drift between calls
            parts, res = inputs[k]
            outs[r][k] = ex.call(r, parts[r], res, rng, skip_push=(skip == (r, k)))

    ts = [threading.Thread(target=rank, args=(r,)) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    assert not any(t.is_alive() for t in ts), "a rank hung"
    return outs, inputs


@pytest.mark.parametrize("world,rows", [(2, 9), (3, 13), (4, 7), (8, 20)])
def test_every_rank_gets_the_exact_sum_over_drifting_calls(world, rows):
    for seed in range(4):
        ex = TwoShot(world, rows, cols=3)
        outs, inputs = _run(ex, calls=6, seed=seed)
        assert ex.errors == [0] * world
        for k, (parts, res) in enumerate(inputs):
            want = [[res[i][c] + sum(parts[r][i][c] for r in range(world)) for c in range(3)]
                    for i in range(rows)]
            for r in range(world):
                assert outs[r][k] == want, (world, rows, seed, k, r)


def test_a_rank_that_never_pushes_is_reported_without_a_hang():
    world, rows = 3, 12
    ex = TwoShot(world, rows, cols=2, wait_limit_s=0.2)
    _, _ = _run(ex, calls=2, seed=5, skip=(1, 1))
    # every owner missed rank 1's partials of call 2; rank 1's own stripe
    # still reduced, so the others' gathers of it completed or ran out
    assert all(e in (PUSH_TIMEOUT, GATHER_TIMEOUT) for r, e in enumerate(ex.errors) if r != 1)
    assert ex.errors[0] == PUSH_TIMEOUT and ex.errors[2] == PUSH_TIMEOUT


def test_one_buffer_would_do():
    """The two phases already order every reuse: a rank pushes call f + 1 only
    after gathering all of call f, so with one buffer instead of two per
    parity the sums stay exact (the kernel keeps two as a margin)."""
    for seed in range(6):
        ex = TwoShot(3, 13, cols=3, parity=False)
        outs, inputs = _run(ex, calls=8, seed=seed)
        assert ex.errors == [0, 0, 0]
        for k, (parts, res) in enumerate(inputs):
            want = [[res[i][c] + sum(parts[r][i][c] for r in range(3)) for c in range(3)]
                    for i in range(13)]
            assert all(outs[r][k] == want for r in range(3))
