"""The in-kernel all-reduce's exchange protocol (flag-in-word inbox words,
per-tile call counters, parity double buffering, bounded polls) on a host
model of it (tests/ar_protocol_model.py), CPU only.  Faults are injected on
the host: a rank that skips its pushes, or pushes a stale or future call
number.  Receivers must return within the wait limit with the timeout code
recorded, never hang; a fresh exchange then works again."""
import random
import time

import pytest

from tests.ar_protocol_model import TIMEOUT_CODE, Exchange, run_ranks

WORLD, TILES, WORDS = 4, 3, 8


def payload(rank, call, tile):
    return [(rank + 1) * 1000 + call * 10 + tile + w for w in range(WORDS)]


def expected(call, tile):
    return [sum(payload(r, call, tile)[w] for r in range(WORLD)) for w in range(WORDS)]


def test_repeated_calls_reduce_exactly_on_every_rank():
    ex = Exchange(WORLD, TILES, WORDS)

    def rank_fn(r):
        got = []
        for call in range(6):
            for tile in range(TILES):
                got.append(ex.call(r, tile, payload(r, call, tile)))
        return got

    outs = run_ranks(ex, rank_fn, WORLD)
    want = [expected(c, t) for c in range(6) for t in range(TILES)]
    assert all(o == want for o in outs)
    assert ex.errors == [0] * WORLD


def test_parity_buffers_let_ranks_drift_one_call_apart():
    """Random delays before each push: a rank that finished call c may push
    call c+1 while a slower rank still reads call c's words; the two calls
    use different parity buffers, so no word is overwritten before it is read."""
    ex = Exchange(WORLD, 1, WORDS, wait_limit_s=2.0)
    rnd = [random.Random(r) for r in range(WORLD)]

    def rank_fn(r):
        got = []
        for call in range(12):
            got.append(ex.call(r, 0, payload(r, call, 0),
                               delay_push_s=rnd[r].random() * 0.004))
        return got

    outs = run_ranks(ex, rank_fn, WORLD)
    want = [expected(c, 0) for c in range(12)]
    assert all(o == want for o in outs)
    assert ex.errors == [0] * WORLD


@pytest.mark.parametrize("fault", ["skip", "stale", "future"])
def test_a_faulty_rank_is_detected_by_every_receiver_without_hanging(fault):
    ex = Exchange(WORLD, TILES, WORDS, wait_limit_s=0.2)
    bad_rank, bad_call = 2, 3

    def rank_fn(r):
        for call in range(5):
            ex.call(r, 1, payload(r, call, 1),
                    fault=fault if (r == bad_rank and call == bad_call) else None)
        return True

    t0 = time.monotonic()
    run_ranks(ex, rank_fn, WORLD)
    elapsed = time.monotonic() - t0
    # every receiver of the bad rank's words gave up with the timeout code ...
    assert all(ex.errors[r] == TIMEOUT_CODE for r in range(WORLD) if r != bad_rank)
    # ... within a bounded time (each rank gives up at most once per call)
    assert elapsed < 5 * ex.wait_limit_s * WORLD + 5


def test_a_fresh_exchange_works_after_a_fault():
    """Recovery is host-side: destroy the communicator and create a new one
    (fresh inboxes and counters); calls then reduce exactly again."""
    ex = Exchange(WORLD, 1, WORDS, wait_limit_s=0.1)
    run_ranks(ex, lambda r: ex.call(r, 0, payload(r, 0, 0),
                                    fault="skip" if r == 1 else None), WORLD)
    assert any(ex.errors)
    fresh = Exchange(WORLD, 1, WORDS)
    outs = run_ranks(fresh, lambda r: [fresh.call(r, 0, payload(r, c, 0)) for c in range(3)],
                     WORLD)
    assert all(o == [expected(c, 0) for c in range(3)] for o in outs)
    assert fresh.errors == [0] * WORLD
