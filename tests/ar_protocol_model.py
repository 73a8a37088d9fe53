"""Host model of the in-kernel all-reduce exchange (csrc/gemv.cu allreduce_tile,
csrc/comm.h layout), for protocol and failure tests on CPU.

Per rank: inbox[parity][source rank][tile][word] of (payload, call number)
8-byte words and counters[tile] (the last call completed on that tile).  One
call on a tile, on every rank:
  1. f = counters[tile] + 1, parity = f & 1;
  2. push (payload word, f) into every peer's inbox[parity][own rank][tile];
  3. for each source rank in rank order, poll the own inbox word until its
     call number equals f, giving up after a time limit (the kernel records
     error 0x501 and carries on with whatever the word holds);
  4. sum the payloads in rank order; counters[tile] = f.
Ranks run as threads; `faults` drops or corrupts a rank's pushes to show what
the receivers see.  Payloads are integers here, so sums are exact.
"""
from __future__ import annotations

import threading
import time

TIMEOUT_CODE = 0x501


class Exchange:
    def __init__(self, world: int, tiles: int, words: int, wait_limit_s: float = 0.2):
        self.world, self.tiles, self.words = world, tiles, words
        self.wait_limit_s = wait_limit_s
        # inbox[rank][parity][src][tile][word] = (payload, call number)
        self.inbox = [[[[[(0, 0)] * words for _ in range(tiles)] for _ in range(world)]
                       for _ in range(2)] for _ in range(world)]
        self.counters = [[0] * tiles for _ in range(world)]
        self.errors = [0] * world
        self.lock = threading.Lock()   # word stores are atomic 8-byte stores on the device

    def call(self, rank: int, tile: int, payload: list, fault: str = None,
             delay_push_s: float = 0.0) -> list:
        """One all-reduce call of `rank` on `tile`; returns the summed words.
        fault: None, "skip" (push nothing), "stale" (push call number f - 2,
        which has this call's parity), "future" (push f + 2)."""
        f = self.counters[rank][tile] + 1
        par = f & 1
        if delay_push_s:
            time.sleep(delay_push_s)
        if fault != "skip":
            tag = {None: f, "stale": f - 2, "future": f + 2}[fault]
            for r in range(self.world):
                if r == rank:
                    continue
                for w in range(self.words):
                    with self.lock:
                        self.inbox[r][par][rank][tile][w] = (payload[w], tag)
        total = [0] * self.words
        gave_up = False
        for src in range(self.world):
            for w in range(self.words):
                if src == rank:
                    d = payload[w]
                else:
                    with self.lock:
                        v = self.inbox[rank][par][src][tile][w]
                    if v[1] != f and not gave_up:
                        t0 = time.monotonic()
                        while True:
                            with self.lock:
                                v = self.inbox[rank][par][src][tile][w]
                            if v[1] == f:
                                break
                            if time.monotonic() - t0 > self.wait_limit_s:
                                self.errors[rank] = self.errors[rank] or TIMEOUT_CODE
                                gave_up = True
                                break
                            time.sleep(0)
                    d = v[0]
                total[w] += d
        self.counters[rank][tile] = f
        return total


def run_ranks(ex: Exchange, fn, world: int):
    """Run fn(rank) on `world` threads; returns their results in rank order."""
    out = [None] * world
    errs = []

    def body(r):
        try:
            out[r] = fn(r)
        except Exception as e:   # surfaced to the test
            errs.append(e)

    ts = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=30)
        assert not t.is_alive(), "a rank did not return"
    if errs:
        raise errs[0]
    return out
