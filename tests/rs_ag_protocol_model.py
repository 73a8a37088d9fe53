"""Host model of the prefill two-shot all-reduce (csrc/comm_prefill.cu and the
kEpiPushStripe epilogue of csrc/gemm.cu), for protocol tests on CPU.

Per rank, one exchange buffer:
  recv [2 parities][world sources][stripe rows][cols]  partials pushed to this owner
  red  [2 parities][stripe rows][cols]                 this owner's reduced rows
  pflag[2 parities][world sources][tiles]              call number of the last push
  rflag[2 parities][tiles]                             call number of the last reduction
One call f on every rank (parity f & 1, stripe = rows per owner):
  1. the projection's epilogue: tiles in any order; each tile's partial rows go
     into its owner's recv[parity][own rank], then pflag[parity][own rank][tile]
     = f in the owner's buffer (data first, flag last);
  2. after the rank's own projection has finished (stream order): for each of
     its own tiles, wait (bounded) until every source's flag reads f, sum the
     sources in rank order, add the residual, write the output rows and red,
     then rflag = f; for every other tile, wait (bounded) until the owner's
     rflag reads f and copy the owner's red rows.
A wait that runs out records 0x701 (partials) or 0x702 (reduced rows) and
skips its tile, as the kernel does.  Values are integers, so sums are exact.
"""
from __future__ import annotations

import random
import threading
import time

PUSH_TIMEOUT, GATHER_TIMEOUT = 0x701, 0x702


class TwoShot:
    def __init__(self, world: int, rows: int, cols: int, tile_rows: int = 2,
                 wait_limit_s: float = 0.3, parity: bool = True):
        self.world, self.rows, self.cols, self.tile_rows = world, rows, cols, tile_rows
        self.parity = parity
        per_rank = -(-rows // world)
        self.stripe = -(-per_rank // tile_rows) * tile_rows
        self.m_tiles = -(-rows // tile_rows)
        self.wait_limit_s = wait_limit_s
        self.recv = [[[[[0] * cols for _ in range(self.stripe)] for _ in range(world)]
                      for _ in range(2)] for _ in range(world)]
        self.red = [[[[0] * cols for _ in range(self.stripe)] for _ in range(2)]
                    for _ in range(world)]
        self.pflag = [[[[0] * self.m_tiles for _ in range(world)] for _ in range(2)]
                      for _ in range(world)]
        self.rflag = [[[0] * self.m_tiles for _ in range(2)] for _ in range(world)]
        self.calls = [0] * world
        self.errors = [0] * world
        self.lock = threading.Lock()   # stands for the atomicity of one 16-byte store

    def owner(self, mt: int) -> int:
        return (mt * self.tile_rows) // self.stripe

    def _wait(self, read, f, rank, code) -> bool:
        t0 = time.monotonic()
        while read() != f:
            if time.monotonic() - t0 > self.wait_limit_s:
                if self.errors[rank] == 0:
                    self.errors[rank] = code
                return False
            time.sleep(0.0005)
        return True

    def call(self, rank: int, partial, residual, rng: random.Random, skip_push: bool = False):
        """One q3_gemm_allreduce of `rank`: partial / residual are rows x cols
        integer lists; returns the output rows."""
        self.calls[rank] += 1
        f = self.calls[rank]
        par = f & 1 if self.parity else 0
        # 1. the GEMM epilogue: tiles in any order, data before flag
        if not skip_push:
            tiles = list(range(self.m_tiles))
            rng.shuffle(tiles)
            for mt in tiles:
                o = self.owner(mt)
                for r in range(mt * self.tile_rows, min((mt + 1) * self.tile_rows, self.rows)):
                    for c in range(self.cols):
                        with self.lock:
                            self.recv[o][par][rank][r - o * self.stripe][c] = partial[r][c]
                    if rng.random() < 0.2:
                        time.sleep(0.0002)
                with self.lock:
                    self.pflag[o][par][rank][mt] = f
        # 2. reduce own tiles, then gather the others
        out = [[None] * self.cols for _ in range(self.rows)]
        mine = [mt for mt in range(self.m_tiles) if self.owner(mt) == rank]
        others = [mt for mt in range(self.m_tiles) if self.owner(mt) != rank]
        for mt in mine:
            ok = all(self._wait(lambda s=s: self.pflag[rank][par][s][mt], f, rank, PUSH_TIMEOUT)
                     for s in range(self.world))
            if not ok:
                continue
            for r in range(mt * self.tile_rows, min((mt + 1) * self.tile_rows, self.rows)):
                lr = r - rank * self.stripe
                for c in range(self.cols):
                    acc = 0
                    for s in range(self.world):
                        with self.lock:
                            acc += self.recv[rank][par][s][lr][c]
                    v = residual[r][c] + acc
                    out[r][c] = v
                    with self.lock:
                        self.red[rank][par][lr][c] = v
                if rng.random() < 0.2:
                    time.sleep(0.0002)
            with self.lock:
                self.rflag[rank][par][mt] = f
        for mt in others:
            o = self.owner(mt)
            if not self._wait(lambda: self.rflag[o][par][mt], f, rank, GATHER_TIMEOUT):
                continue
            for r in range(mt * self.tile_rows, min((mt + 1) * self.tile_rows, self.rows)):
                for c in range(self.cols):
                    with self.lock:
                        out[r][c] = self.red[o][par][r - o * self.stripe][c]
                if rng.random() < 0.2:
                    time.sleep(0.0002)
        return out
