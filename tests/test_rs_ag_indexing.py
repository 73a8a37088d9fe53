"""Index arithmetic of the prefill two-shot all-reduce, restated on the host
from csrc/comm_prefill.cu (q3_prefill_comm_create sizing, rs_ag_kernel's item
mapping) and csrc/gemm.cu (kEpiPushStripe's destination rows and flags):
every output tile is handled exactly once per rank, each rank reduces exactly
the tiles of its own stripe first, and every push, flag and reduced-stripe
offset stays inside the region the communicator allocated.  CPU only."""
import itertools

import pytest

TILE_M, TILE_N = 128, 256


def ceil_div(a, b):
    return -(-a // b)


def comm_sizes(world, max_rows, max_cols):
    stripe_max = ceil_div(ceil_div(max_rows, world), TILE_M) * TILE_M
    max_tiles = ceil_div(max_rows, TILE_M) * ceil_div(max_cols, TILE_N)
    return stripe_max, max_tiles


def items(M, N, world, rank):
    """rs_ag_kernel: item -> (mt, nt, mine), in item order."""
    stripe = ceil_div(ceil_div(M, world), TILE_M) * TILE_M
    m_tiles = ceil_div(M, TILE_M)
    n_tiles = ceil_div(N, TILE_N)
    own_r0 = rank * stripe
    own_r1 = min(own_r0 + stripe, M)
    own_m0 = min(own_r0 // TILE_M, m_tiles)
    own_m1 = ceil_div(own_r1, TILE_M) if own_r1 > own_r0 else own_m0
    n_own = (own_m1 - own_m0) * n_tiles
    out = []
    for item in range(m_tiles * n_tiles):
        if item < n_own:
            mt, nt, mine = own_m0 + item // n_tiles, item % n_tiles, True
        else:
            j = item - n_own
            mt = j // n_tiles
            if mt >= own_m0:
                mt += own_m1 - own_m0
            nt, mine = j % n_tiles, False
        out.append((mt, nt, mine))
    return out, stripe, n_tiles


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_every_tile_once_and_own_tiles_first(world):
    for M, N in itertools.product([17, 40, 127, 128, 129, 300, 1000, 4096, 8192],
                                  [32, 256, 512, 1088, 4096]):
        for rank in range(world):
            its, stripe, n_tiles = items(M, N, world, rank)
            tiles = [(mt, nt) for mt, nt, _ in its]
            m_tiles = ceil_div(M, TILE_M)
            assert sorted(tiles) == [(m, n) for m in range(m_tiles) for n in range(n_tiles)]
            seen_other = False
            for mt, nt, mine in its:
                owner = (mt * TILE_M) // stripe
                assert owner < world
                assert mine == (owner == rank), (M, N, world, rank, mt)
                if not mine:
                    seen_other = True
                assert not (mine and seen_other), "own tiles come first"


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_offsets_stay_inside_the_communicator(world):
    max_rows, max_cols = 8192, 4096
    stripe_max, max_tiles = comm_sizes(world, max_rows, max_cols)
    for M, N in itertools.product([17, 129, 1000, 8191, 8192], [32, 544, 4096]):
        its, stripe, n_tiles = items(M, N, world, 0)
        assert stripe <= stripe_max
        for mt in range(ceil_div(M, TILE_M)):
            owner = (mt * TILE_M) // stripe
            for nt in range(n_tiles):
                # push epilogue: rows of the tile below M, whole 32-column chunks below N
                for row in (mt * TILE_M, min(mt * TILE_M + TILE_M, M) - 1):
                    lr = row - owner * stripe
                    assert 0 <= lr < stripe
                    last_col = min(nt * TILE_N + TILE_N, N) - 1
                    assert lr * N + last_col < stripe_max * max_cols
                key = mt * n_tiles + nt
                assert 4 * key + 3 < 4 * max_tiles
