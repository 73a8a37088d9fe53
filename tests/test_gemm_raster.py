"""The tcgen05 GEMM's tile rasters (csrc/gemm.cu tile_coords), restated on the
host: the column order and every grouped order visit each output tile exactly
once, so the raster only changes which tiles share L2 at a time."""
import pytest


def tile_coords(tile, m_tiles, n_tiles, group_m):
    if group_m <= 0:
        return tile % m_tiles, tile // m_tiles
    per_group = group_m * n_tiles
    first_m = (tile // per_group) * group_m
    gm = min(m_tiles - first_m, group_m)
    inner = tile % per_group
    return first_m + inner % gm, inner // gm


@pytest.mark.parametrize("m_tiles,n_tiles", [(64, 24), (1, 1), (7, 3), (65, 17), (3, 40)])
@pytest.mark.parametrize("group_m", [0, 1, 4, 8, 16, 100])
def test_every_tile_once(m_tiles, n_tiles, group_m):
    seen = {tile_coords(t, m_tiles, n_tiles, group_m) for t in range(m_tiles * n_tiles)}
    assert seen == {(m, n) for m in range(m_tiles) for n in range(n_tiles)}


def test_grouped_wave_touches_fewer_rows_and_columns():
    """One wave of 148 CTAs on the 8192 x 6144 prefill QKV GEMM (64 x 24 tiles)."""
    def footprint(g):
        tiles = [tile_coords(t, 64, 24, g) for t in range(148)]
        return len({m for m, _ in tiles}), len({n for _, n in tiles})
    assert footprint(0) == (64, 3)
    m, n = footprint(16)
    assert m == 16 and n == 10
