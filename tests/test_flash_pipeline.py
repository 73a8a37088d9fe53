"""The tcgen05 prefill attention kernel's pipeline protocol, replayed on the
host (tests/flash_pipeline_model.py) under seeded random interleavings: every
tile reaches every role in order with no race on a shared-memory or TMEM
buffer and no lapped barrier, and a wait that runs out ends the kernel with
its error code and nothing in flight.  CPU only."""
import pytest

from tests.flash_pipeline_model import Model, ModelMN


@pytest.mark.parametrize("n_kb", [1, 2, 3, 4, 5, 8, 13])
def test_every_interleaving_delivers_each_tile_once_without_races(n_kb):
    for seed in range(150):
        m = Model(n_kb, seed)
        assert m.run() == "done", (n_kb, seed)
        assert m.errors == [], (n_kb, seed, m.errors[:3])
        assert m.err == 0 and not m.abort
        assert all(m.seen[w] == list(range(n_kb)) for w in range(4))


@pytest.mark.parametrize("n_kb", [2, 3, 6])
def test_a_wait_that_runs_out_ends_every_role_with_nothing_in_flight(n_kb):
    codes = set()
    for seed in range(300):
        m = Model(n_kb, seed, fault_at=1 + seed % 40)
        assert m.run() == "done", (n_kb, seed)
        assert m.errors == [], (n_kb, seed, m.errors[:3])
        if m.err:
            codes.add(m.err)
            assert 0x601 <= m.err <= 0x60b
    assert len(codes) >= 4, sorted(hex(c) for c in codes)   # faults land in several roles


def test_the_named_barrier_handoff_could_hang_after_a_timeout():
    """The earlier hand-off (bar.sync across both transposer warps) hangs
    when one warp leaves its loop on a timeout and the other reaches the
    barrier; the per-warp release above never does."""
    hung = 0
    for seed in range(400):
        m = Model(4, seed, fault_at=1 + seed % 40, named_barrier=True)
        hung += m.run() == "deadlock"
    assert hung > 0
    for seed in range(150):                          # without a fault it is fine too
        m = Model(4, seed, named_barrier=True)
        assert m.run() == "done" and m.errors == []


@pytest.mark.parametrize("n_kb", [1, 2, 3, 4, 5, 8, 13])
@pytest.mark.parametrize("rescale_p", [0.0, 0.3, 1.0])
def test_mn_variant_delivers_each_tile_without_races(n_kb, rescale_p):
    """Variant 1 (V in place, O accumulated in TMEM, lazy rescale): every O MMA
    reads the previous tile's O, softmax rescales touch O only between two O
    MMAs, P buffers are rewritten only after the O MMA that read them."""
    rescaled = 0
    for seed in range(150):
        m = ModelMN(n_kb, seed, rescale_p=rescale_p)
        assert m.run() == "done", (n_kb, seed)
        assert m.errors == [], (n_kb, seed, m.errors[:3])
        assert m.err == 0 and not m.abort
        assert all(m.seen[w] == list(range(n_kb)) for w in range(4))
        rescaled += m.rescales
    assert rescaled > 0 or rescale_p == 0.0 or n_kb == 1


@pytest.mark.parametrize("n_kb", [2, 3, 6])
def test_mn_variant_ends_cleanly_after_a_timeout(n_kb):
    codes = set()
    for seed in range(300):
        m = ModelMN(n_kb, seed, fault_at=1 + seed % 40)
        assert m.run() == "done", (n_kb, seed)
        assert m.errors == [], (n_kb, seed, m.errors[:3])
        if m.err:
            codes.add(m.err)
            assert 0x611 <= m.err <= 0x618
    assert len(codes) >= 3, sorted(hex(c) for c in codes)


@pytest.mark.parametrize("n_kb", [1, 2, 3, 4, 5, 8, 13])
@pytest.mark.parametrize("rescale_p", [0.0, 0.3, 1.0])
def test_two_tile_variant_delivers_each_tile_without_races(n_kb, rescale_p):
    """Variant 2 (two query tiles, separate K and V rings, P written over S in
    TMEM): every PV reads the P of its own tile and step, every S MMA writes
    only after the PV that read the P it overwrites, O rescales fall between
    two PVs of the tile, and K/V stages are refilled only after both tiles
    are done with them."""
    from tests.flash_pipeline_model import ModelPP
    rescaled = 0
    for seed in range(150):
        m = ModelPP(n_kb, seed, rescale_p=rescale_p)
        assert m.run() == "done", (n_kb, seed)
        assert m.errors == [], (n_kb, seed, m.errors[:3])
        assert m.err == 0 and not m.abort
        assert all(m.seen[(t, w)] == [0] for t in range(2) for w in range(4))
        rescaled += m.rescales
    assert rescaled > 0 or rescale_p == 0.0 or n_kb == 1


@pytest.mark.parametrize("items", [[3, 1], [1, 1, 1], [5, 2, 4, 1], [2, 6, 2, 6, 3]])
def test_two_tile_variant_runs_items_back_to_back_without_races(items):
    """The persistent form: Q is replaced only after the item's last S MMAs,
    O[t] only after the previous item's O[t] was read out, and the K/V rings
    and every barrier phase run on across items."""
    from tests.flash_pipeline_model import ModelPP
    for seed in range(150):
        m = ModelPP(0, seed, rescale_p=0.3, items=items)
        assert m.run() == "done", (items, seed)
        assert m.errors == [], (items, seed, m.errors[:3])
        assert m.err == 0 and not m.abort
        assert all(m.seen[(t, w)] == list(range(len(items)))
                   for t in range(2) for w in range(4))


@pytest.mark.parametrize("n_kb", [2, 3, 6])
def test_two_tile_variant_ends_cleanly_after_a_timeout(n_kb):
    from tests.flash_pipeline_model import ModelPP
    codes = set()
    for seed in range(300):
        m = ModelPP(n_kb, seed, fault_at=1 + seed % 40, items=[n_kb, 2, n_kb])
        assert m.run() == "done", (n_kb, seed)
        assert m.errors == [], (n_kb, seed, m.errors[:3])
        if m.err:
            codes.add(m.err)
            assert 0x631 <= m.err <= 0x63c
    assert len(codes) >= 3, sorted(hex(c) for c in codes)
