"""Paged KV page allocator (q3_kv_pages_*, host C++; no GPU): bucketed growth,
all-or-nothing reservations, deterministic page order (the same on every
tensor-parallel rank), and the position -> (page, offset) layout that the
block table encodes."""
import os
import random
import socket

import pytest
import torch
import torch.multiprocessing as mp

from q3vl import _lib
from q3vl.kv_pages import KVPagePool, pages_for_bytes


class ModelPool:
    """Plain-Python statement of the allocator's contract, for the randomized test."""

    def __init__(self, num_pages, page_tokens, buckets, max_pages):
        self.free = list(range(num_pages - 1, -1, -1))
        self.own = {}
        self.pt, self.buckets, self.max_pages = page_tokens, buckets, max_pages

    def reserve(self, slot, tokens):
        own = self.own.setdefault(slot, [])
        if tokens <= len(own) * self.pt:
            return len(own) * self.pt
        cap = next((b for b in self.buckets if b >= tokens), None) if self.buckets else \
            -(-tokens // self.pt) * self.pt
        if cap is None or cap // self.pt > self.max_pages:
            raise ValueError("too large")
        grow = cap // self.pt - len(own)
        if grow > len(self.free):
            raise MemoryError
        for _ in range(grow):
            own.append(self.free.pop())
        return cap

    def release(self, slot):
        for p in reversed(self.own.pop(slot, [])):
            self.free.append(p)


def test_bucketed_growth_keeps_pages_in_place():
    pool = KVPagePool(64, 256, max_seqs=4)
    assert pool.reserve(0, 1) == 2048 and pool.slot_pages(0) == 8
    assert pool.reserve(0, 2048) == 2048 and pool.slot_pages(0) == 8     # already covered
    first = pool.table([0])[0, :8].tolist()
    assert first == list(range(8))
    assert pool.reserve(0, 2049) == 4096 and pool.slot_pages(0) == 16
    row = pool.table([0])[0]
    assert row[:8].tolist() == first                                     # prefix stays put
    assert row[16:].eq(-1).all() and pool.free_pages == 64 - 16
    pool.close()


def test_release_returns_pages_in_reusable_order():
    pool = KVPagePool(32, 128, max_seqs=3, buckets=())
    pool.reserve(0, 300)                      # 3 pages: 0, 1, 2
    pool.reserve(1, 129)                      # 2 pages: 3, 4
    before = pool.table([0])[0, :3].tolist()
    pool.release(0)
    assert pool.slot_pages(0) == 0 and pool.free_pages == 32 - 2
    pool.reserve(2, 384)
    assert pool.table([2])[0, :3].tolist() == before
    pool.close()


def test_exhaustion_is_all_or_nothing():
    pool = KVPagePool(20, 256, max_seqs=4)
    pool.reserve(0, 2048)
    with pytest.raises(_lib.Q3Error) as e:
        pool.reserve(1, 4096)                 # needs 16, 12 free
    assert e.value.status == _lib.Q3_ERR_NO_MEMORY
    assert pool.slot_pages(1) == 0 and pool.free_pages == 12
    assert pool.reserve(1, 2000) == 2048
    pool.close()


def test_invalid_requests_are_rejected():
    with pytest.raises(_lib.Q3Error, match="multiple of 64"):
        KVPagePool(8, 100, buckets=())
    with pytest.raises(_lib.Q3Error, match="ascending"):
        KVPagePool(8, 64, buckets=(256, 128))
    with pytest.raises(_lib.Q3Error, match="multiple of page_tokens"):
        KVPagePool(8, 256, buckets=(1000,))
    pool = KVPagePool(64, 256, max_seqs=2)
    with pytest.raises(_lib.Q3Error, match="largest bucket"):
        pool.reserve(0, 8193)
    with pytest.raises(_lib.Q3Error, match="slot"):
        pool.reserve(2, 10)
    pool.reserve(0, 4096)
    with pytest.raises(_lib.Q3Error, match="width"):
        pool.table([0], width=8)
    pool.close()


@pytest.mark.parametrize("seed,buckets", [(1, (512, 1024, 2048)), (2, ()), (3, (2048, 4096))])
def test_random_operations_match_the_contract(seed, buckets):
    rnd = random.Random(seed)
    pt, n_pages, seqs = 128, 96, 6
    max_pages = (max(buckets) // pt) if buckets else 40
    pool = KVPagePool(n_pages, pt, max_seqs=seqs, buckets=buckets, max_pages_per_seq=max_pages)
    model = ModelPool(n_pages, pt, buckets, max_pages)
    for _ in range(400):
        slot = rnd.randrange(seqs)
        if rnd.random() < 0.3:
            pool.release(slot)
            model.release(slot)
            continue
        tokens = rnd.randint(0, (max(buckets) if buckets else max_pages * pt) + 64)
        try:
            want = model.reserve(slot, tokens)
        except (ValueError, MemoryError) as exc:
            with pytest.raises(_lib.Q3Error) as e:
                pool.reserve(slot, tokens)
            want_status = _lib.Q3_ERR_NO_MEMORY if isinstance(exc, MemoryError) \
                else _lib.Q3_ERR_INVALID
            assert e.value.status == want_status
            continue
        assert pool.reserve(slot, tokens) == want
        table = pool.table(range(seqs))
        for s in range(seqs):
            own = model.own.get(s, [])
            assert table[s, :len(own)].tolist() == own
            assert table[s, len(own):].eq(-1).all()
        assert pool.free_pages == len(model.free)
    # no page is held twice
    held = [p for s in range(seqs) for p in model.own.get(s, [])]
    assert len(held) == len(set(held)) and len(held) + pool.free_pages == n_pages
    pool.close()


def test_block_table_layout_round_trips_a_contiguous_cache():
    """Position p of a slot lives in page table[p // page_tokens] at offset
    p % page_tokens; scattering a contiguous [Hkv, L, D] cache through the
    table and gathering it back is the identity, and each 64-position
    attention tile stays inside one page."""
    pt, Hkv, D = 128, 2, 8
    pool = KVPagePool(24, pt, max_seqs=3, buckets=(512, 1024))
    pool.reserve(1, 300)
    pool.reserve(0, 700)
    pool.reserve(2, 1)
    pages = torch.zeros(24, Hkv, pt, D)
    g = torch.Generator().manual_seed(0)
    caches = {s: torch.randn(Hkv, L, D, generator=g) for s, L in ((0, 700), (1, 300), (2, 1))}
    tab = pool.table([0, 1, 2])
    for s, c in caches.items():
        L = c.shape[1]
        pos = torch.arange(L)
        page, off = tab[s][pos // pt].long(), pos % pt
        assert (page >= 0).all()
        pages[page, :, off] = c.permute(1, 0, 2)
    for s, c in caches.items():
        L = c.shape[1]
        pos = torch.arange(L)
        back = pages[tab[s][pos // pt].long(), :, pos % pt].permute(1, 0, 2)
        assert torch.equal(back, c)
        tiles = pos // 64
        for t in tiles.unique():
            assert tab[s][(pos[tiles == t] // pt)].unique().numel() == 1
    pool.close()


def test_pages_for_bytes_sizes_the_8b_decoder():
    # 36 layers, 8 KV heads, D 128, bf16: 144 KiB per token
    n = pages_for_bytes(100 * 10**9, 36, 8, 256)
    assert n * 256 * 144 * 1024 <= 100 * 10**9 < (n + 1) * 256 * 144 * 1024


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen3-vl_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from q3vl.kv_pages import KVPagePool as Pool

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pool = Pool(64, 256, max_seqs=4)
        rnd = random.Random(7)          # the server broadcasts the same schedule to every rank
        for _ in range(100):
            slot = rnd.randrange(4)
            if rnd.random() < 0.3:
                pool.release(slot)
            else:
                try:
                    pool.reserve(slot, rnd.randint(1, 8192))
                except Exception:
                    pass
        table = pool.table(range(4))
        gathered = [torch.empty_like(table) for _ in range(world)]
        dist.all_gather(gathered, table)
        if rank == 0:
            q.put(all(torch.equal(gathered[0], t) for t in gathered))
        pool.close()
    finally:
        dist.destroy_process_group()


def test_ranks_issuing_the_same_calls_hold_the_same_tables():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    same = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert same


def test_decoder_page_tables_for_a_batch():
    """Qwen3VLDecoderFused._paged_kv: slots grow to the KV bucket, the block
    table lands in one persistent tensor per (pool, batch), and a pool that
    does not match the decoder is refused (host logic, CPU tensors)."""
    from model_fused import Qwen3VLDecoderFused
    from q3vl.kv_pages import PagedLayer
    dec = Qwen3VLDecoderFused.__new__(Qwen3VLDecoderFused)
    dec.num_layers, dec.device, dec._page_tables = 2, torch.device("cpu"), {}
    pool = KVPagePool(40, 64, max_seqs=4, buckets=(256, 512), layers=2, kv_heads=1,
                      head_dim=8, device="cpu")
    pool.reserve(3, 1)
    layers = dec._paged_kv(pool, 2, 512, slots=[1, 3])
    assert len(layers) == 2 and all(isinstance(x, PagedLayer) for x in layers)
    k, v = layers[0]
    assert k is pool.k[0] and v is pool.v[0]
    table = layers[0].table
    assert table.shape == (2, 8) and table.dtype == torch.int32
    assert pool.slot_pages(1) == 8 and pool.slot_pages(3) == 8
    assert table[1, :4].tolist() == [0, 1, 2, 3]        # slot 3 kept its first pages
    again = dec._paged_kv(pool, 2, 256, slots=[1, 3])
    assert again[0].table is table                      # one tensor per (pool, batch)
    with pytest.raises(ValueError, match="layers"):
        dec._paged_kv(KVPagePool(8, 64, max_seqs=1, buckets=(256,), layers=1, kv_heads=1,
                                 head_dim=8, device="cpu"), 1, 256)
    with pytest.raises(ValueError, match="bucket"):
        dec._paged_kv(pool, 1, 1024)
    pool.close()



def test_per_sequence_rope_delta_rows_equal_the_shared_table():
    """Qwen3VLDecoderFused._decode_rope: equal deltas collapse to one int;
    different deltas give RowRope tables whose row b * rows + t is the shared
    RotaryEmbedding row t + delta_b, bit for bit (CPU)."""
    from model_fused import Qwen3VLDecoderFused, RotaryEmbedding, RowRope
    dec = Qwen3VLDecoderFused.__new__(Qwen3VLDecoderFused)
    dec.device, dec._row_ropes = torch.device("cpu"), {}
    dec.rotary = RotaryEmbedding(128, max_seq_len=4096, base=5e6)
    assert dec._decode_rope(7, 2, 256) == 7
    assert dec._decode_rope(torch.tensor([[-3], [-3]]), 2, 256) == -3
    rr = dec._decode_rope(torch.tensor([[-30], [-24]]), 2, 256)
    assert isinstance(rr, RowRope) and rr.rows == 256
    for b, d in enumerate((-30, -24)):
        for t in (30, 100, 255):
            assert torch.equal(rr.cos[b * 256 + t], dec.rotary.cos_cached[t + d])
            assert torch.equal(rr.sin[b * 256 + t], dec.rotary.sin_cached[t + d])
    again = dec._decode_rope([-1, -2], 2, 256)
    assert again is rr and torch.equal(rr.cos[5], dec.rotary.cos_cached[4])   # same buffer
    with pytest.raises(ValueError, match="rope deltas"):
        dec._decode_rope([1, 2, 3], 2, 256)
