"""Paged KV on the GPU: the page write and decode attention through a block
table reproduce the contiguous cache path bit for bit (same kernel arithmetic,
only the row addresses differ)."""
import pytest
import torch

from q3vl import ops
from q3vl.kv_pages import KVPagePool

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF16 = torch.bfloat16


def rnd(*shape, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(BF16)


@pytest.mark.parametrize("B,Hq,Hkv,lens,page", [(3, 32, 8, (700, 64, 1500), 256),
                                                 (2, 8, 2, (1, 333), 64),
                                                 (4, 16, 16, (2048, 2048, 100, 1024), 128)])
def test_paged_decode_matches_contiguous(B, Hq, Hkv, lens, page):
    pool = KVPagePool(64 if page >= 128 else 96, page, max_seqs=B, buckets=(2048,), layers=1,
                      kv_heads=Hkv, device=DEV)
    pool.reserve(B - 1, 10)                                  # interleave the slots' pages
    for b in range(B):
        pool.reserve(b, lens[b])
    L = max(lens)
    table = pool.device_table(range(B))
    k = rnd(B, Hkv, L, 128, seed=1).to(DEV)
    v = rnd(B, Hkv, L, 128, seed=2).to(DEV)
    # write every position through the page-write kernel, then decode each row
    ops.kv_pages_write(k, v, pool.k[0], pool.v[0], table, start_pos=0)
    assert ops.device_error(clear=True) == 0
    q = rnd(B, Hq, 128, seed=3).to(DEV)
    for b in range(B):
        n = lens[b]
        want = ops.attn_decode(q[b:b + 1].contiguous(), k[b:b + 1].contiguous(),
                               v[b:b + 1].contiguous(), kv_len=n)
        got = ops.attn_decode_paged(q[b:b + 1].contiguous(), pool.k[0], pool.v[0],
                                    table[b:b + 1].contiguous(), kv_len=n)
        assert torch.equal(got, want), f"row {b} (len {n})"
    assert ops.device_error(clear=True) == 0
    pool.close()


def test_page_write_at_a_device_position_and_bad_table_entries():
    pool = KVPagePool(8, 64, max_seqs=2, buckets=(), layers=1, kv_heads=2, device=DEV)
    pool.reserve(0, 128)
    table = pool.device_table([0, 1])                     # slot 1 holds no pages (-1)
    k = rnd(2, 2, 1, 128, seed=4).to(DEV)
    v = rnd(2, 2, 1, 128, seed=5).to(DEV)
    pos = torch.tensor([70], dtype=torch.int32, device=DEV)
    ops.kv_pages_write(k, v, pool.k[0], pool.v[0], table, pos_dev=pos)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0x403          # row 1 skipped, recorded
    pg = int(table[0, 70 // 64])
    assert torch.equal(pool.k[0][pg, :, 70 % 64].cpu(), k[0, :, 0].cpu())
    assert torch.equal(pool.v[0][pg, :, 70 % 64].cpu(), v[0, :, 0].cpu())
    pool.close()


def test_norm_rope_writes_the_same_rows_into_pages():
    """q3_qkv_norm_rope_paged: q and the K/V rows it writes through the table
    equal q3_qkv_norm_rope's q and contiguous cache rows, bit for bit."""
    B, S, Hq, Hkv, start = 2, 5, 8, 2, 70
    qkv = rnd(B * S, (Hq + 2 * Hkv) * 128, seed=6).to(DEV)
    qn, kn = (1 + 0.1 * rnd(128, seed=7).float()).to(BF16).to(DEV), \
        (1 + 0.1 * rnd(128, seed=8).float()).to(BF16).to(DEV)
    t = torch.arange(256, dtype=torch.float32)[:, None] * 0.01
    cos, sin = t.cos().repeat(1, 64).to(BF16).to(DEV), t.sin().repeat(1, 64).to(BF16).to(DEV)
    kc = torch.zeros(B, Hkv, 256, 128, dtype=BF16, device=DEV)
    vc = torch.zeros_like(kc)
    q_ref, _, _ = ops.qkv_norm_rope(qkv, qn, kn, cos, sin, B=B, S=S, Hq=Hq, Hkv=Hkv,
                                    start_pos=start, k_cache=kc, v_cache=vc)
    pool = KVPagePool(16, 64, max_seqs=2, buckets=(256,), layers=1, kv_heads=Hkv, device=DEV)
    pool.reserve(1, 256)
    pool.reserve(0, 256)
    table = pool.device_table([0, 1])
    q = ops.qkv_norm_rope_paged(qkv, qn, kn, cos, sin, B=B, S=S, Hq=Hq, Hkv=Hkv,
                                k_pages=pool.k[0], v_pages=pool.v[0], block_table=table,
                                start_pos=start)
    assert torch.equal(q, q_ref)
    tab = table.cpu()
    for b in range(B):
        for pos in range(start, start + S):
            pg = int(tab[b, pos // 64])
            assert torch.equal(pool.k[0][pg, :, pos % 64], kc[b, :, pos])
            assert torch.equal(pool.v[0][pg, :, pos % 64], vc[b, :, pos])
    assert ops.device_error(clear=True) == 0
    pool.close()


@pytest.mark.parametrize("name", ["decoder_tiny_tp1", "decoder_tiny8_tp1"])
@pytest.mark.parametrize("graphs", [True, False])
def test_tiny_decoder_generates_the_reference_tokens_through_pages(graphs, name):
    """generate_tokens with the KV cache in a page pool (slot 2, whose pages do
    not start at page 0) reproduces the reference decoder's 32 greedy tokens."""
    import loader_fused
    from tests.golden import cases
    from tests.helpers import load_golden
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    s = c["spec"]
    spec = loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                 inter=s.inter, vocab=s.vocab, layers=s.layers,
                                 rope_theta=s.rope_theta, eps=s.eps)
    w = cases.decoder_weights(name)
    dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"], w["lm_head"],
                                     spec, 0, 1, DEV, c["max_seq"])
    dec.use_graphs = graphs
    pool = KVPagePool(24, 64, max_seqs=4, buckets=(256,), layers=s.layers, kv_heads=s.kv_heads,
                      device=DEV)
    pool.reserve(0, 10)
    ids = cases.decoder_prompt(name).to(DEV)
    toks = dec.generate_tokens(ids, c["new_tokens"], eos_token_id=-1, kv_pages=pool, slots=[2])
    assert toks[0].tolist() == g["tokens"].tolist()
    assert ops.device_error(clear=True) == 0
    pool.close()


@pytest.mark.parametrize("split", [8, 24])
def test_chunked_prefill_through_pages_matches_one_shot(split):
    """Prefill in two calls on a page pool (the second reads the first call's
    K/V through the block table) gives the one-shot prefill's last logits."""
    import loader_fused
    from tests.golden import cases
    from tests.helpers import compare
    name = "decoder_tiny_tp1"
    c = cases.DECODER_CASES[name]
    s = c["spec"]
    spec = loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                 inter=s.inter, vocab=s.vocab, layers=s.layers,
                                 rope_theta=s.rope_theta, eps=s.eps)
    w = cases.decoder_weights(name)
    dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"], w["lm_head"],
                                     spec, 0, 1, DEV, c["max_seq"])
    pool = KVPagePool(24, 64, max_seqs=2, buckets=(256,), layers=s.layers, kv_heads=s.kv_heads,
                      device=DEV)
    pool.reserve(0, 10)
    pool.reserve(1, 256)
    kv = pool.layers(pool.device_table([1]))
    ids = cases.decoder_prompt(name).to(DEV)
    dec.forward(ids[:, :split], 0, kv)
    got = dec.forward(ids[:, split:].contiguous(), split, kv)
    want = dec.forward(ids, 0, dec.init_kv_cache(1))
    compare("chunked paged prefill", got.float().cpu(), want.float().cpu(), max_abs=5e-2,
            rel_scale=True, min_cos=0.999)
    assert ops.device_error(clear=True) == 0
    pool.close()


@pytest.mark.parametrize("B,Hq,Hkv,S,start,page", [(2, 32, 8, 700, 0, 256),
                                                  (3, 8, 2, 300, 90, 128)])
def test_tc_prefill_through_pages_matches_contiguous(B, Hq, Hkv, S, start, page):
    """q3_attn_prefill_tc_paged (variant 2 through a block table) gives the
    contiguous variant 2's bits: the same arithmetic, and the page rows past
    the last key hold finite values that get probability 0."""
    L = start + S
    pool = KVPagePool(64, page, max_seqs=B, buckets=(2048,), layers=1, kv_heads=Hkv, device=DEV)
    pool.reserve(B - 1, 10)                                  # interleave the slots' pages
    for b in range(B):
        pool.reserve(b, L)
    table = pool.device_table(range(B))
    k = rnd(B, Hkv, L, 128, seed=6).to(DEV)
    v = rnd(B, Hkv, L, 128, seed=7).to(DEV)
    ops.kv_pages_write(k, v, pool.k[0], pool.v[0], table, start_pos=0)
    q = rnd(B, Hq, S, 128, seed=8).to(DEV)
    want = ops.attn_prefill_tc(q, k, v, start_pos=start, variant=2)
    got = ops.attn_prefill_tc_paged(q, pool.k[0], pool.v[0], table, start_pos=start)
    assert torch.equal(got, want)
    assert ops.device_error(clear=True) == 0
    pool.close()
