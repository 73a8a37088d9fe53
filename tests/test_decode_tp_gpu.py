"""The tensor-parallel decode step kernel (q3_decode_tp) on one GPU, on a
single-rank communicator (its all-reduce is the identity):

- through the drop-in decoder (Q3VL_TP_KERNEL=1, decode graph): the tiny
  decoders' greedy tokens equal the reference's golden tokens, with
  contiguous and with paged caches;
- at one TP8 rank's shard shapes of the 8B model (hidden 4096, 4 query heads,
  1 KV head, inter 1536): two consecutive decode steps through the kernel
  match the per-kernel path layer by layer's output (max-abs <= 3e-2 of the
  output scale, cosine >= 0.9999), and the K/V rows it writes match;
- the paged plan (q3_decode_tp_create_paged) reproduces the contiguous plan's
  output and K/V rows bit for bit.
The two-GPU run of the same kernel is in tests/test_tp_gpu.py."""
import pytest
import torch

import loader_fused
from q3vl import ops
from q3vl.comm import SoloComm
from tests.golden import cases
from tests.helpers import compare, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _spec(s):
    return loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                 inter=s.inter, vocab=s.vocab, layers=s.layers,
                                 rope_theta=s.rope_theta, eps=s.eps)


@pytest.mark.parametrize("name", ["decoder_tiny_tp1", "decoder_tiny8_tp1"])
def test_tiny_decoder_greedy_tokens_through_the_step_kernel(name, monkeypatch):
    monkeypatch.setenv("Q3VL_TP_KERNEL", "1")
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    w = cases.decoder_weights(name)
    dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"], w["lm_head"],
                                     _spec(c["spec"]), 0, 1, DEV, c["max_seq"])
    assert dec.use_tp_kernel
    ids = cases.decoder_prompt(name).to(DEV)
    toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
    assert any(p is not None for p in dec._tp_plans.values()), "the step kernel did not run"
    assert toks == g["tokens"].tolist()
    assert ops.device_error(clear=True) == 0
    dec.close()


@pytest.mark.parametrize("name", ["decoder_tiny_tp1", "decoder_tiny8_tp1"])
def test_tiny_decoder_greedy_tokens_through_the_paged_step_kernel(name, monkeypatch):
    """The same tokens with the KV cache in a page pool (slot 2, pages not
    starting at page 0): the drop-in decoder builds the paged step plan."""
    from q3vl.kv_pages import KVPagePool
    monkeypatch.setenv("Q3VL_TP_KERNEL", "1")
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    s = c["spec"]
    w = cases.decoder_weights(name)
    dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"], w["lm_head"],
                                     _spec(s), 0, 1, DEV, c["max_seq"])
    pool = KVPagePool(24, 64, max_seqs=4, buckets=(256,), layers=s.layers, kv_heads=s.kv_heads,
                      device=DEV)
    pool.reserve(0, 10)
    ids = cases.decoder_prompt(name).to(DEV)
    toks = dec.generate_tokens(ids, c["new_tokens"], eos_token_id=-1, kv_pages=pool, slots=[2])
    assert any(p is not None for p in dec._tp_plans.values()), "the paged step kernel did not run"
    assert toks[0].tolist() == g["tokens"].tolist()
    assert ops.device_error(clear=True) == 0
    pool.close()
    dec.close()


def _plan(dec, kv, B, comm):
    layers = []
    for Ly, (kc, vc) in zip(dec.layers, kv):
        ab, mlp = Ly.attn_block, Ly.mlp_block
        layers.append(dict(w_qkv=ab.qkv_weight_km, w_o=Ly.o_proj.weight_km,
                           w_gate_up=mlp.gate_up_weight_il, w_down=mlp.down_weight_km,
                           input_norm=ab.input_norm_weight, post_norm=mlp.post_norm_weight,
                           q_norm=ab.q_norm_weight, k_norm=ab.k_norm_weight, k_cache=kc,
                           v_cache=vc))
    cos, sin, _ = dec.rotary.tables(DEV)
    H = dec.layers[0].attn_block.input_norm_weight.numel()
    return ops.DecodeTPPlan(layers, batch=B, hidden=H, q_heads=dec.num_q_heads,
                            kv_heads=dec.num_kv_heads,
                            inter=dec.layers[0].mlp_block.down_weight_km.shape[1],
                            max_seq=kv[0][0].shape[2], eps=dec._eps, cos=cos, sin=sin, comm=comm)


@pytest.mark.parametrize("B,P", [(8, 200), (3, 1000)])
def test_tp8_shard_step_matches_the_per_kernel_layers(B, P):
    spec = loader_fused.TextSpec(hidden=4096, q_heads=4, kv_heads=1, inter=1536, vocab=2048,
                                 layers=2)
    dec = loader_fused.random_decoder(spec, 0, 1, DEV, seed=3, max_seq=2048)
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, spec.vocab, (B, P), generator=g).to(DEV)
    kv = dec.init_kv_cache(B)
    dec.prefill(ids, kv)
    kv2 = [(k.clone(), v.clone()) for k, v in kv]
    comm = SoloComm(max_cols=spec.hidden, device=DEV)
    plan = _plan(dec, kv2, B, comm)
    tok = torch.randint(0, spec.vocab, (B, 2), generator=g).to(DEV)
    for step in range(2):
        pos = P + step
        x0 = dec._embed(tok[:, step:step + 1]).view(B, -1)
        want = x0.view(B, 1, -1)
        for i in range(spec.layers):
            want = dec.forward_layer(want, i, kv, pos, 1)
        got = x0.clone()
        kv_len = torch.tensor([pos + 1], dtype=torch.int32, device=DEV)
        plan.run(got, kv_len)
        torch.cuda.synchronize()
        assert ops.device_error(clear=True) == 0
        compare(f"step {step} hidden", got.float().cpu(), want.view(B, -1).float().cpu(),
                max_abs=3e-2, rel_scale=True, min_cos=0.9999)
        for i in range(spec.layers):
            # k rows are normed (values up to about 4, where a bf16 step is 1/32):
            # the two paths round the projection's sum in a different order
            compare(f"step {step} layer {i} k row", kv2[i][0][:, :, pos].float().cpu(),
                    kv[i][0][:, :, pos].float().cpu(), max_abs=5e-2, min_cos=0.9999)
            compare(f"step {step} layer {i} v row", kv2[i][1][:, :, pos].float().cpu(),
                    kv[i][1][:, :, pos].float().cpu(), max_abs=5e-2, min_cos=0.9999)
    plan.close()
    comm.close()


@pytest.mark.parametrize("B,P,page", [(8, 300, 128), (2, 1000, 64)])
def test_paged_step_matches_the_contiguous_step(B, P, page):
    """q3_decode_tp_create_paged: the same step with the caches in a page pool
    (slots interleaved, so pages are not in position order) gives the
    contiguous plan's output and writes the same K/V rows, bit for bit."""
    from q3vl.kv_pages import KVPagePool
    spec = loader_fused.TextSpec(hidden=4096, q_heads=4, kv_heads=1, inter=1536, vocab=2048,
                                 layers=2)
    dec = loader_fused.random_decoder(spec, 0, 1, DEV, seed=5, max_seq=2048)
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, spec.vocab, (B, P), generator=g).to(DEV)
    kv = dec.init_kv_cache(B)
    dec.prefill(ids, kv)
    pool = KVPagePool((B + 1) * 2048 // page + 8, page, max_seqs=B + 1, buckets=(2048,),
                      layers=spec.layers, kv_heads=spec.kv_heads, device=DEV)
    pool.reserve(B, 3 * page)                       # another slot's pages first
    for b in reversed(range(B)):
        pool.reserve(b, 2048)
    table = pool.device_table(range(B))
    for i, (k, v) in enumerate(kv):                  # copy the prefilled rows into pages
        ops.kv_pages_write(k[:, :, :P].contiguous(), v[:, :, :P].contiguous(), pool.k[i],
                           pool.v[i], table, start_pos=0)
    comm = SoloComm(max_cols=spec.hidden, device=DEV)
    flat = _plan(dec, kv, B, comm)
    layers = []
    for i, Ly in enumerate(dec.layers):
        ab, mlp = Ly.attn_block, Ly.mlp_block
        layers.append(dict(w_qkv=ab.qkv_weight_km, w_o=Ly.o_proj.weight_km,
                           w_gate_up=mlp.gate_up_weight_il, w_down=mlp.down_weight_km,
                           input_norm=ab.input_norm_weight, post_norm=mlp.post_norm_weight,
                           q_norm=ab.q_norm_weight, k_norm=ab.k_norm_weight,
                           k_cache=pool.k[i], v_cache=pool.v[i]))
    cos, sin, _ = dec.rotary.tables(DEV)
    paged = ops.DecodeTPPlan(layers, batch=B, hidden=spec.hidden, q_heads=spec.q_heads,
                             kv_heads=spec.kv_heads, inter=spec.inter, max_seq=2048,
                             eps=dec._eps, cos=cos, sin=sin, comm=comm, block_table=table)
    tok = torch.randint(0, spec.vocab, (B, 2), generator=g).to(DEV)
    tab = table.cpu()
    for step in range(2):
        pos = P + step
        x0 = dec._embed(tok[:, step:step + 1]).view(B, -1)
        kv_len = torch.tensor([pos + 1], dtype=torch.int32, device=DEV)
        xa, xb = x0.clone(), x0.clone()
        flat.run(xa, kv_len)
        paged.run(xb, kv_len)
        torch.cuda.synchronize()
        assert ops.device_error(clear=True) == 0
        assert torch.equal(xa, xb), f"step {step}: paged output differs"
        for i, (k, v) in enumerate(kv):
            for b in range(B):
                pg = int(tab[b, pos // page])
                assert torch.equal(pool.k[i][pg, :, pos % page], k[b, :, pos]), (step, i, b)
                assert torch.equal(pool.v[i][pg, :, pos % page], v[b, :, pos]), (step, i, b)
    flat.close()
    paged.close()
    pool.close()
    dec.close()
