"""Decoder parity through the drop-in Python API (model_fused / loader_fused)
on one GPU: module outputs vs the reference fixtures, logits within
tolerance, greedy tokens identical over 32 steps."""
import pytest
import torch

import loader_fused
import model_fused
from oracle import decoder as odec
from oracle import ref as oref
from tests.golden import cases
from tests.helpers import as_tensor, compare, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _spec(s: odec.Spec) -> loader_fused.TextSpec:
    return loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                 inter=s.inter, vocab=s.vocab, layers=s.layers,
                                 rope_theta=s.rope_theta, eps=s.eps)


def _decoder(weights, spec, tp=1, rank=0, max_seq=256):
    return loader_fused.build_decoder(weights["layers"], weights["embed"], weights["final_norm"],
                                      weights["lm_head"], _spec(spec), rank, tp, DEV, max_seq)


def test_attention_block_module_vs_reference():
    g = load_golden("attn_block")
    c = cases.attn_block_case()
    blk = model_fused.AttentionBlock(c["qkv_w"].to(DEV), None, c["o_w"].to(DEV),
                                     c["in_norm"].to(DEV), c["q_norm"].to(DEV),
                                     c["k_norm"].to(DEV), c["Hq"], c["Hkv"], 128, 1e-6)
    rot = model_fused.RotaryEmbedding(128, max_seq_len=c["max_seq"], base=5e6)
    cos, sin = rot.get(c["S"], offset=c["start"], device=DEV)
    q, k, v = blk(c["hidden"].to(DEV), cos, sin)
    assert torch.allclose(blk.qkv_weight.cpu().float(), c["qkv_w"].float())
    for name, got in (("q", q), ("k", k), ("v", v)):
        compare(f"AttentionBlock {name}", got.cpu(), as_tensor(g[name]), max_abs=3.2e-2,
                min_cos=0.9999)


def test_layer8b_forward_layer_vs_reference():
    """One Qwen3-VL-8B-shape layer (TP1): prefill 8 tokens then one decode step."""
    g = load_golden("layer8b")
    c = cases.layer8b_case()
    dec = _decoder(c["weights"], c["spec"], max_seq=c["max_seq"])
    kv = dec.init_kv_cache(1)
    h1 = dec.forward_layer(c["hidden"].to(DEV), 0, kv, 0, c["S"])
    h2 = dec.forward_layer(c["hidden_dec"].to(DEV), 0, kv, c["S"], 1)
    compare("layer8b prefill", h1.cpu(), as_tensor(g["prefill"]), max_abs=5e-2, rel_scale=True,
            min_cos=0.999)
    compare("layer8b decode", h2.cpu(), as_tensor(g["decode"]), max_abs=5e-2, rel_scale=True,
            min_cos=0.999)


@pytest.mark.parametrize("name", ["decoder_tiny_tp1", "decoder_tiny8_tp1"])
@pytest.mark.parametrize("graphs", [True, False])
def test_tiny_decoder_generate_vs_reference(graphs, name):
    """Prefill logits within tolerance and 32 greedy tokens identical to the
    reference decoder's generate (decoder_tiny8_tp1's tokens change from step
    to step)."""
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    dec = _decoder(cases.decoder_weights(name), c["spec"], max_seq=c["max_seq"])
    dec.use_graphs = graphs
    ids = cases.decoder_prompt(name).to(DEV)
    logits = dec.forward(ids, 0, dec.init_kv_cache(1))
    compare("tiny logits", logits.cpu(), as_tensor(g["logits"]), max_abs=5e-2, rel_scale=True,
            min_cos=0.999)
    toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
    assert toks == g["tokens"].tolist()


def test_generate_batched_matches_per_row():
    name = "decoder_tiny_tp1"
    c = cases.DECODER_CASES[name]
    dec = _decoder(cases.decoder_weights(name), c["spec"], max_seq=c["max_seq"])
    gen = torch.Generator().manual_seed(5)
    ids = torch.randint(0, c["spec"].vocab, (3, 24), generator=gen).to(DEV)
    batched = dec.generate_tokens(ids, 12, eos_token_id=None)
    for b in range(3):
        single = dec.generate_tokens(ids[b:b + 1], 12, eos_token_id=None)
        assert batched[b].tolist() == single[0].tolist()


def test_eos_stops_like_reference():
    name = "decoder_tiny_tp1"
    c = cases.DECODER_CASES[name]
    g = load_golden(name)
    dec = _decoder(cases.decoder_weights(name), c["spec"], max_seq=c["max_seq"])
    ids = cases.decoder_prompt(name).to(DEV)
    ref_toks = g["tokens"].tolist()
    eos = ref_toks[5]
    first = ref_toks.index(eos, 1) if eos in ref_toks[1:] else None
    got = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=eos)
    want = [ref_toks[0]] + (ref_toks[1:first] if first else ref_toks[1:])
    assert got == want


def test_mrope_prefill_vs_oracle():
    """forward_layer with 3-axis position_ids (interleaved M-RoPE) vs the oracle
    layer run on HF-convention cos/sin."""
    c = cases.layer8b_case()
    dec = _decoder(c["weights"], c["spec"], max_seq=512)
    S = 300
    pos = oref.config2_position_ids(seq=S)          # text, 16x16 image, text
    gen = torch.Generator().manual_seed(9)
    hidden = torch.randn(1, S, 4096, generator=gen).to(torch.bfloat16)
    out = dec.forward_layer(hidden.to(DEV), 0, dec.init_kv_cache(1), 0, S,
                            position_ids=pos.to(DEV)).cpu()
    o = odec.OracleDecoder(c["spec"], c["weights"], tp=1)
    cos, sin = oref.mrope_cos_sin(pos, oref.inv_freq(128, 5e6))
    want = o.forward_layer(hidden, 0, o.init_kv_cache(1, 512), 0, rope=(cos[:, None],
                                                                         sin[:, None]))
    compare("mrope layer", out, want, max_abs=5e-2, rel_scale=True, min_cos=0.999)


def test_mrope_layer_vs_transformers_layer():
    """forward_layer with 3-axis position_ids on a text / 16x16 image / text
    prompt vs transformers' Qwen3VLTextDecoderLayer (fixture mrope_layer,
    bf16): max-abs <= 5e-2 of the output scale, cosine >= 0.999."""
    g = load_golden("mrope_layer")
    spec = cases.MROPE_LAYER_SPEC
    w = odec.make_weights(spec, seed=17, std=0.05, random_norms=True)
    _, hidden, pos = cases.mrope_layer_case()
    dec = _decoder(w, spec, max_seq=spec.max_seq)
    out = dec.forward_layer(hidden.to(DEV), 0, dec.init_kv_cache(1), 0, cases.MROPE_LAYER_S,
                            position_ids=pos.to(DEV)).cpu()
    compare("mrope layer vs transformers", out, as_tensor(g["bf16"]), max_abs=5e-2,
            rel_scale=True, min_cos=0.999)


@pytest.mark.parametrize("graphs", [True, False])
def test_multimodal_generate_matches_transformers(graphs):
    """generate_with_embeds on a text / image / text prompt with 3-axis
    position ids, deepstack features and the rope delta: the two greedy tokens
    of transformers' Qwen3VLTextModel (prefill, then a cached decode step at
    P + delta; fixture mm_decode)."""
    g = load_golden("mm_decode")
    name = "decoder_tiny_tp1"
    c = cases.DECODER_CASES[name]
    w, emb, pos, delta, mask, deep = cases.mm_decode_case()
    dec = _decoder(w, c["spec"], max_seq=c["max_seq"])
    dec.use_graphs = graphs
    toks = dec.generate_with_embeds(emb.to(DEV), max_new_tokens=2, eos_token_id=-1,
                                    deepstack_embeds=[d.to(DEV) for d in deep],
                                    visual_mask=mask.to(DEV), position_ids=pos.to(DEV),
                                    rope_delta=delta)
    assert toks == g["tokens"].tolist()


@pytest.mark.parametrize("graphs", [True, False])
def test_batched_multimodal_generate_with_per_sequence_deltas(graphs):
    """Two image prompts of one length but different layouts (rope deltas -30
    and -24) generated as one batch give each prompt's own tokens."""
    import numpy as np
    name = "decoder_tiny8_tp1"
    c = cases.DECODER_CASES[name]
    w = cases.decoder_weights(name)
    dec = _decoder(w, c["spec"], max_seq=c["max_seq"])
    dec.use_graphs = graphs
    g = torch.Generator().manual_seed(3)

    def prompt(t0, grid, t1):
        n_img = grid[0] * (grid[1] // 2) * (grid[2] // 2)
        P = t0 + n_img + t1
        ids = torch.randint(0, 1024, (1, P), generator=g)
        emb = w["embed"][ids].clone()
        types = np.zeros((1, P), np.int32)
        types[0, t0:t0 + n_img] = 1
        emb[0, torch.from_numpy(types[0] == 1)] = (torch.randn(n_img, 512, generator=g) *
                                                   0.05).to(torch.bfloat16)
        pos, delta = oref.rope_index(types, None, np.array([list(grid)]), None, 2)
        return emb, pos, int(delta[0])

    rows = [prompt(6, (1, 12, 12), 18), prompt(10, (1, 8, 16), 18)]
    assert [d for _, _, d in rows] == [-30, -24]
    alone = [dec.generate_with_embeds(e.to(DEV), max_new_tokens=6, eos_token_id=-1,
                                      position_ids=p.to(DEV), rope_delta=d) for e, p, d in rows]
    batch = dec.generate_with_embeds(torch.cat([r[0] for r in rows]).to(DEV), max_new_tokens=6,
                                     eos_token_id=-1,
                                     position_ids=torch.cat([r[1] for r in rows], 1).to(DEV),
                                     rope_delta=torch.tensor([[-30], [-24]]))
    assert batch == alone


def test_generate_with_embeds_deepstack():
    name = "decoder_tiny_tp1"
    c = cases.DECODER_CASES[name]
    w = cases.decoder_weights(name)
    dec = _decoder(w, c["spec"], max_seq=c["max_seq"])
    ids = cases.decoder_prompt(name)
    emb = w["embed"][ids]
    mask = torch.zeros(ids.shape[1], dtype=torch.bool)
    mask[5:15] = True
    gen = torch.Generator().manual_seed(4)
    ds = [torch.randn(10, 512, generator=gen).to(torch.bfloat16) for _ in range(2)]
    got = dec.generate_with_embeds(emb.to(DEV), max_new_tokens=8, eos_token_id=-1,
                                   deepstack_embeds=[d.to(DEV) for d in ds],
                                   visual_mask=mask.to(DEV))
    # oracle: deepstack add after layers 0 and 1 (model_fused.py:339-341)
    o = odec.OracleDecoder(c["spec"], w, tp=1)
    kv = o.init_kv_cache(1, c["max_seq"])
    h = emb.clone()
    for i in range(o.n_layers):
        h = o.forward_layer(h, i, kv, 0)
        if i < len(ds):
            h = h.clone()
            h[0, mask] = h[0, mask] + ds[i]
    toks = [int(o.logits(h)[0, -1].argmax())]
    P = ids.shape[1]
    for i in range(7):
        lg = o.forward(torch.tensor([[toks[-1]]]), P + i, kv)
        toks.append(int(lg[0, -1].argmax()))
    assert got == toks


def test_generate_with_embeds_deepstack_batched_rows():
    """A [B, S] visual mask injects each sequence's own deepstack rows: a batch
    of two prompts gives the tokens each prompt gives alone."""
    name = "decoder_tiny_tp1"
    c = cases.DECODER_CASES[name]
    w = cases.decoder_weights(name)
    dec = _decoder(w, c["spec"], max_seq=c["max_seq"])
    ids = cases.decoder_prompt(name)
    P = ids.shape[1]
    ids2 = torch.roll(ids, 7, dims=1)
    emb = torch.cat([w["embed"][ids], w["embed"][ids2]], 0)      # [2, P, H]
    mask = torch.zeros(2, P, dtype=torch.bool)
    mask[0, 5:15] = True
    mask[1, 20:26] = True
    gen = torch.Generator().manual_seed(5)
    ds = [torch.randn(16, 512, generator=gen).to(torch.bfloat16) for _ in range(2)]
    got = dec.generate_with_embeds(emb.to(DEV), max_new_tokens=8, eos_token_id=-1,
                                   deepstack_embeds=[d.to(DEV) for d in ds],
                                   visual_mask=mask.to(DEV))
    for b, (lo, hi) in enumerate(((0, 10), (10, 16))):
        one = dec.generate_with_embeds(emb[b:b + 1].to(DEV), max_new_tokens=8, eos_token_id=-1,
                                       deepstack_embeds=[d[lo:hi].to(DEV) for d in ds],
                                       visual_mask=mask[b].to(DEV))
        assert got[b] == one, f"row {b}: batched {got[b]} vs alone {one}"


def test_random_init_loader_shapes():
    spec = loader_fused.TextSpec(hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=2048,
                                 layers=2)
    dec = loader_fused.random_decoder(spec, 0, 1, DEV, seed=3, max_seq=128)
    assert dec.layers[0].attn_block.qkv_weight.shape == (512, (8 + 4) * 128)
    assert dec.layers[0].mlp_block.gate_up_weight.shape == (512, 2048)
    out = dec.generate(torch.randint(0, 2048, (1, 16)).to(DEV), max_new_tokens=4,
                       eos_token_id=-1)
    assert len(out) == 4
