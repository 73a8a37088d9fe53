"""Prefill attention on the tcgen05 tensor cores (q3_attn_prefill_tc) vs fp32
attention and vs the mma.sync kernel, and through the decoder
(Q3VL_PREFILL_TC).  Variants 0 (V transposed in shared memory), 1 (V as an
MN-major operand with O in TMEM) and 2 (two heads of a KV group per CTA,
128-key tiles, P in TMEM; needs Hq/Hkv even).  Tolerances: max-abs <= 2e-2
and cosine >= 0.9999 against fp32, as for q3_attn_prefill."""
import math

import pytest
import torch

from oracle import ref as oref
from q3vl import ops
from tests.golden import cases
from tests.helpers import compare

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF16 = torch.bfloat16


def rnd(*shape, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(BF16)


@pytest.mark.parametrize("B,Hq,Hkv,S,start,causal,rows",
                         [(1, 32, 8, 2048, 0, True, 2048),     # the prefill benchmark shape
                          (2, 8, 2, 200, 0, True, 256),       # cache longer than the prompt
                          (1, 4, 1, 130, 70, True, 512),      # prompt continuing at 70
                          (1, 8, 8, 96, 0, False, 96),
                          (3, 4, 4, 1, 37, True, 64),          # one query row
                          (1, 4, 1, 700, 0, True, 700),        # 6 query blocks, ragged tail
                          (2, 8, 2, 333, 5, False, 400)])      # non-causal, ragged, offset
@pytest.mark.parametrize("variant", [0, 1, 2])
def test_tc_prefill_matches_fp32(B, Hq, Hkv, S, start, causal, rows, variant):
    if variant == 2 and (Hq // Hkv) % 2:
        pytest.skip("variant 2 pairs the query heads of a KV head")
    q = rnd(B, Hq, S, 128, seed=30)
    k = rnd(B, Hkv, rows, 128, seed=31)
    v = rnd(B, Hkv, rows, 128, seed=32)
    out = ops.attn_prefill_tc(q.to(DEV), k.to(DEV), v.to(DEV), start_pos=start,
                              causal=causal, variant=variant).cpu()
    if causal:
        want = oref.causal_attention_fp32(q, k, v, start)
    else:
        # keys 0 .. start + S - 1 (the cache rows this call may read)
        rep, kk, vv = Hq // Hkv, k[:, :, :start + S], v[:, :, :start + S]
        s = q.float() @ kk.float().repeat_interleave(rep, 1).transpose(-2, -1) / math.sqrt(128)
        want = torch.softmax(s, -1) @ vv.float().repeat_interleave(rep, 1)
    compare("prefill tc", out, want, max_abs=2e-2, min_cos=0.9999)
    # and the mma.sync kernel on the same inputs
    legacy = ops.attn_prefill(q.to(DEV), k.to(DEV), v.to(DEV), start_pos=start,
                              causal=causal).cpu()
    compare("tc vs mma.sync", out, legacy, max_abs=2e-2, min_cos=0.9999)
    assert ops.device_error(clear=True) == 0


@pytest.mark.parametrize("variant", [0, 1, 2])
def test_tc_prefill_writes_the_bshd_layout(variant):
    B, Hq, Hkv, S = 2, 8, 2, 160
    q, k, v = rnd(B, Hq, S, 128, seed=33), rnd(B, Hkv, S, 128, seed=34), rnd(B, Hkv, S, 128, seed=35)
    o = torch.empty(B, S, Hq, 128, dtype=BF16, device=DEV)
    ops.attn_prefill_tc(q.to(DEV), k.to(DEV), v.to(DEV), out=o.transpose(1, 2), variant=variant)
    want = oref.causal_attention_fp32(q, k, v).transpose(1, 2)
    compare("prefill tc bshd", o.cpu(), want, max_abs=2e-2, min_cos=0.9999)


@pytest.mark.parametrize("variant", ["0", "1", "2"])
def test_decoder_generates_the_reference_tokens_with_tc_prefill(variant, monkeypatch):
    monkeypatch.setenv("Q3VL_PREFILL_TC_VARIANT", variant)
    import loader_fused
    from tests.helpers import load_golden
    name = "decoder_tiny_tp1"
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    s = c["spec"]
    spec = loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                 inter=s.inter, vocab=s.vocab, layers=s.layers,
                                 rope_theta=s.rope_theta, eps=s.eps)
    w = cases.decoder_weights(name)
    dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"], w["lm_head"],
                                     spec, 0, 1, DEV, c["max_seq"])
    dec.prefill_tc = True
    ids = cases.decoder_prompt(name).to(DEV)
    toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
    assert toks == g["tokens"].tolist()


def test_tc_prefill_variant1_rescales_on_growing_scores():
    """Scores that grow along the keys move each row's base many times (the
    lazy-rescale path of variant 1); the result must still match fp32."""
    B, Hq, Hkv, S = 1, 4, 1, 640
    g = torch.Generator().manual_seed(36)
    q = torch.randn(B, Hq, S, 128, generator=g)
    k = torch.randn(B, Hkv, S, 128, generator=g) * 0.2
    # a component along q's mean direction that grows with the key index
    dirn = q.mean(dim=(0, 1, 2))
    # (about 20 log2 units over the prompt for a row with unit projection, so
    # the base moves more than once per such row)
    k = k + (torch.arange(S, dtype=torch.float32) / 4.0)[None, None, :, None] * dirn / dirn.norm()
    v = torch.randn(B, Hkv, S, 128, generator=g)
    q, k, v = q.to(BF16), k.to(BF16), v.to(BF16)
    want = oref.causal_attention_fp32(q, k, v, 0)
    for variant in (0, 1, 2):
        out = ops.attn_prefill_tc(q.to(DEV), k.to(DEV), v.to(DEV), variant=variant).cpu()
        compare(f"growing scores, variant {variant}", out, want, max_abs=2e-2, min_cos=0.9999)
    assert ops.device_error(clear=True) == 0
