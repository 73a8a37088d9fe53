"""The persistent whole-step decode kernel (q3_decode_step) against the
per-kernel decode path (each of which is parity-tested against the oracle and
the reference fixtures) on 8B-shape layers, and the golden tiny decoder's
greedy tokens through the decode graph that uses it.

Tolerances (bf16): hidden output and KV rows max-abs <= 2e-2 of the output
scale and cosine >= 0.9999 (the two paths sum the same products in different
orders: split-K partitions and split-attention merges differ); sums of squares
rtol 1e-4; greedy tokens identical to the reference's."""
import dataclasses

import pytest
import torch

import loader_fused
from q3vl import ops
from tests.golden import cases
from tests.helpers import compare, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _decoder(layers=2, seed=3, max_seq=1280):
    spec = dataclasses.replace(loader_fused.QWEN3_VL_8B, layers=layers, vocab=4096)
    return loader_fused.random_decoder(spec, 0, 1, DEV, seed=seed, max_seq=max_seq)


@pytest.mark.parametrize("B,P,rope_delta", [(8, 100, 0), (8, 1151, 0), (12, 64, 7), (1, 1, 0),
                                            (16, 200, 0)])
def test_step_kernel_matches_per_kernel_decode(B, P, rope_delta):
    dec = _decoder()
    g = torch.Generator().manual_seed(B * 1000 + P)
    prompt = torch.randint(0, 4096, (B, P), generator=g).to(DEV)
    kv = dec.init_kv_cache(B)
    logits = dec.forward(prompt, 0, kv)
    tok = ops.argmax(logits.view(B, -1))
    kv2 = [(k.clone(), v.clone()) for k, v in kv]
    # per-kernel path (eager), new token at cache position P
    xa = dec._embed(tok.view(B, 1)).view(B, -1)
    xa, pend = dec._run(xa, B, 1, P, kv, rope_delta=rope_delta)
    assert pend is None
    # whole-step kernel on a copy of the cache
    plan = dec._step_plan(B, kv2)
    ss = torch.full((4096 // 128, 16), float("nan"), device=DEV)
    kv_len = torch.tensor([P + 1], dtype=torch.int32, device=DEV)
    xb = dec._embed(tok.view(B, 1)).view(B, -1).clone()
    plan.run(xb, ss, kv_len, rope_delta)
    torch.cuda.synchronize()
    assert ops.device_error(clear=True) == 0
    compare(f"step hidden B={B} P={P}", xb, xa, max_abs=2e-2, rel_scale=True, min_cos=0.9999)
    for layer, ((ka, va), (kb, vb)) in enumerate(zip(kv, kv2)):
        compare(f"k row layer {layer}", kb[:, :, P], ka[:, :, P], max_abs=2e-2, rel_scale=True,
                min_cos=0.9999)
        compare(f"v row layer {layer}", vb[:, :, P], va[:, :, P], max_abs=2e-2, rel_scale=True,
                min_cos=0.9999)
        # rows before P are untouched
        assert torch.equal(kb[:, :, :P], ka[:, :, :P])
    want_ss = (xb.float() ** 2).view(B, 32, 128).sum(-1).t()
    assert torch.allclose(ss[:, :B], want_ss, rtol=1e-4), (ss[:, :B] - want_ss).abs().max()
    assert torch.all(ss[:, B:] == 0)
    plan.close()


def test_step_kernel_repeated_steps_and_reuse():
    """Two plans' worth of steps on one cache: the kernel's grid counters reset
    themselves between launches, and successive positions extend the cache."""
    B, P = 8, 300
    dec = _decoder(seed=5)
    g = torch.Generator().manual_seed(9)
    prompt = torch.randint(0, 4096, (B, P), generator=g).to(DEV)
    kv = dec.init_kv_cache(B)
    tok = ops.argmax(dec.forward(prompt, 0, kv).view(B, -1))
    kv2 = [(k.clone(), v.clone()) for k, v in kv]
    plan = dec._step_plan(B, kv2)
    ss = torch.zeros(32, 16, device=DEV)
    for i in range(4):
        xa = dec._embed(tok.view(B, 1)).view(B, -1)
        xa, _ = dec._run(xa, B, 1, P + i, kv)
        xb = dec._embed(tok.view(B, 1)).view(B, -1).clone()
        plan.run(xb, ss, torch.tensor([P + i + 1], dtype=torch.int32, device=DEV))
        compare(f"step {i}", xb, xa, max_abs=2e-2, rel_scale=True, min_cos=0.9999)
        tok = ops.argmax(ops.gemm(xa, dec.lm_head.weight_km))  # both paths take the same token
    assert ops.device_error(clear=True) == 0
    plan.close()


def test_golden_tiny_decoder_tokens_through_step_kernel():
    """Greedy tokens of the reference's tiny decoder (fixture decoder_tiny_tp1)
    through the CUDA-graph decode loop built on q3_decode_step."""
    from tests.test_model_gpu import _decoder as build
    name = "decoder_tiny_tp1"
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    dec = build(cases.decoder_weights(name), c["spec"], max_seq=c["max_seq"])
    dec.use_step_kernel = True
    assert dec._step_ok(1)
    dec.use_graphs = True
    ids = cases.decoder_prompt(name).to(DEV)
    toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
    assert len(dec._step_plans) == 1
    assert toks == g["tokens"].tolist()
    assert ops.device_error(clear=True) == 0
    dec.close()
