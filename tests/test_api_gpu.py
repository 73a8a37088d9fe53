"""The reference's kernels/*.py and model.py entry points on the CUDA path,
called with the reference's own layouts and checked against the fixtures."""
import math

import pytest
import torch

import model
from kernels.decode_attention import decode_attention_simple
from kernels.prefill_attention import prefill_gqa_flash_attention
from kernels.rope import qwen3_rope
from oracle import decoder as odec
from oracle import ref as oref
from tests.golden import cases
from tests.helpers import as_tensor, compare, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_qwen3_rope_reference_layout_bit_exact():
    g = load_golden("kernels_kat")
    x, cos, sin, *_ = cases.kernels_kat_inputs()
    cs = torch.cat([cos, sin], dim=-1).float()
    out = qwen3_rope(x.to(DEV), cs.to(DEV), num_heads=4, head_dim=128,
                     require_tile_multiple=True)
    assert torch.equal(out.cpu(), as_tensor(g["rope"]))


def test_prefill_gqa_flash_attention_reference_layout():
    g = load_golden("kernels_kat")
    _, _, _, q, k, v = cases.kernels_kat_inputs()
    S = q.shape[2]
    mask = torch.triu(torch.full((S, S), float("-inf"), dtype=torch.bfloat16), diagonal=1)
    out = prefill_gqa_flash_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                      torch.eye(128, dtype=torch.bfloat16, device=DEV),
                                      mask.to(DEV), 1.0 / math.sqrt(128), 4, 1, 128)
    compare("prefill_gqa_flash_attention", out.cpu(), as_tensor(g["attn"]), max_abs=2e-2,
            min_cos=0.9999)
    with pytest.raises(ValueError):
        prefill_gqa_flash_attention(q.to(DEV), k.to(DEV), v.to(DEV), None,
                                    torch.zeros(S, S, device=DEV), 0.1, 4, 1, 128)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
def test_decode_attention_simple_reference_layout(dtype, tol):
    g = torch.Generator().manual_seed(3)
    Hq, Hkv, Sk, L = 4, 1, 512, 300
    q = torch.randn(Hq, 128, generator=g).to(dtype)
    k = torch.randn(Hkv, 128, Sk, generator=g).to(dtype)   # D-major as the NKI kernel
    v = torch.randn(Hkv, Sk, 128, generator=g).to(dtype)
    mask = torch.full((128, Sk), float("-inf"), dtype=torch.bfloat16)
    mask[0, :L] = 0
    out = decode_attention_simple(q.to(DEV), k.to(DEV), v.to(DEV), mask.to(DEV), None,
                                  1.0 / math.sqrt(128), Hq, Hkv, 128)
    want = oref.decode_attention_fp32(q[None].float(), k.transpose(1, 2)[None, :, :L].float(),
                                      v[None, :, :L].float())[0]
    compare("decode_attention_simple", out.cpu(), want, max_abs=tol, min_cos=0.9999)


def test_model_py_decoder_matches_reference_tokens():
    """model.Qwen3VLDecoder built from per-matmul modules (model.py:87-97)."""
    name = "decoder_tiny_tp1"
    g = load_golden(name)
    c = cases.DECODER_CASES[name]
    w = cases.decoder_weights(name)
    s = c["spec"]
    layers = []
    for lw in w["layers"]:
        sh = odec.shard_layer(lw, 0, 1)
        dev = {k: v.to(DEV) for k, v in sh.items()}
        layers.append(model.DecoderLayer(
            model.FusedLinear(dev["qkv"]), model.FusedLinear(dev["o"]),
            model.FusedLinear(dev["gate_up"]), model.FusedLinear(dev["down"]),
            model.RMSNorm(dev["input_norm"]), model.RMSNorm(dev["post_norm"]),
            dev["q_norm"], dev["k_norm"]))
    dec = model.Qwen3VLDecoder(
        layers, model.FusedLinear(w["lm_head"].t().contiguous().to(DEV)),
        torch.nn.Embedding.from_pretrained(w["embed"].to(DEV)),
        model.RMSNorm(w["final_norm"].to(DEV)), model.RotaryEmbedding(128, c["max_seq"], 5e6),
        1, s.q_heads, s.kv_heads, 128, c["max_seq"], DEV)
    ids = cases.decoder_prompt(name).to(DEV)
    assert dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1) == \
        g["tokens"].tolist()
    # helper functions keep the reference semantics
    x = torch.randn(2, 4, 8, 128, dtype=torch.bfloat16)
    wn = (1 + 0.1 * torch.randn(128)).to(torch.bfloat16)
    compare("head_rms_norm", model.head_rms_norm(x.to(DEV), wn.to(DEV)).cpu(),
            oref.rmsnorm(x, wn), max_abs=3.2e-2, min_cos=0.99999)
    cos, sin = oref.rotary_tables(128, 8, 5e6)
    compare("apply_rotary", model.apply_rotary(x.to(DEV), cos.to(DEV), sin.to(DEV)).cpu(),
            x * torch.cat([cos, cos], -1) + oref.rotate_half(x) * torch.cat([sin, sin], -1),
            max_abs=3.2e-2, min_cos=0.99999)
