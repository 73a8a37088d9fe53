"""Weight fusing + tensor-parallel sharding -- drop-in for the reference
loader_fused.py (load_model(model_path, rank, world_size, device,
compile_backend) -> (decoder, vision_model, processor, hf_model)).

Two sources of weights:
  * an HF Qwen3-VL checkpoint directory (the reference path,
    loader_fused.py:55-177): q/k/v fused and column-sharded, o/down
    row-sharded, gate/up column-sharded, lm_head vocab-sharded, exactly the
    reference's layout rules;
  * `random:<seed>` (or a missing path): seeded N(0, 0.02) bf16 weights of the
    Qwen3-VL-8B text decoder shape, generated directly on the device per rank
    (no checkpoint or tokenizer ships with this repository).
compile_backend is accepted for signature compatibility and ignored: the
kernels are precompiled for sm_100a.
"""
from __future__ import annotations

import dataclasses
import os
import time

import torch

from model_fused import (AttentionBlock, DecoderLayer, FusedLinear, MLPBlock, OProjection,
                         Qwen3VLDecoderFused, RMSNorm, RotaryEmbedding)


def shard_column(weight, rank, tp):
    """loader_fused.py:28-30: rows [rank*n, (rank+1)*n) of an [out, in] weight."""
    chunk = weight.shape[0] // tp
    return weight[rank * chunk:(rank + 1) * chunk].contiguous()


def shard_row(weight, rank, tp):
    """loader_fused.py:33-35: columns [rank*n, (rank+1)*n) of an [out, in] weight."""
    chunk = weight.shape[1] // tp
    return weight[:, rank * chunk:(rank + 1) * chunk].contiguous()


@dataclasses.dataclass
class TextSpec:
    hidden: int = 4096
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 12288
    vocab: int = 151936
    layers: int = 36
    rope_theta: float = 5e6
    eps: float = 1e-6


QWEN3_VL_8B = TextSpec()


def build_decoder(layer_weights, embed, final_norm, lm_head, spec, rank, tp, device,
                  max_seq=None):
    """Fuse, shard and wrap HF-convention ([out, in]) weights into a
    Qwen3VLDecoderFused (loader_fused.py:82-219).  `layer_weights` is a list of
    dicts with q, k, v, o, gate, up, down, input_norm, post_norm, q_norm, k_norm;
    tensors may already be on `device`."""
    if spec.q_heads % tp or spec.kv_heads % tp:
        raise ValueError(f"tp={tp} must divide {spec.q_heads} q and {spec.kv_heads} kv heads")
    dev = torch.device(device)
    hq, hkv = spec.q_heads // tp, spec.kv_heads // tp
    layers = []
    for lw in layer_weights:
        lw = {k: v.to(dev) for k, v in lw.items()}
        qkv = torch.cat([shard_column(lw["q"], rank, tp), shard_column(lw["k"], rank, tp),
                         shard_column(lw["v"], rank, tp)], dim=0).t()
        o = shard_row(lw["o"], rank, tp).t()
        gu = torch.cat([shard_column(lw["gate"], rank, tp),
                        shard_column(lw["up"], rank, tp)], dim=0).t()
        down = shard_row(lw["down"], rank, tp).t()
        attn = AttentionBlock(qkv, lw.get("qkv_bias"), o, lw["input_norm"], lw["q_norm"],
                              lw["k_norm"], hq, hkv, spec.head_dim, spec.eps)
        layers.append(DecoderLayer(attn, OProjection(o), MLPBlock(gu, down, lw["post_norm"],
                                                                  spec.eps)))
        del lw, qkv, o, gu, down
    n = lm_head.shape[0] // tp
    lm = FusedLinear(lm_head[rank * n:(rank + 1) * n].to(dev).t())
    emb = torch.nn.Embedding.from_pretrained(embed.to(dev), freeze=True)
    fn = RMSNorm(final_norm.to(dev), eps=spec.eps)
    if max_seq is None:
        max_seq = int(os.environ.get("MAX_SEQ_LEN", "4096"))
    rot = RotaryEmbedding(spec.head_dim, max_seq_len=max_seq, base=spec.rope_theta)
    return Qwen3VLDecoderFused(layers, lm, emb, fn, rot, tp, hq, hkv, spec.head_dim, max_seq,
                               dev)


def random_layer_weights(spec: TextSpec, layer: int, seed: int, device, std: float = 0.02):
    """Seeded N(0, std) bf16 weights of one layer, generated on `device` (the
    whole tensor, so every TP degree shards the same global weights)."""
    H, I, D = spec.hidden, spec.inter, spec.head_dim
    shapes = dict(q=(spec.q_heads * D, H), k=(spec.kv_heads * D, H), v=(spec.kv_heads * D, H),
                  o=(H, spec.q_heads * D), gate=(I, H), up=(I, H), down=(H, I))
    out = {}
    for j, (name, shp) in enumerate(shapes.items()):
        g = torch.Generator(device=device).manual_seed(seed * 1000003 + layer * 97 + j)
        out[name] = (torch.randn(*shp, generator=g, device=device, dtype=torch.float32)
                     * std).to(torch.bfloat16)
    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=device)  # noqa: E731
    out.update(input_norm=ones(H), post_norm=ones(H), q_norm=ones(D), k_norm=ones(D))
    return out


def random_decoder(spec: TextSpec, rank: int, tp: int, device, seed: int = 0, max_seq=None,
                   std: float = 0.02):
    dev = torch.device(device)
    # a generator: each layer's full weights are made, sharded and dropped in turn
    layers = (random_layer_weights(spec, i, seed, dev, std) for i in range(spec.layers))

    def rn(shape, j):
        g = torch.Generator(device=dev).manual_seed(seed * 1000003 + 99991 * (j + 1))
        return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

    embed = rn((spec.vocab, spec.hidden), 1)
    lm_head = rn((spec.vocab, spec.hidden), 2)
    final_norm = torch.ones(spec.hidden, dtype=torch.bfloat16, device=dev)
    return build_decoder(layers, embed, final_norm, lm_head, spec, rank, tp, dev, max_seq)


def _hf_layer_weights(lang_model, i, H, D):
    attn = lang_model.layers[i].self_attn
    mlp = lang_model.layers[i].mlp
    lw = dict(q=attn.q_proj.weight.data, k=attn.k_proj.weight.data, v=attn.v_proj.weight.data,
              o=attn.o_proj.weight.data, gate=mlp.gate_proj.weight.data,
              up=mlp.up_proj.weight.data, down=mlp.down_proj.weight.data,
              input_norm=lang_model.layers[i].input_layernorm.weight.data.clone(),
              post_norm=lang_model.layers[i].post_attention_layernorm.weight.data.clone())
    if hasattr(attn, "q_norm"):
        lw["q_norm"] = attn.q_norm.weight.data.clone()
        lw["k_norm"] = attn.k_norm.weight.data.clone()
    else:
        lw["q_norm"] = torch.ones(D, dtype=torch.bfloat16)
        lw["k_norm"] = torch.ones(D, dtype=torch.bfloat16)
    return lw


def _head_dim(cfg) -> int:
    """The attention head size of a text config.  loader_fused.py:69 takes
    hidden // heads, which equals the config's head_dim for Qwen3-VL-8B (4096 /
    32 = 128); other sizes set head_dim apart from it (the weights' shapes
    follow head_dim), so it is read from the config when present."""
    hd = getattr(cfg, "head_dim", None)
    return int(hd) if hd else cfg.hidden_size // cfg.num_attention_heads


def load_model(model_path, rank, world_size, device, compile_backend='neuron'):
    """loader_fused.py:38-237.  Returns (decoder, vision_model, processor, hf_model).

    model_path names a local Hugging Face checkpoint directory; a path that
    does not exist raises FileNotFoundError, as from_pretrained does in the
    reference (loader_fused.py:56-60).  Random-init weights are served only on
    an explicit request: model_path "random" (seed 0) or "random:<seed>", which
    returns (decoder, None, None, None)."""
    t0 = time.time()
    mp = "" if model_path is None else str(model_path)
    if mp == "random" or mp.startswith("random:"):
        seed = int(mp.split(":", 1)[1]) if ":" in mp else 0
        dec = random_decoder(QWEN3_VL_8B, rank, world_size, device, seed=seed)
        if rank == 0:
            print(f"[LOAD] random-init Qwen3-VL-8B text decoder, TP-{world_size}: "
                  f"{time.time() - t0:.1f}s")
        return dec, None, None, None
    if not os.path.isdir(mp):
        raise FileNotFoundError(
            f"load_model: checkpoint directory {mp!r} does not exist (pass 'random' or "
            f"'random:<seed>' for random-init weights)")

    from transformers import AutoModelForImageTextToText, AutoProcessor
    processor = AutoProcessor.from_pretrained(model_path)
    hf_model = AutoModelForImageTextToText.from_pretrained(
        model_path, dtype=torch.bfloat16, attn_implementation="eager").eval().requires_grad_(False)
    lang = hf_model.model.language_model
    cfg = lang.config
    rope_theta = getattr(cfg, "rope_theta", None)
    if rope_theta is None:
        rope_theta = (getattr(cfg, "rope_scaling", {}) or {}).get("rope_theta", 1000000.0)
    spec = TextSpec(hidden=cfg.hidden_size, q_heads=cfg.num_attention_heads,
                    kv_heads=cfg.num_key_value_heads,
                    head_dim=_head_dim(cfg),
                    inter=cfg.intermediate_size, vocab=hf_model.lm_head.weight.shape[0],
                    layers=cfg.num_hidden_layers, rope_theta=rope_theta, eps=cfg.rms_norm_eps)
    layers = [_hf_layer_weights(lang, i, spec.hidden, spec.head_dim) for i in range(spec.layers)]
    if hasattr(lang, "norm"):
        final_norm = lang.norm.weight.data.clone()
    elif hasattr(lang, "final_layernorm"):
        final_norm = lang.final_layernorm.weight.data.clone()
    else:
        raise AttributeError("Cannot find final norm")
    dec = build_decoder(layers, lang.embed_tokens.weight.data, final_norm,
                        hf_model.lm_head.weight.data, spec, rank, world_size, device)
    vision = None
    if hasattr(hf_model.model, "visual"):
        vision = hf_model.model.visual.to(device)
    elif hasattr(hf_model.model, "vision_model"):
        vision = hf_model.model.vision_model.to(device)
    if rank == 0:
        print(f"[READY] Qwen3-VL decoder on q3vl kernels, TP-{world_size}: "
              f"{time.time() - t0:.1f}s")
    return dec, vision, processor, hf_model
