"""Restated reference decoder with tensor-parallel emulation (CPU).

Test infrastructure (see oracle/__init__.py).  Restates
Qwen3VLDecoderFused.forward_layer / forward / generate (model_fused.py:234-328)
over weights sharded exactly as loader_fused.py:28-35,82-109 shards them;
`tp` ranks are emulated in one process and the all-reduce of
model_fused.py:267,274 is the sum of the ranks' bf16 partials (fp32 sum,
one bf16 rounding).
"""
from __future__ import annotations

import dataclasses

import torch

from . import ref

D = ref.HEAD_DIM


@dataclasses.dataclass
class Spec:
    hidden: int = 4096
    q_heads: int = 32
    kv_heads: int = 8
    inter: int = 12288
    vocab: int = 151936
    layers: int = 36
    max_seq: int = 4096
    rope_theta: float = 5e6
    eps: float = 1e-6


QWEN3_VL_8B = Spec()


def make_weights(spec: Spec, seed: int = 0, std: float = 0.02, random_norms: bool = False,
                 n_layers: int | None = None, on_layer=None):
    """HF-convention ([out, in]) seeded N(0, std) bf16 weights, drawn layer by
    layer (q, k, v, o, gate, up, down, norms), then embedding, final norm and
    lm_head.  Norm weights are 1.0 unless random_norms (1 + N(0, 0.1)).
    on_layer(i, layer_dict), when given, receives each layer as soon as it is
    drawn and its return value is kept in its place (a caller that shards the
    layer keeps only its shard, so an 8B-shape model never sits whole in
    memory); the draws, and so the weights, are the same either way."""
    g = torch.Generator().manual_seed(seed)
    H, I = spec.hidden, spec.inter
    qd, kd = spec.q_heads * D, spec.kv_heads * D

    def rn(*shape, s=std):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * s).to(torch.bfloat16)

    def norm(n):
        if random_norms:
            return (1.0 + torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
        return torch.ones(n, dtype=torch.bfloat16)

    layers = []
    for i in range(spec.layers if n_layers is None else n_layers):
        lw = dict(
            q=rn(qd, H), k=rn(kd, H), v=rn(kd, H), o=rn(H, qd),
            gate=rn(I, H), up=rn(I, H), down=rn(H, I),
            input_norm=norm(H), post_norm=norm(H), q_norm=norm(D), k_norm=norm(D))
        layers.append(lw if on_layer is None else on_layer(i, lw))
    embed = rn(spec.vocab, H)
    final_norm = norm(H)
    lm_head = rn(spec.vocab, H)
    return dict(layers=layers, embed=embed, final_norm=final_norm, lm_head=lm_head)


# -- loader_fused.py:28-35 --------------------------------------------------
def shard_column(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    n = w.shape[0] // tp
    return w[rank * n:(rank + 1) * n].contiguous()


def shard_row(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    n = w.shape[1] // tp
    return w[:, rank * n:(rank + 1) * n].contiguous()


def shard_layer(lw: dict, rank: int, tp: int) -> dict:
    """Per-rank fused [in, out] weights (loader_fused.py:87-121)."""
    qkv = torch.cat([shard_column(lw["q"], rank, tp), shard_column(lw["k"], rank, tp),
                     shard_column(lw["v"], rank, tp)], dim=0).t().contiguous()
    gate_up = torch.cat([shard_column(lw["gate"], rank, tp),
                         shard_column(lw["up"], rank, tp)], dim=0).t().contiguous()
    return dict(qkv=qkv, o=shard_row(lw["o"], rank, tp).t().contiguous(), gate_up=gate_up,
                down=shard_row(lw["down"], rank, tp).t().contiguous(),
                input_norm=lw["input_norm"], post_norm=lw["post_norm"],
                q_norm=lw["q_norm"], k_norm=lw["k_norm"])


def shard_lm_head(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    n = w.shape[0] // tp
    return w[rank * n:(rank + 1) * n].t().contiguous()  # loader_fused.py:153-157


def allreduce_sum(parts):
    acc = parts[0].float()
    for p in parts[1:]:
        acc = acc + p.float()
    return acc.to(parts[0].dtype)


class OracleDecoder:
    """Qwen3VLDecoderFused semantics on CPU for `tp` emulated ranks."""

    def __init__(self, spec: Spec, weights: dict, tp: int = 1):
        self.spec, self.tp = spec, tp
        self.hq = spec.q_heads // tp
        self.hkv = spec.kv_heads // tp
        self.shards = [[shard_layer(lw, r, tp) for r in range(tp)] for lw in weights["layers"]]
        self.lm_head = [shard_lm_head(weights["lm_head"], r, tp) for r in range(tp)]
        self.embed = weights["embed"]
        self.final_norm = weights["final_norm"]
        self.cos, self.sin = ref.rotary_tables(D, spec.max_seq, spec.rope_theta)
        self.n_layers = len(weights["layers"])

    def init_kv_cache(self, B: int, max_seq: int | None = None):
        """caches[layer][rank] = (k, v) [B, Hkv/tp, max_seq, D] (model_fused.py:224-232)."""
        S = self.spec.max_seq if max_seq is None else max_seq
        return [[(torch.zeros(B, self.hkv, S, D, dtype=torch.bfloat16),
                  torch.zeros(B, self.hkv, S, D, dtype=torch.bfloat16))
                 for _ in range(self.tp)] for _ in range(self.n_layers)]

    def forward_layer(self, hidden, layer: int, caches, start_pos: int, rope=None):
        """model_fused.py:234-277.  rope=(cos, sin) [B,1,S,D] overrides the 1-D table."""
        B, S, _ = hidden.shape
        if rope is None:
            cos = self.cos[start_pos:start_pos + S]
            sin = self.sin[start_pos:start_pos + S]
        else:
            cos, sin = rope
        attn_parts = []
        for r in range(self.tp):
            w = self.shards[layer][r]
            q, k, v = ref.attention_block(hidden, w["qkv"], None, w["input_norm"], w["q_norm"],
                                          w["k_norm"], cos, sin, self.hq, self.hkv,
                                          self.spec.eps)
            kc, vc = caches[layer][r]
            kc[:, :, start_pos:start_pos + S] = k
            vc[:, :, start_pos:start_pos + S] = v
            a = ref.eager_attention(q, kc, vc, start_pos)
            a = a.transpose(1, 2).contiguous().view(B, S, self.hq * D)
            attn_parts.append(a @ w["o"])
        hidden = hidden + allreduce_sum(attn_parts)
        mlp_parts = [ref.mlp_block(hidden, self.shards[layer][r]["gate_up"],
                                   self.shards[layer][r]["down"],
                                   self.shards[layer][r]["post_norm"], self.spec.eps)
                     for r in range(self.tp)]
        return hidden + allreduce_sum(mlp_parts)

    def logits(self, hidden):
        """final norm + lm_head on the last token + all_gather (model_fused.py:286-293)."""
        h = ref.rmsnorm(hidden, self.final_norm, self.spec.eps)[:, -1:, :]
        return torch.cat([h @ self.lm_head[r] for r in range(self.tp)], dim=-1)

    def forward(self, input_ids, start_pos: int, caches, n_layers: int | None = None):
        hidden = self.embed[input_ids]
        for i in range(self.n_layers if n_layers is None else n_layers):
            hidden = self.forward_layer(hidden, i, caches, start_pos)
        return self.logits(hidden)

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens: int, eos_token_id: int = 151645,
                 max_seq: int | None = None):
        """Greedy decode (model_fused.py:302-328), batched: returns [B, T] ids with
        each row cut at its first EOS (EOS itself excluded, as the reference)."""
        B, P = input_ids.shape
        caches = self.init_kv_cache(B, max_seq)
        nxt = self.forward(input_ids, 0, caches)[:, -1, :].argmax(-1)
        out = [nxt]
        for i in range(max_new_tokens - 1):
            nxt = self.forward(nxt.view(B, 1), P + i, caches)[:, -1, :].argmax(-1)
            out.append(nxt)
        return torch.stack(out, dim=1)
