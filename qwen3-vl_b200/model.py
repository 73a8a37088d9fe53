"""Per-matmul Qwen3-VL decoder API on B200 -- drop-in for the reference model.py.

Same names as model.py:24-346: FusedLinear, RMSNorm, RotaryEmbedding,
apply_rotary, head_rms_norm, DecoderLayer(qkv, o_proj, gate_up, down,
input_norm, post_norm, q_norm_weight, k_norm_weight) and Qwen3VLDecoder.
The decoder runs the same fused kernel sequence as model_fused: each
DecoderLayer's modules are wrapped into the fused blocks once, at
construction, without copying the math.
"""
from __future__ import annotations

import torch

import model_fused as mf
from model_fused import FusedLinear, RMSNorm, RotaryEmbedding  # noqa: F401  (same API)
from q3vl import ops


def apply_rotary(x, cos, sin):
    """model.py:68-77: rotate_half RoPE on x [B, H, S, D] with cos/sin [S, D/2]."""
    B, H, S, D = x.shape
    xs = x.permute(2, 0, 1, 3).reshape(S, B * H, D).contiguous()
    cs = torch.cat([cos, sin], dim=-1).float().contiguous()
    return ops.rope(xs, cs).view(S, B, H, D).permute(1, 2, 0, 3)


def head_rms_norm(x, weight, eps=1e-6):
    """model.py:80-84: per-head RMSNorm over head_dim."""
    return ops.rmsnorm(x.contiguous(), weight, eps)


class DecoderLayer:
    """model.py:87-97."""

    def __init__(self, qkv, o_proj, gate_up, down, input_norm, post_norm, q_norm_weight,
                 k_norm_weight):
        self.qkv = qkv
        self.o_proj = o_proj
        self.gate_up = gate_up
        self.down = down
        self.input_norm = input_norm
        self.post_norm = post_norm
        self.q_norm_weight = q_norm_weight
        self.k_norm_weight = k_norm_weight


def _fused_layer(layer: DecoderLayer, Hq: int, Hkv: int, D: int) -> mf.DecoderLayer:
    eps = getattr(layer.input_norm, "eps", 1e-6)
    attn = mf.AttentionBlock(layer.qkv.weight, layer.qkv.bias, layer.o_proj.weight,
                             layer.input_norm.weight, layer.q_norm_weight, layer.k_norm_weight,
                             Hq, Hkv, D, eps)
    mlp = mf.MLPBlock(layer.gate_up.weight, layer.down.weight, layer.post_norm.weight,
                      getattr(layer.post_norm, "eps", eps))
    return mf.DecoderLayer(attn, mf.OProjection(layer.o_proj.weight), mlp)


class Qwen3VLDecoder(mf.Qwen3VLDecoderFused):
    """model.py:100-346: same constructor and methods (init_kv_cache,
    forward_layer, forward, prefill, decode_step, generate, generate_with_embeds)."""

    def __init__(self, layers, lm_head, embed_tokens, final_norm, rotary, tp_size, num_q_heads,
                 num_kv_heads, head_dim, max_seq_len, device):
        self.source_layers = layers
        fused = [_fused_layer(l, num_q_heads, num_kv_heads, head_dim) for l in layers]
        super().__init__(fused, lm_head, embed_tokens, final_norm, rotary, tp_size, num_q_heads,
                         num_kv_heads, head_dim, max_seq_len, device)
        self.kv_dim = num_kv_heads * head_dim
