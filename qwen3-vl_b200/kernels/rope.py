"""qwen3_rope on B200 -- drop-in for kernels/rope.py:24-96.

x (seq_len, num_heads, head_dim) bf16, cos_sin (seq_len, head_dim) f32 with
cos in the first head_dim/2 columns and sin in the rest; returns
x * cat(cos, cos) + rotate_half(x) * cat(sin, sin) in fp32, rounded to bf16
(bit-identical to the reference test's rope_ref, test_kernels.py:126-134).
The reference requires seq_len % 128 == 0 (kernels/rope.py:46); this kernel
accepts any seq_len and keeps that check only as an explicit opt-in.
"""
from __future__ import annotations

import torch

from q3vl import ops


def qwen3_rope(x: torch.Tensor, cos_sin: torch.Tensor, num_heads: int = 4,
               head_dim: int = 128, require_tile_multiple: bool = False) -> torch.Tensor:
    if x.dim() != 3 or x.shape[1] != num_heads or x.shape[2] != head_dim:
        raise ValueError(f"qwen3_rope: x must be (seq_len, {num_heads}, {head_dim}), "
                         f"got {tuple(x.shape)}")
    if require_tile_multiple and x.shape[0] % 128:
        raise ValueError("qwen3_rope: seq_len must be a multiple of 128")
    return ops.rope(x.contiguous(), cos_sin.float().contiguous())
