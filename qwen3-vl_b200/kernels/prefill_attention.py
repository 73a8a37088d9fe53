"""prefill_gqa_flash_attention on B200 -- drop-in for kernels/prefill_attention.py:28-149.

Layouts as the reference: q (num_q_heads, head_dim, seq_len), k (num_kv_heads,
head_dim, seq_len), v (num_kv_heads, seq_len, head_dim), all bf16; returns
(num_q_heads, seq_len, head_dim) bf16.  The NKI transpose helper `identity`
is ignored.  `mask` must be the causal mask the reference builds
(0 on and below the diagonal, -inf above; kernels/prefill_attention.py:12-13)
or None; the causal structure is applied inside the kernel instead of reading
an S x S mask from memory.
"""
from __future__ import annotations

import math

import torch

from q3vl import ops


def _check_causal(mask: torch.Tensor, S: int):
    if mask is None:
        return
    if mask.shape != (S, S):
        raise ValueError(f"mask must be ({S}, {S}), got {tuple(mask.shape)}")
    # spot-check the structure on a few rows instead of scanning S*S values
    rows = torch.unique(torch.tensor([0, S // 2, S - 1], device=mask.device))
    for r in rows.tolist():
        row = mask[r].float()
        if not (torch.all(row[:r + 1] == 0) and torch.all(torch.isinf(row[r + 1:]))):
            raise ValueError("only the causal mask (0 at/below the diagonal, -inf above) "
                             "is supported")


def prefill_gqa_flash_attention(q, k, v, identity=None, mask=None, softmax_scale=None,
                                num_q_heads=4, num_kv_heads=1, head_dim=128):
    Hq, D, S = q.shape
    if Hq != num_q_heads or k.shape[0] != num_kv_heads or D != head_dim:
        raise ValueError("prefill_gqa_flash_attention: shapes do not match the head counts")
    _check_causal(mask, S)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    qb = q.transpose(1, 2).contiguous()[None]           # [1, Hq, S, D]
    kb = k.transpose(1, 2).contiguous()[None]           # [1, Hkv, S, D]
    vb = v.contiguous()[None]
    return ops.attn_prefill(qb, kb, vb, causal=True, scale=scale)[0]
