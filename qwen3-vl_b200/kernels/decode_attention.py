"""decode_attention_simple on B200 -- drop-in for kernels/decode_attention.py:56-134.

The reference kernel is an unfinished stub that returns q
(kernels/decode_attention.py:122-134); its intended semantics are the S=1
eager attention of forward_layer (model_fused.py:248-262), which this
implements.  Layouts as the reference: q (num_q_heads, head_dim), k_cache
(num_kv_heads, head_dim, seq_k) (D-major), v_cache (num_kv_heads, seq_k,
head_dim); mask (128, seq_k) whose row 0 is 0 on attended positions and -inf
elsewhere (a valid prefix); identity is ignored.  Returns (num_q_heads,
head_dim) in q's dtype (bf16 or fp32).
"""
from __future__ import annotations

import math

import torch

from q3vl import ops


def _valid_length(mask: torch.Tensor, seq_k: int) -> int:
    if mask is None:
        return seq_k
    row = mask[0].float()
    ok = ~torch.isinf(row)
    n = int(ok.sum().item())
    if n == 0 or not bool(ok[:n].all()):
        raise ValueError("mask row 0 must attend to a non-empty prefix")
    return n


def decode_attention_simple(q, k_cache, v_cache, mask=None, identity=None, softmax_scale=None,
                            num_q_heads=4, num_kv_heads=1, head_dim=128):
    Hq, D = q.shape
    seq_k = k_cache.shape[2]
    if Hq != num_q_heads or k_cache.shape[0] != num_kv_heads or D != head_dim:
        raise ValueError("decode_attention_simple: shapes do not match the head counts")
    L = _valid_length(mask, seq_k)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    kc = k_cache.transpose(1, 2).contiguous()[None]     # [1, Hkv, seq_k, D]
    vc = v_cache.contiguous()[None]
    return ops.attn_decode(q.contiguous()[None], kc, vc, kv_len=L, scale=scale)[0]
