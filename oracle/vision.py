"""Restated Qwen3-VL vision tower (CPU, PyTorch): the checker for the vision path.

Test infrastructure, like the rest of oracle/: only tests/ and the fixture
generator use it.  The reference runs transformers' Qwen3VLVisionModel
eagerly (vision.py:51-53, :74-76); this restates transformers 5.5.0
modeling_qwen3_vl.py, citing the lines each step follows:

  patch embed       Qwen3VLVisionPatchEmbed :72-89 (Conv3d with stride =
                    kernel, i.e. one GEMM over flattened (C, T, P, P) patches)
  position embed    fast_pos_embed_interpolate :702-763 (bilinear on the
                    sqrt(num_position_embeddings)^2 learned grid, then the
                    merge-block token order)
  rotary            rot_pos_emb :662-700 + Qwen3VLVisionRotaryEmbedding :92-105
                    (row and column angles, head_dim/4 frequencies each)
  blocks            Qwen3VLVisionBlock :265-296, Qwen3VLVisionAttention :182-262
                    (packed qkv, rotary in fp32 :131-142, non-causal attention
                    within each frame, eager softmax in fp32), Qwen3VLVisionMLP
                    :59-69 (gelu tanh)
  mergers           Qwen3VLVisionPatchMerger :108-121 (2x2 merge of consecutive
                    tokens; LayerNorm before the merge for the final merger,
                    after it for the deepstack mergers; exact-erf GELU)
  forward           Qwen3VLVisionModel.forward :765-823

Weights are a dict of tensors named as in the HF module's state_dict.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def patch_embed(x, w, b, dtype):
    """x [N, C*T*P*P] -> [N, hidden]; Conv3d weight [hidden, C, T, P, P].
    Stride equals the kernel, so this is the GEMM x @ w.view(hidden, -1).T + b;
    it is written as the convolution so that the CPU accumulation order, and
    with it every bf16 rounding, is the reference's."""
    hidden, C, T, P = w.shape[0], w.shape[1], w.shape[2], w.shape[3]
    y = F.conv3d(x.to(dtype).view(-1, C, T, P, P), w.to(dtype), b.to(dtype), stride=(T, P, P))
    return y.view(-1, hidden)


def pos_embed_interpolate(table, grid_thw, merge):
    """Bilinear position embeddings in merge-block token order.  table
    [side*side, hidden] (the learned grid); returns [N, hidden] in table dtype."""
    side = int(math.isqrt(table.shape[0]))
    out = []
    for t, h, w in grid_thw.tolist():
        hi = torch.linspace(0, side - 1, h)
        wi = torch.linspace(0, side - 1, w)
        h0, w0 = hi.int(), wi.int()
        h1 = (h0 + 1).clip(max=side - 1)
        w1 = (w0 + 1).clip(max=side - 1)
        dh, dw = (hi - h0)[:, None], (wi - w0)[None, :]
        # four corners; weights built in fp32 then cast to the table dtype,
        # products and the 4-term sum in that dtype (left to right)
        corners = ((h0, w0, (1 - dh) * (1 - dw)), (h0, w1, (1 - dh) * dw),
                   (h1, w0, dh * (1 - dw)), (h1, w1, dh * dw))
        acc = None
        for hh, ww, wt in corners:
            idx = (hh[:, None] * side + ww[None, :]).reshape(-1).long()
            term = table[idx] * wt.reshape(-1, 1).to(table.dtype)
            acc = term if acc is None else acc + term
        acc = acc.repeat(t, 1).view(t, h // merge, merge, w // merge, merge, -1)
        out.append(acc.permute(0, 1, 3, 2, 4, 5).reshape(-1, table.shape[1]))
    return torch.cat(out)


def rotary_cos_sin(grid_thw, head_dim, merge, theta=10000.0):
    """(cos, sin) fp32 [N, head_dim]: token (row r, col c) takes angles
    r*inv_freq then c*inv_freq (head_dim/4 each), the pair repeated twice."""
    dim = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
    rows, cols = [], []
    for t, h, w in grid_thw.tolist():
        bh, bw = h // merge, w // merge
        r = (torch.arange(bh)[:, None, None, None] * merge
             + torch.arange(merge)[None, None, :, None]).expand(bh, bw, merge, merge)
        c = (torch.arange(bw)[None, :, None, None] * merge
             + torch.arange(merge)[None, None, None, :]).expand(bh, bw, merge, merge)
        rows.append(r.reshape(-1).repeat(t))
        cols.append(c.reshape(-1).repeat(t))
    r = torch.cat(rows).float()
    c = torch.cat(cols).float()
    ang = torch.cat([torch.outer(r, inv), torch.outer(c, inv)], dim=-1)
    emb = torch.cat([ang, ang], dim=-1)
    return emb.cos(), emb.sin()


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def frame_bounds(grid_thw):
    """Token offsets of every frame (attention never crosses them)."""
    sizes = []
    for t, h, w in grid_thw.tolist():
        sizes += [h * w] * t
    cu = [0]
    for s in sizes:
        cu.append(cu[-1] + s)
    return cu


def attention(x, wq, bq, wo, bo, cos, sin, heads, cu):
    """Qwen3VLVisionAttention.forward, eager path (per-frame chunks)."""
    n, dim = x.shape
    hd = dim // heads
    qkv = F.linear(x, wq, bq).reshape(n, 3, heads, hd).permute(1, 0, 2, 3)
    q, k, v = qkv[0], qkv[1], qkv[2]
    dt = q.dtype
    c, s = cos[:, None, :].float(), sin[:, None, :].float()
    q = (q.float() * c + _rotate_half(q.float()) * s).to(dt)
    k = (k.float() * c + _rotate_half(k.float()) * s).to(dt)
    outs = []
    scale = hd ** -0.5
    for a, b in zip(cu[:-1], cu[1:]):
        qh, kh, vh = (t[a:b].transpose(0, 1) for t in (q, k, v))      # [heads, L, hd]
        sc = torch.matmul(qh, kh.transpose(1, 2)) * scale
        p = torch.softmax(sc, dim=-1, dtype=torch.float32).to(dt)
        outs.append(torch.matmul(p, vh).transpose(0, 1))               # [L, heads, hd]
    o = torch.cat(outs).reshape(n, dim)
    return F.linear(o, wo, bo)


def layer_norm(x, w, b, eps=1e-6):
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


def block(x, p, pre, heads, cos, sin, cu, dtype):
    g = lambda n: p[pre + n].to(dtype)  # noqa: E731
    h = layer_norm(x, g("norm1.weight"), g("norm1.bias"))
    x = x + attention(h, g("attn.qkv.weight"), g("attn.qkv.bias"), g("attn.proj.weight"),
                      g("attn.proj.bias"), cos, sin, heads, cu)
    h = layer_norm(x, g("norm2.weight"), g("norm2.bias"))
    h = F.linear(h, g("mlp.linear_fc1.weight"), g("mlp.linear_fc1.bias"))
    h = F.gelu(h, approximate="tanh")
    return x + F.linear(h, g("mlp.linear_fc2.weight"), g("mlp.linear_fc2.bias"))


def merger(x, p, pre, merge, postshuffle, dtype):
    g = lambda n: p[pre + n].to(dtype)  # noqa: E731
    width = x.shape[-1] * merge * merge
    if postshuffle:
        x = layer_norm(x.reshape(-1, width), g("norm.weight"), g("norm.bias"))
    else:
        x = layer_norm(x, g("norm.weight"), g("norm.bias")).reshape(-1, width)
    x = F.gelu(F.linear(x, g("linear_fc1.weight"), g("linear_fc1.bias")))
    return F.linear(x, g("linear_fc2.weight"), g("linear_fc2.bias"))


def vision_forward(pixels, grid_thw, p, *, depth, heads, merge=2, deepstack=(8, 16, 24),
                   dtype=torch.bfloat16):
    """-> (pooler_output [N/merge^2, out], [deepstack features], last_hidden [N, hidden])."""
    x = patch_embed(pixels, p["patch_embed.proj.weight"], p["patch_embed.proj.bias"], dtype)
    x = x + pos_embed_interpolate(p["pos_embed.weight"].to(dtype), grid_thw, merge)
    head_dim = x.shape[1] // heads
    cos, sin = rotary_cos_sin(grid_thw, head_dim, merge)
    cu = frame_bounds(grid_thw)
    feats = []
    for i in range(depth):
        x = block(x, p, f"blocks.{i}.", heads, cos, sin, cu, dtype)
        if i in deepstack:
            j = list(deepstack).index(i)
            feats.append(merger(x, p, f"deepstack_merger_list.{j}.", merge, True, dtype))
    return merger(x, p, "merger.", merge, False, dtype), feats, x
