"""Restated reference math for the decoder hot path (CPU, PyTorch).

Test infrastructure (see oracle/__init__.py): the checker for the CUDA path.
Each function cites the reference file:line it restates.  bf16 rounding
points follow the reference: every torch op on bf16 tensors rounds its result.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

HEAD_DIM = 128


# ---------------------------------------------------------------------------
# a1: RMSNorm -- model_fused.py:37-40 (model.py:44-47)
# ---------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv).to(x.dtype) * w


# ---------------------------------------------------------------------------
# a2: 1-D rotary tables -- RotaryEmbedding, model_fused.py:43-58
# ---------------------------------------------------------------------------
def inv_freq(head_dim: int = HEAD_DIM, base: float = 5e6) -> torch.Tensor:
    return 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))


def rotary_tables(head_dim: int, max_seq_len: int, base: float):
    """bf16 cos/sin [max_seq_len, head_dim/2] (model_fused.py:45-50)."""
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq(head_dim, base))
    return freqs.cos().to(torch.bfloat16), freqs.sin().to(torch.bfloat16)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat((-x2, x1), dim=-1)


# ---------------------------------------------------------------------------
# a9: rope_ref -- test_kernels.py:126-134 (oracle of kernels/rope.py:24-96)
# ---------------------------------------------------------------------------
def rope_fp32(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [S, N, D] bf16; cos/sin [S, D/2] f32 -> fp32 math, bf16 result."""
    cf = torch.cat([cos, cos], dim=-1).unsqueeze(1)
    sf = torch.cat([sin, sin], dim=-1).unsqueeze(1)
    xf = x.float()
    return (xf * cf + rotate_half(xf) * sf).to(torch.bfloat16)


# ---------------------------------------------------------------------------
# a4: interleaved M-RoPE -- transformers 5.5.0 modeling_qwen3_vl.py:352-386
# (Qwen3VLTextRotaryEmbedding.forward, apply_interleaved_mrope) and
# apply_rotary_pos_emb :410-432.
# ---------------------------------------------------------------------------
def mrope_freqs(position_ids: torch.Tensor, inv_f: torch.Tensor, section=(24, 20, 20)):
    """position_ids [3, B, S] int -> fp32 angles [B, S, D/2] after interleaving."""
    pos = position_ids.float()                              # (3, B, S)
    freqs = pos[..., None] * inv_f[None, None, None, :]     # (3, B, S, D/2)
    out = freqs[0].clone()
    for axis, offset in ((1, 1), (2, 2)):
        idx = slice(offset, section[axis] * 3, 3)
        out[..., idx] = freqs[axis][..., idx]
    return out


def mrope_cos_sin(position_ids, inv_f, section=(24, 20, 20), dtype=torch.bfloat16):
    """cos/sin [B, S, D] cast to the activation dtype, as HF returns them."""
    f = mrope_freqs(position_ids, inv_f, section)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope_bf16(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, H, S, D]; cos/sin broadcastable [B, 1, S, D] (HF apply_rotary_pos_emb)."""
    return x * cos + rotate_half(x) * sin


def config2_position_ids(seq: int = 2048, text0: int = 100, grid: int = 16) -> torch.Tensor:
    """3-axis positions of the prefill workload: tokens 0..text0-1 text
    (t=h=w=index), then a grid x grid image at t=text0, h=text0+row,
    w=text0+col, then text continuing from text0 + grid (the convention of
    get_vision_position_ids / get_rope_index, modeling_qwen3_vl.py:975-1122)."""
    n_img = grid * grid
    full = max(seq, text0 + n_img)
    pos = torch.zeros(3, full, dtype=torch.int64)
    t = torch.arange(text0)
    pos[:, :text0] = t
    r = torch.arange(n_img) // grid
    c = torch.arange(n_img) % grid
    pos[0, text0:text0 + n_img] = text0
    pos[1, text0:text0 + n_img] = text0 + r
    pos[2, text0:text0 + n_img] = text0 + c
    rest = full - text0 - n_img
    if rest > 0:
        pos[:, text0 + n_img:] = text0 + grid + torch.arange(rest)
    return pos[:, None, :seq]   # [3, 1, S]


def rope_index(types, mask, image_thw, video_thw, merge: int = 2):
    """3-axis position ids and per-sequence rope deltas, restating
    transformers 5.5.0 modeling_qwen3_vl.py:1031-1122 (Qwen3VLModel.get_rope_index)
    with get_vision_position_ids :975-1029 (temp_merge_size 1, time_interval 1).

    types [B, S] int (0 text, 1 image, 2 video); mask [B, S] or None (nonzero =
    kept); image_thw [Ni, 3] / video_thw [Nv, 3] ints or None.  Returns
    (pos int64 [3, B, S], delta int64 [B]).  Steps:
      - each video is split into t frames of grid (1, h, w) (:1071-1073);
      - the kept tokens of a sequence are cut into runs of one type (:1096-1101);
      - a text run takes consecutive positions on all three axes from the
        running position and advances it by its length (:1106-1110);
      - an image / frame run takes the next grid of its kind (grids are
        consumed in batch order, :1082-1085) and token i of the run gets
        t = p, h = p + i // (w' t), w = p + i % w' with h' = h // merge,
        w' = w // merge (:1013-1024); p advances by max(h, w) // merge (:1118);
      - masked tokens keep position 0; delta = max position + 1 - kept tokens.
    A run whose length differs from its grid's token count, or a run with no
    grid left, raises ValueError (the reference fails on both)."""
    import numpy as np
    types = np.asarray(types, dtype=np.int64)
    B, S = types.shape
    keep = np.ones((B, S), dtype=bool) if mask is None else (np.asarray(mask) != 0)
    grids = {1: [], 2: []}
    if image_thw is not None:
        grids[1] = [tuple(int(v) for v in g) for g in np.asarray(image_thw).reshape(-1, 3)]
    if video_thw is not None:
        for t, h, w in np.asarray(video_thw).reshape(-1, 3):
            grids[2] += [(1, int(h), int(w))] * int(t)
    nxt = {1: 0, 2: 0}
    pos = np.zeros((3, B, S), dtype=np.int64)
    delta = np.zeros(B, dtype=np.int64)
    for b in range(B):
        idx = np.nonzero(keep[b])[0]
        tt = types[b, idx]
        if len(idx) == 0:
            raise ValueError("rope_index: a sequence with no kept token")
        if ((tt < 0) | (tt > 2)).any():
            raise ValueError("rope_index: token type outside {0, 1, 2}")
        out = np.zeros((3, len(idx)), dtype=np.int64)
        p, j = 0, 0
        while j < len(idx):
            e = j
            while e < len(idx) and tt[e] == tt[j]:
                e += 1
            n = e - j
            kind = int(tt[j])
            if kind == 0:
                out[:, j:e] = p + np.arange(n)
                p += n
            else:
                if nxt[kind] >= len(grids[kind]):
                    raise ValueError("rope_index: more vision runs than grids")
                gt, gh, gw = grids[kind][nxt[kind]]
                nxt[kind] += 1
                hh, ww = gh // merge, gw // merge
                if n != gt * hh * ww:
                    raise ValueError("rope_index: vision run length differs from its grid")
                i = np.arange(n)
                out[0, j:e] = p
                out[1, j:e] = p + i // (ww * gt)
                out[2, j:e] = p + i % ww
                p += max(gh, gw) // merge
            j = e
        pos[:, b, idx] = out
        delta[b] = out.max() + 1 - len(idx)
    return torch.from_numpy(pos), torch.from_numpy(delta)


# ---------------------------------------------------------------------------
# a3: AttentionBlock.forward -- model_fused.py:87-131
# ---------------------------------------------------------------------------
def attention_block(hidden, qkv_w, qkv_b, in_norm_w, q_norm_w, k_norm_w, cos, sin, Hq, Hkv,
                    eps=1e-6):
    """qkv_w [H, (Hq+2Hkv)*D] ([in, out]); cos/sin [S, D/2] (1-D) or [B, 1, S, D]
    (already expanded M-RoPE).  Returns q [B,Hq,S,D], k/v [B,Hkv,S,D]."""
    B, S, _ = hidden.shape
    D = HEAD_DIM
    h = rmsnorm(hidden, in_norm_w, eps)
    qkv = h @ qkv_w
    if qkv_b is not None:
        qkv = qkv + qkv_b
    qd, kd = Hq * D, Hkv * D
    q = qkv[..., :qd].view(B, S, Hq, D).transpose(1, 2)
    k = qkv[..., qd:qd + kd].view(B, S, Hkv, D).transpose(1, 2)
    v = qkv[..., qd + kd:].view(B, S, Hkv, D).transpose(1, 2)
    q = rmsnorm(q, q_norm_w, eps)
    k = rmsnorm(k, k_norm_w, eps)
    if cos.dim() == 2:
        cf = torch.cat([cos, cos], dim=-1)[None, None]
        sf = torch.cat([sin, sin], dim=-1)[None, None]
    else:
        cf, sf = cos, sin
    q = q * cf + rotate_half(q) * sf
    k = k * cf + rotate_half(k) * sf
    return q, k, v


# ---------------------------------------------------------------------------
# a6: eager GQA attention over the static cache -- model_fused.py:248-262
# (causal mask model_fused.py:219-222)
# ---------------------------------------------------------------------------
def eager_attention(q, k_cache, v_cache, start_pos: int):
    """q [B,Hq,S,D]; caches [B,Hkv,maxS,D]; returns [B,Hq,S,D] in q.dtype."""
    B, Hq, S, D = q.shape
    Hkv, maxS = k_cache.shape[1], k_cache.shape[2]
    rep = Hq // Hkv
    kf = k_cache.unsqueeze(2).expand(-1, -1, rep, -1, -1).reshape(B, Hq, maxS, D)
    vf = v_cache.unsqueeze(2).expand(-1, -1, rep, -1, -1).reshape(B, Hq, maxS, D)
    scale = 1.0 / math.sqrt(D)
    w = torch.matmul(q, kf.transpose(-2, -1)) * scale
    mask = torch.triu(torch.full((maxS, maxS), float("-inf"), dtype=torch.bfloat16), diagonal=1)
    w = w + mask[start_pos:start_pos + S, :maxS][None, None]
    w = F.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(w, vf)


def decode_attention_fp32(q, k, v, scale=None):
    """Config-1 oracle: fp32 softmax(q k^T * scale) v with GQA grouping
    h -> h // (Hq/Hkv) (the eager path at S=1 in fp32).  q [B,Hq,D],
    k/v [B,Hkv,L,D]."""
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    rep = Hq // Hkv
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    kf = k.repeat_interleave(rep, dim=1).double()
    vf = v.repeat_interleave(rep, dim=1).double()
    s = torch.einsum("bhd,bhld->bhl", q.double(), kf) * scale
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhl,bhld->bhd", p, vf).to(q.dtype)


# ---------------------------------------------------------------------------
# a7: attention_ref -- test_kernels.py:184-214 (oracle of
# kernels/prefill_attention.py:28-149); layouts q [Hq,D,S], k [Hkv,D,S], v [Hkv,S,D]
# ---------------------------------------------------------------------------
def prefill_attention_nki_layout(q, k, v, scale):
    Hq, D, S = q.shape
    rep = Hq // k.shape[0]
    out = torch.zeros(Hq, S, D, dtype=torch.bfloat16)
    mask = torch.triu(torch.full((S, S), float("-inf")), diagonal=1)
    for h in range(Hq):
        g = h // rep
        qt, kt, vt = q[h].T.float(), k[g].T.float(), v[g].float()
        a = torch.softmax(qt @ kt.T * scale + mask, dim=-1)
        out[h] = (a @ vt).to(torch.bfloat16)
    return out


def causal_attention_fp32(q, k, v, start_pos=0, scale=None):
    """fp32 causal GQA attention, q [B,Hq,S,D], k/v [B,Hkv,start+S,D]."""
    B, Hq, S, D = q.shape
    rep = Hq // k.shape[1]
    L = start_pos + S
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    kf = k[:, :, :L].float().repeat_interleave(rep, dim=1)
    vf = v[:, :, :L].float().repeat_interleave(rep, dim=1)
    s = torch.matmul(q.float(), kf.transpose(-2, -1)) * scale
    qi = torch.arange(S)[:, None] + start_pos
    kj = torch.arange(L)[None, :]
    s = s.masked_fill(kj > qi, float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), vf)


# ---------------------------------------------------------------------------
# a11: MLPBlock.forward -- model_fused.py:157-172 (returns the partial sum)
# ---------------------------------------------------------------------------
def mlp_block(hidden, gate_up_w, down_w, post_norm_w, eps=1e-6):
    h = rmsnorm(hidden, post_norm_w, eps)
    gu = h @ gate_up_w
    gate, up = gu.chunk(2, dim=-1)
    return (F.silu(gate) * up) @ down_w
