"""Torch-facing wrappers around the q3vl C ABI.

Every wrapper validates device, dtype, shape and contiguity, then launches on
torch's current CUDA stream.  Tensors must already live on a CUDA device: the
path has no CPU fallback and raises instead.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import _lib
from ._lib import (Q3_BF16, Q3_EPI_NONE, Q3_EPI_RESIDUAL, Q3_EPI_SWIGLU, Q3_F32, call)

HEAD_DIM = 128
_EPI = {"none": Q3_EPI_NONE, "residual": Q3_EPI_RESIDUAL, "swiglu": Q3_EPI_SWIGLU}


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(name: str, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name}: tensors must be on a CUDA device (no CPU fallback); "
                               f"got {t.device}")


def _bf16(name: str, *ts):
    for t in ts:
        if t is not None and t.dtype != torch.bfloat16:
            raise TypeError(f"{name}: expected bfloat16, got {t.dtype}")


def _contig(name: str, *ts):
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError(f"{name}: tensors must be contiguous")


# ----------------------------------------------------------------------------
# a1: RMSNorm (+ fused residual add)
# ----------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, add: torch.Tensor = None,
            h_out: torch.Tensor = None, out: torch.Tensor = None) -> torch.Tensor:
    """y = bf16(bf16(h*rsqrt(mean(h^2)+eps))*w) with h = x (+ add, written to h_out)."""
    _cuda("rmsnorm", x, weight, add, h_out, out)
    _bf16("rmsnorm", x, weight, add, h_out, out)
    _contig("rmsnorm", x, weight, add, h_out, out)
    hidden = x.shape[-1]
    if weight.numel() != hidden:
        raise ValueError(f"rmsnorm: weight has {weight.numel()} elements, hidden is {hidden}")
    if add is not None and add.shape != x.shape:
        raise ValueError("rmsnorm: add must match x")
    y = torch.empty_like(x) if out is None else out
    call("q3_rmsnorm", _p(x), _p(add), _p(h_out), _p(weight), _p(y), x.numel() // hidden,
         hidden, float(eps), _stream())
    return y


# ----------------------------------------------------------------------------
# a9 / a4: RoPE and M-RoPE tables
# ----------------------------------------------------------------------------
def rope(x: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """x bf16 [S, N, 128], cos_sin f32 [S, 128] -> rotate_half RoPE (bf16)."""
    _cuda("rope", x, cos_sin)
    _bf16("rope", x)
    _contig("rope", x, cos_sin)
    if cos_sin.dtype != torch.float32:
        raise TypeError("rope: cos_sin must be float32")
    S, N, D = x.shape
    if cos_sin.shape != (S, D):
        raise ValueError(f"rope: cos_sin shape {tuple(cos_sin.shape)} != {(S, D)}")
    out = torch.empty_like(x)
    call("q3_rope", _p(x), _p(cos_sin), _p(out), S, N, D, _stream())
    return out


def mrope_cos_sin(position_ids: torch.Tensor, inv_freq: torch.Tensor,
                  mrope_section=(24, 20, 20)):
    """position_ids int64 [3, n] -> (cos, sin) f32 [n, D/2] (interleaved M-RoPE)."""
    _cuda("mrope_cos_sin", position_ids, inv_freq)
    if position_ids.dtype != torch.int64 or inv_freq.dtype != torch.float32:
        raise TypeError("mrope_cos_sin: position_ids int64, inv_freq float32")
    pos = position_ids.reshape(3, -1).contiguous()
    n = pos.shape[1]
    half = inv_freq.numel()
    cos = torch.empty(n, half, dtype=torch.float32, device=pos.device)
    sin = torch.empty_like(cos)
    call("q3_mrope_cos_sin", _p(pos), _p(inv_freq.contiguous()), n, 2 * half,
         int(mrope_section[1]), int(mrope_section[2]), _p(cos), _p(sin), _stream())
    return cos, sin


# ----------------------------------------------------------------------------
# vision tower: linears with bias epilogues, LayerNorm, position embeddings,
# 2-D RoPE, frame-local attention
# ----------------------------------------------------------------------------
_EPI_BIAS = {"bias": _lib.Q3_EPI_BIAS, "bias_gelu_tanh": _lib.Q3_EPI_BIAS_GELU_TANH,
             "bias_gelu": _lib.Q3_EPI_BIAS_GELU, "bias_residual": _lib.Q3_EPI_BIAS_RESIDUAL}


def gemm_bias(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, epilogue: str = "bias",
              residual: torch.Tensor = None, out: torch.Tensor = None) -> torch.Tensor:
    """nn.Linear with bias (w [N, K], the module's own layout) and a fused
    epilogue: "bias", "bias_gelu_tanh", "bias_gelu" (erf) or "bias_residual"
    (out = residual + linear; `out` may be `residual` itself)."""
    _cuda("gemm_bias", a, w, bias, residual, out)
    _bf16("gemm_bias", a, w, bias)
    _contig("gemm_bias", a, w, bias)
    if epilogue not in _EPI_BIAS:
        raise ValueError(f"gemm_bias: unknown epilogue {epilogue!r}")
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K or bias.numel() != N:
        raise ValueError(f"gemm_bias: shapes a {tuple(a.shape)} w {tuple(w.shape)} "
                         f"bias {tuple(bias.shape)}")
    if epilogue == "bias_residual":
        if residual is None or tuple(residual.shape) != (M, N) or not residual.is_contiguous():
            raise ValueError("gemm_bias: bias_residual needs a contiguous [M, N] residual")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    call("q3_gemm_bias", _p(a), _p(w), _p(bias), _p(out), M, N, K, _EPI_BIAS[epilogue],
         _p(residual), _stream())
    return out


def layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-6,
              out: torch.Tensor = None) -> torch.Tensor:
    """nn.LayerNorm over the last dim (bf16 in and out, fp32 statistics)."""
    _cuda("layernorm", x, w, b, out)
    _bf16("layernorm", x, w, b)
    _contig("layernorm", x, w, b)
    cols = x.shape[-1]
    out = torch.empty_like(x) if out is None else out
    call("q3_layernorm", _p(x), _p(w), _p(b), _p(out), x.numel() // cols, cols, float(eps),
         _stream())
    return out


def vision_pos_embed(table: torch.Tensor, imgs: torch.Tensor, imgs_host: torch.Tensor,
                     merge: int, n_tok: int) -> torch.Tensor:
    """Bilinear position embeddings [n_tok, hidden] in merge-block token order;
    imgs int32 [n_img, 4] = (t, h, w, first token) on the device, imgs_host the
    same on the host."""
    _cuda("vision_pos_embed", table, imgs)
    side = int(round(table.shape[0] ** 0.5))
    out = torch.empty(n_tok, table.shape[1], dtype=torch.bfloat16, device=table.device)
    call("q3_vision_pos_embed", _p(table), side, table.shape[1], _p(imgs), _p(imgs_host),
         imgs.shape[0], int(merge), int(n_tok), _p(out), _stream())
    return out


def vision_rope(qkv: torch.Tensor, heads: int, inv_freq: torch.Tensor, imgs: torch.Tensor,
                imgs_host: torch.Tensor, merge: int) -> torch.Tensor:
    """2-D RoPE in place on q and k of the packed qkv [n_tok, 3 * heads * 72]."""
    _cuda("vision_rope", qkv, inv_freq, imgs)
    _contig("vision_rope", qkv)
    call("q3_vision_rope", _p(qkv), int(heads), qkv.shape[1] // (3 * heads), _p(inv_freq),
         _p(imgs), _p(imgs_host), imgs.shape[0], int(merge), qkv.shape[0], _stream())
    return qkv


def vision_attention(qkv: torch.Tensor, heads: int, blocks: torch.Tensor,
                     blocks_host: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """Attention inside each frame: qkv [n_tok, 3 * heads * 72] -> [n_tok, heads * 72];
    blocks int32 [n_blocks, 3] = (frame first token, frame length, first query row)."""
    _cuda("vision_attention", qkv, blocks, out)
    _contig("vision_attention", qkv)
    n_tok, width = qkv.shape
    hd = width // (3 * heads)
    if out is None:
        out = torch.empty(n_tok, heads * hd, dtype=torch.bfloat16, device=qkv.device)
    call("q3_vision_attention", _p(qkv), _p(out), int(heads), hd, _p(blocks), _p(blocks_host),
         blocks.shape[0], n_tok, _stream())
    return out


_ROPE_INDEX_ERRORS = {
    1: "more vision runs than grids",
    2: "vision run length differs from its grid",
    3: "token type outside {0, 1, 2}",
    4: "a sequence with no kept token",
}


def rope_index(mm_token_type_ids: torch.Tensor, image_grid_thw: torch.Tensor = None,
               video_grid_thw: torch.Tensor = None, attention_mask: torch.Tensor = None, *,
               spatial_merge_size: int = 2):
    """3-axis position ids [3, B, S] int64 and rope deltas [B, 1] int64 on the
    device (Qwen3VLModel.get_rope_index, transformers 5.5.0
    modeling_qwen3_vl.py:1031-1122).  Synchronizes once to read the
    per-sequence status, and raises ValueError where the reference fails."""
    _cuda("rope_index", mm_token_type_ids)
    dev = mm_token_type_ids.device
    if mm_token_type_ids.dim() != 2:
        raise ValueError("rope_index: mm_token_type_ids must be [B, S]")
    B, S = mm_token_type_ids.shape
    types = mm_token_type_ids.to(dev, torch.int32).contiguous()
    mask = None
    if attention_mask is not None:
        if tuple(attention_mask.shape) != (B, S):
            raise ValueError("rope_index: attention_mask must match mm_token_type_ids")
        mask = (attention_mask.to(dev) != 0).to(torch.int32).contiguous()

    def grids(g):
        if g is None or g.numel() == 0:
            return None, 0
        g = g.to(dev, torch.int64).reshape(-1, 3).contiguous()
        return g, g.shape[0]
    img, n_img = grids(image_grid_thw)
    vid, n_vid = grids(video_grid_thw)
    pos = torch.empty(3, B, S, dtype=torch.int64, device=dev)
    delta = torch.empty(B, dtype=torch.int64, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    nbytes = _lib.raw("q3_rope_index_workspace_bytes")(B)
    ws = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=dev)
    call("q3_rope_index", _p(types), _p(mask), B, S, _p(img), n_img, _p(vid), n_vid,
         int(spatial_merge_size), _p(pos), _p(delta), _p(status), _p(ws), nbytes, _stream())
    bad = status.cpu()
    if bool((bad != 0).any()):
        b = int((bad != 0).nonzero()[0, 0])
        raise ValueError(f"rope_index: sequence {b}: "
                         f"{_ROPE_INDEX_ERRORS.get(int(bad[b]), int(bad[b]))}")
    return pos, delta.view(B, 1)


# ----------------------------------------------------------------------------
# a3 epilogue + a5: QK-norm, RoPE, KV write
# ----------------------------------------------------------------------------
def qkv_norm_rope(qkv: torch.Tensor, q_norm_w, k_norm_w, cos, sin, *, B: int, S: int, Hq: int,
                  Hkv: int, start_pos: int = 0, pos_dev: torch.Tensor = None,
                  cs_use_pos: bool = True, cs_offset: int = 0, cs_stride_b: int = 0,
                  k_cache=None, v_cache=None, want_q: bool = True, want_kv: bool = False,
                  eps: float = 1e-6):
    """Per-head QK-RMSNorm + RoPE on a fused qkv [B*S, (Hq+2Hkv)*128]; writes the
    rotated k and v into the caches at the cache position (start_pos or
    *pos_dev).  RoPE row of token (b, s) = cs_use_pos*pos + cs_offset +
    b*cs_stride_b + s."""
    _cuda("qkv_norm_rope", qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, pos_dev)
    _bf16("qkv_norm_rope", qkv, q_norm_w, k_norm_w, k_cache, v_cache)
    _contig("qkv_norm_rope", qkv, cos, sin, k_cache, v_cache)
    if qkv.numel() != B * S * (Hq + 2 * Hkv) * HEAD_DIM:
        raise ValueError("qkv_norm_rope: qkv size does not match B,S,Hq,Hkv")
    if cos.dtype == torch.bfloat16:
        cs_dtype = Q3_BF16
    elif cos.dtype == torch.float32:
        cs_dtype = Q3_F32
    else:
        raise TypeError("qkv_norm_rope: cos/sin must be bf16 or f32")
    dev = qkv.device
    q = torch.empty(B, Hq, S, HEAD_DIM, dtype=torch.bfloat16, device=dev) if want_q else None
    k = v = None
    if want_kv:
        k = torch.empty(B, Hkv, S, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        v = torch.empty_like(k)
    max_seq = k_cache.shape[2] if k_cache is not None else 0
    if pos_dev is not None and pos_dev.dtype != torch.int32:
        raise TypeError("qkv_norm_rope: pos_dev must be int32")
    call("q3_qkv_norm_rope", _p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin), cs_dtype,
         1 if cs_use_pos else 0, int(cs_offset), int(cs_stride_b), _p(q), _p(k), _p(v),
         _p(k_cache),
         _p(v_cache), B, S, Hq, Hkv, HEAD_DIM, int(start_pos), _p(pos_dev), int(max_seq),
         float(eps), _stream())
    return q, k, v


def qkv_norm_rope_paged(qkv: torch.Tensor, q_norm_w, k_norm_w, cos, sin, *, B: int, S: int,
                        Hq: int, Hkv: int, k_pages: torch.Tensor, v_pages: torch.Tensor,
                        block_table: torch.Tensor, start_pos: int = 0,
                        pos_dev: torch.Tensor = None, cs_use_pos: bool = True,
                        cs_offset: int = 0, cs_stride_b: int = 0, eps: float = 1e-6):
    """qkv_norm_rope with the rotated k and v written into page pools through
    block_table; returns q [B, Hq, S, 128]."""
    _cuda("qkv_norm_rope_paged", qkv, q_norm_w, k_norm_w, cos, sin, k_pages, v_pages,
          block_table, pos_dev)
    _bf16("qkv_norm_rope_paged", qkv, q_norm_w, k_norm_w, k_pages, v_pages)
    _contig("qkv_norm_rope_paged", qkv, cos, sin, k_pages, v_pages, block_table)
    if qkv.numel() != B * S * (Hq + 2 * Hkv) * HEAD_DIM:
        raise ValueError("qkv_norm_rope_paged: qkv size does not match B,S,Hq,Hkv")
    cs_dtype = {torch.bfloat16: Q3_BF16, torch.float32: Q3_F32}.get(cos.dtype)
    if cs_dtype is None:
        raise TypeError("qkv_norm_rope_paged: cos/sin must be bf16 or f32")
    if block_table.dtype != torch.int32 or (pos_dev is not None and pos_dev.dtype != torch.int32):
        raise TypeError("qkv_norm_rope_paged: block_table and pos_dev must be int32")
    num_pages, _, page_tokens, _ = k_pages.shape
    q = torch.empty(B, Hq, S, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device)
    call("q3_qkv_norm_rope_paged", _p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin),
         cs_dtype, 1 if cs_use_pos else 0, int(cs_offset), int(cs_stride_b), _p(q), _p(k_pages),
         _p(v_pages), B, S, Hq, Hkv, HEAD_DIM, int(start_pos), _p(pos_dev), _p(block_table),
         block_table.shape[1], page_tokens, num_pages, float(eps), _stream())
    return q


# ----------------------------------------------------------------------------
# a6/a8: decode attention
# ----------------------------------------------------------------------------
# Split-K workspaces, one per (device, shape); never freed, because captured
# decode graphs keep their addresses.
_ws_cache: dict = {}


def decode_workspace(B: int, Hq: int, Hkv: int, device) -> torch.Tensor | None:
    """Workspace large enough for any KV length (the split count saturates at
    about two CTAs per SM, so the size is bounded)."""
    nbytes = _lib.raw("q3_attn_decode_workspace_bytes")(B, Hq, Hkv, HEAD_DIM, 1 << 30)
    if nbytes == 0:
        return None
    key = (str(torch.device(device)), B, Hq, Hkv)
    ws = _ws_cache.get(key)
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("decode workspace must be allocated before graph capture")
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def attn_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: int,
                scale: float = None, kv_len_dev: torch.Tensor = None, out: torch.Tensor = None,
                workspace: torch.Tensor = None) -> torch.Tensor:
    """q [B, Hq, 128]; caches [B, Hkv, max_seq, 128]; attends to [0, kv_len).

    With kv_len_dev (int32 device scalar), kv_len is the upper bound used to
    size the split-K grid and the actual length is read on the device."""
    _cuda("attn_decode", q, k_cache, v_cache, kv_len_dev)
    _contig("attn_decode", q, k_cache, v_cache)
    if q.dtype == torch.float32:
        dt = Q3_F32
    elif q.dtype == torch.bfloat16:
        dt = Q3_BF16
    else:
        raise TypeError("attn_decode: q must be float32 or bfloat16")
    if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError("attn_decode: q, k_cache, v_cache must share a dtype")
    B, Hq, D = q.shape
    _, Hkv, max_seq, _ = k_cache.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q) if out is None else out
    ws = workspace if workspace is not None else decode_workspace(B, Hq, Hkv, q.device)
    call("q3_attn_decode", _p(q), _p(k_cache), _p(v_cache), _p(o), B, Hq, Hkv, D, int(kv_len),
         _p(kv_len_dev), max_seq, float(scale), dt, _p(ws), 0 if ws is None else ws.numel(),
         _stream())
    return o


def attn_decode_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                      block_table: torch.Tensor, kv_len: int, scale: float = None,
                      kv_len_dev: torch.Tensor = None, out: torch.Tensor = None) -> torch.Tensor:
    """attn_decode over paged K/V: q bf16 [B, Hq, 128]; k_pages / v_pages
    [num_pages, Hkv, page_tokens, 128]; block_table int32 [B, width] on the
    device (position t of row b in page block_table[b, t // page_tokens])."""
    _cuda("attn_decode_paged", q, k_pages, v_pages, block_table, kv_len_dev)
    _bf16("attn_decode_paged", q, k_pages, v_pages)
    _contig("attn_decode_paged", q, k_pages, v_pages, block_table)
    if block_table.dtype != torch.int32:
        raise TypeError("attn_decode_paged: block_table must be int32")
    B, Hq, D = q.shape
    num_pages, Hkv, page_tokens, _ = k_pages.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    o = torch.empty_like(q) if out is None else out
    ws = decode_workspace(B, Hq, Hkv, q.device)
    call("q3_attn_decode_paged", _p(q), _p(k_pages), _p(v_pages), _p(o), B, Hq, Hkv, D,
         int(kv_len), _p(kv_len_dev), _p(block_table), block_table.shape[1], page_tokens,
         num_pages, float(scale), _p(ws), 0 if ws is None else ws.numel(), _stream())
    return o


def kv_pages_write(k_rows: torch.Tensor, v_rows: torch.Tensor, k_pages: torch.Tensor,
                   v_pages: torch.Tensor, block_table: torch.Tensor, start_pos: int = 0,
                   pos_dev: torch.Tensor = None) -> None:
    """Copy new K/V rows bf16 [B, Hkv, S, 128] into their pages at positions
    start_pos (or *pos_dev) .. + S - 1 of each sequence."""
    _cuda("kv_pages_write", k_rows, v_rows, k_pages, v_pages, block_table, pos_dev)
    _bf16("kv_pages_write", k_rows, v_rows, k_pages, v_pages)
    _contig("kv_pages_write", k_rows, v_rows, k_pages, v_pages, block_table)
    B, Hkv, S, D = k_rows.shape
    num_pages, _, page_tokens, _ = k_pages.shape
    call("q3_kv_pages_write", _p(k_rows), _p(v_rows), _p(k_pages), _p(v_pages), B, Hkv, S, D,
         _p(block_table), block_table.shape[1], page_tokens, num_pages, int(start_pos),
         _p(pos_dev), _stream())


def attn_decode_qkv(qkv: torch.Tensor, q_norm_w, k_norm_w, cos, sin, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, *, Hq: int, Hkv: int, kv_len: int,
                    kv_len_dev: torch.Tensor = None, cs_offset: int = 0, scale: float = None,
                    eps: float = 1e-6, out: torch.Tensor = None) -> torch.Tensor:
    """Decode attention straight from the raw QKV projection: per-head
    QK-RMSNorm + RoPE of the new token, its K/V row written to the caches at
    kv_len-1, and GQA attention over [0, kv_len).  qkv bf16 [B, (Hq+2Hkv)*128];
    bf16 cos/sin tables; returns out [B, Hq, 128]."""
    _cuda("attn_decode_qkv", qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, kv_len_dev)
    _bf16("attn_decode_qkv", qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache)
    _contig("attn_decode_qkv", qkv, cos, sin, k_cache, v_cache)
    B = qkv.shape[0]
    if qkv.numel() != B * (Hq + 2 * Hkv) * HEAD_DIM:
        raise ValueError("attn_decode_qkv: qkv must be [B, (Hq+2Hkv)*128]")
    if kv_len_dev is not None and kv_len_dev.dtype != torch.int32:
        raise TypeError("attn_decode_qkv: kv_len_dev must be int32")
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else scale
    o = torch.empty(B, Hq, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device) if out is None \
        else out
    ws = decode_workspace(B, Hq, Hkv, qkv.device)
    call("q3_attn_decode_qkv", _p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin),
         int(cs_offset), _p(k_cache), _p(v_cache), _p(o), B, Hq, Hkv, HEAD_DIM, int(kv_len),
         _p(kv_len_dev), k_cache.shape[2], float(scale), float(eps), _p(ws),
         0 if ws is None else ws.numel(), _stream())
    return o


def attn_decode_qkv_paged(qkv: torch.Tensor, q_norm_w, k_norm_w, cos, sin,
                          k_pages: torch.Tensor, v_pages: torch.Tensor,
                          block_table: torch.Tensor, *, Hq: int, Hkv: int, kv_len: int,
                          kv_len_dev: torch.Tensor = None, cs_offset: int = 0,
                          scale: float = None, eps: float = 1e-6,
                          out: torch.Tensor = None) -> torch.Tensor:
    """attn_decode_qkv over a page pool (q3_attn_decode_qkv_paged): k_pages /
    v_pages bf16 [num_pages, Hkv, page_tokens, 128]; block_table int32 [B, width]
    on the device, already holding the page of position kv_len - 1."""
    _cuda("attn_decode_qkv_paged", qkv, q_norm_w, k_norm_w, cos, sin, k_pages, v_pages,
          block_table, kv_len_dev)
    _bf16("attn_decode_qkv_paged", qkv, q_norm_w, k_norm_w, cos, sin, k_pages, v_pages)
    _contig("attn_decode_qkv_paged", qkv, cos, sin, k_pages, v_pages, block_table)
    if block_table.dtype != torch.int32:
        raise TypeError("attn_decode_qkv_paged: block_table must be int32")
    B = qkv.shape[0]
    if qkv.numel() != B * (Hq + 2 * Hkv) * HEAD_DIM:
        raise ValueError("attn_decode_qkv_paged: qkv must be [B, (Hq+2Hkv)*128]")
    if kv_len_dev is not None and kv_len_dev.dtype != torch.int32:
        raise TypeError("attn_decode_qkv_paged: kv_len_dev must be int32")
    num_pages, _, page_tokens, _ = k_pages.shape
    scale = 1.0 / math.sqrt(HEAD_DIM) if scale is None else scale
    o = torch.empty(B, Hq, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device) if out is None \
        else out
    ws = decode_workspace(B, Hq, Hkv, qkv.device)
    call("q3_attn_decode_qkv_paged", _p(qkv), _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin),
         int(cs_offset), _p(k_pages), _p(v_pages), _p(o), B, Hq, Hkv, HEAD_DIM, int(kv_len),
         _p(kv_len_dev), _p(block_table), block_table.stride(0), page_tokens, num_pages,
         float(scale), float(eps), _p(ws), 0 if ws is None else ws.numel(), _stream())
    return o


# ----------------------------------------------------------------------------
# a6/a7: prefill attention
# ----------------------------------------------------------------------------
def _strides_bhs(t: torch.Tensor, name: str):
    """(b, h, s) element strides of a [B, H, S, D] view with unit d stride."""
    if t.stride(3) != 1:
        raise ValueError(f"attn_prefill: {name} must have a contiguous head_dim")
    return (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), t.stride(2))


def attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, start_pos: int = 0,
                 causal: bool = True, scale: float = None, out: torch.Tensor = None):
    """q [B, Hq, S, 128] (any strides with unit d), k/v [B, Hkv, >=start+S, 128].

    Returns out as a [B, Hq, S, 128] view (pass `out` to choose the layout)."""
    _cuda("attn_prefill", q, k, v, out)
    _bf16("attn_prefill", q, k, v, out)
    B, Hq, S, D = q.shape
    Hkv = k.shape[1]
    if k.shape[2] < start_pos + S or v.shape != k.shape:
        raise ValueError("attn_prefill: k/v must hold start_pos + S positions")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device=q.device)
    if v.stride() != k.stride():
        raise ValueError("attn_prefill: k and v must share strides")
    call("q3_attn_prefill", _p(q), _p(k), _p(v), _p(out), B, Hq, Hkv, S, D, int(start_pos),
         1 if causal else 0, float(scale), _strides_bhs(q, "q"), _strides_bhs(k, "k"),
         _strides_bhs(out, "out"), _stream())
    return out


def attn_prefill_tc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, start_pos: int = 0,
                    causal: bool = True, scale: float = None, out: torch.Tensor = None,
                    variant: int = None):
    """attn_prefill on the tcgen05 tensor cores.  q contiguous [B, Hq, S, 128];
    k/v [B, Hkv, rows, 128] contiguous with rows >= start_pos + S; out any
    [B, Hq, S, 128] view whose strides are multiples of 8.  variant 0 (V
    transposed in shared memory), 1 (V as an MN-major operand, O in TMEM) or 2
    (two heads of a KV group per CTA, 128-key tiles, P in TMEM; Hq/Hkv even);
    default Q3VL_PREFILL_TC_VARIANT, else 2 where it applies (the fastest on
    B200), else 1."""
    if variant is None:
        env = os.environ.get("Q3VL_PREFILL_TC_VARIANT")
        if env is not None:
            variant = int(env)
        else:
            variant = 2 if (q.shape[1] // max(1, k.shape[1])) % 2 == 0 else 1
    _cuda("attn_prefill_tc", q, k, v, out)
    _bf16("attn_prefill_tc", q, k, v, out)
    _contig("attn_prefill_tc", q, k, v)
    B, Hq, S, D = q.shape
    _, Hkv, rows, _ = k.shape
    if v.shape != k.shape or rows < start_pos + S:
        raise ValueError("attn_prefill_tc: k/v must hold start_pos + S positions")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device=q.device)
    call("q3_attn_prefill_tc", _p(q), _p(k), _p(v), _p(out), B, Hq, Hkv, S, D, int(start_pos),
         1 if causal else 0, float(scale), rows, _strides_bhs(out, "out"), int(variant),
         _stream())
    return out


def attn_prefill_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                       block_table: torch.Tensor, *, start_pos: int, causal: bool = True,
                       scale: float = None, out: torch.Tensor = None):
    """attn_prefill with K/V read through a block table: q [B, Hq, S, 128] at
    positions start_pos.., keys 0..start_pos+S-1 already in the pages
    [num_pages, Hkv, page_tokens, 128]; block_table int32 [B, width]."""
    _cuda("attn_prefill_paged", q, k_pages, v_pages, block_table, out)
    _bf16("attn_prefill_paged", q, k_pages, v_pages, out)
    _contig("attn_prefill_paged", k_pages, v_pages, block_table)
    if block_table.dtype != torch.int32:
        raise TypeError("attn_prefill_paged: block_table must be int32")
    B, Hq, S, D = q.shape
    num_pages, Hkv, page_tokens, _ = k_pages.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device=q.device)
    call("q3_attn_prefill_paged", _p(q), _p(k_pages), _p(v_pages), _p(out), B, Hq, Hkv, S, D,
         int(start_pos), 1 if causal else 0, float(scale), _strides_bhs(q, "q"),
         _strides_bhs(out, "out"), _p(block_table), block_table.shape[1], page_tokens,
         num_pages, _stream())
    return out


def attn_prefill_tc_paged(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                          block_table: torch.Tensor, *, start_pos: int, causal: bool = True,
                          scale: float = None, out: torch.Tensor = None):
    """attn_prefill_paged on the tcgen05 tensor cores (q3_attn_prefill_tc_paged,
    variant 2): q contiguous [B, Hq, S, 128] with Hq / Hkv even; pages of a
    multiple of 128 tokens."""
    _cuda("attn_prefill_tc_paged", q, k_pages, v_pages, block_table, out)
    _bf16("attn_prefill_tc_paged", q, k_pages, v_pages, out)
    _contig("attn_prefill_tc_paged", q, k_pages, v_pages, block_table)
    if block_table.dtype != torch.int32:
        raise TypeError("attn_prefill_tc_paged: block_table must be int32")
    B, Hq, S, D = q.shape
    num_pages, Hkv, page_tokens, _ = k_pages.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, S, D, dtype=torch.bfloat16, device=q.device)
    call("q3_attn_prefill_tc_paged", _p(q), _p(k_pages), _p(v_pages), _p(out), B, Hq, Hkv, S,
         D, int(start_pos), 1 if causal else 0, float(scale), _strides_bhs(out, "out"),
         _p(block_table), block_table.shape[1], page_tokens, num_pages, _stream())
    return out


# ----------------------------------------------------------------------------
# GEMM
# ----------------------------------------------------------------------------
def gemm(a: torch.Tensor, w: torch.Tensor, epilogue: str = "none", residual: torch.Tensor = None,
         out: torch.Tensor = None) -> torch.Tensor:
    """C = a @ w.T for a [..., K] and K-major weights w [N, K] (bf16)."""
    _cuda("gemm", a, w, residual, out)
    _bf16("gemm", a, w, residual, out)
    _contig("gemm", a, w, residual, out)
    K = a.shape[-1]
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"gemm: weight [N={N}, K={w.shape[1]}] does not match K={K}")
    M = a.numel() // K
    epi = _EPI[epilogue]
    n_out = N // 2 if epi == Q3_EPI_SWIGLU else N
    if out is None:
        out = torch.empty(*a.shape[:-1], n_out, dtype=torch.bfloat16, device=a.device)
    if epi == Q3_EPI_RESIDUAL and (residual is None or residual.numel() != M * N):
        raise ValueError("gemm: residual epilogue needs residual [M, N]")
    call("q3_gemm", _p(a), _p(w), _p(out), M, N, K, epi, _p(residual), _stream())
    return out


def gate_up_swiglu(a: torch.Tensor, w_gate_up: torch.Tensor, norm_w: torch.Tensor = None,
                   eps: float = 1e-6, out: torch.Tensor = None) -> torch.Tensor:
    """MLPBlock's silu(h @ Wg) * (h @ Wu) (model_fused.py:160-169) through
    q3_gate_up_swiglu: a [..., K]; w_gate_up [2*inter, K] K-major with gate/up
    rows interleaved in blocks of 8; h = rmsnorm(a; norm_w) when norm_w is
    given (1..16 rows), else a.  Returns [..., inter]."""
    _cuda("gate_up_swiglu", a, w_gate_up, norm_w, out)
    _bf16("gate_up_swiglu", a, w_gate_up, norm_w, out)
    _contig("gate_up_swiglu", a, w_gate_up, out)
    K = a.shape[-1]
    if w_gate_up.shape[1] != K or w_gate_up.shape[0] % 2:
        raise ValueError(f"gate_up_swiglu: weight {tuple(w_gate_up.shape)} does not match K={K}")
    M, inter = a.numel() // K, w_gate_up.shape[0] // 2
    if out is None:
        out = torch.empty(*a.shape[:-1], inter, dtype=torch.bfloat16, device=a.device)
    call("q3_gate_up_swiglu", _p(a), _p(w_gate_up), _p(out), M, inter, K, _p(norm_w),
         float(eps), _stream())
    return out


def gemm_qkv_rope(h: torch.Tensor, w: torch.Tensor, q_norm_w, k_norm_w, cos, sin, *, B: int,
                  S: int, Hq: int, Hkv: int, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  start_pos: int = 0, cs_use_pos: bool = True, cs_offset: int = 0,
                  cs_stride_b: int = 0, eps: float = 1e-6) -> torch.Tensor:
    """Prefill QKV projection with per-head QK-RMSNorm, RoPE and the KV-cache
    write in the tcgen05 epilogue.  h bf16 [B*S, hidden] (normed); returns q
    [B, Hq, S, 128]; k/v go to the caches at start_pos .. start_pos + S - 1."""
    _cuda("gemm_qkv_rope", h, w, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache)
    _bf16("gemm_qkv_rope", h, w, q_norm_w, k_norm_w, k_cache, v_cache)
    _contig("gemm_qkv_rope", h, w, cos, sin, k_cache, v_cache)
    hidden = h.shape[-1]
    if h.numel() != B * S * hidden or w.shape != ((Hq + 2 * Hkv) * HEAD_DIM, hidden):
        raise ValueError("gemm_qkv_rope: h must be [B*S, hidden], w [(Hq+2Hkv)*128, hidden]")
    if cos.dtype == torch.bfloat16:
        cs_dtype = Q3_BF16
    elif cos.dtype == torch.float32:
        cs_dtype = Q3_F32
    else:
        raise TypeError("gemm_qkv_rope: cos/sin must be bf16 or f32")
    q = torch.empty(B, Hq, S, HEAD_DIM, dtype=torch.bfloat16, device=h.device)
    call("q3_gemm_qkv_rope", _p(h), _p(w), hidden, _p(q_norm_w), _p(k_norm_w), _p(cos), _p(sin),
         cs_dtype, 1 if cs_use_pos else 0, int(cs_offset), int(cs_stride_b), _p(q),
         _p(k_cache), _p(v_cache), B, S, Hq, Hkv, HEAD_DIM, int(start_pos), k_cache.shape[2],
         float(eps), _stream())
    return q


def gemm_qkv_rope_paged(h: torch.Tensor, w: torch.Tensor, q_norm_w, k_norm_w, cos, sin, *,
                        B: int, S: int, Hq: int, Hkv: int, k_pages: torch.Tensor,
                        v_pages: torch.Tensor, block_table: torch.Tensor, start_pos: int = 0,
                        cs_use_pos: bool = True, cs_offset: int = 0, cs_stride_b: int = 0,
                        eps: float = 1e-6) -> torch.Tensor:
    """gemm_qkv_rope with k/v written into page pools through block_table."""
    _cuda("gemm_qkv_rope_paged", h, w, q_norm_w, k_norm_w, cos, sin, k_pages, v_pages,
          block_table)
    _bf16("gemm_qkv_rope_paged", h, w, q_norm_w, k_norm_w, k_pages, v_pages)
    _contig("gemm_qkv_rope_paged", h, w, cos, sin, k_pages, v_pages, block_table)
    hidden = h.shape[-1]
    if h.numel() != B * S * hidden or w.shape != ((Hq + 2 * Hkv) * HEAD_DIM, hidden):
        raise ValueError("gemm_qkv_rope_paged: h must be [B*S, hidden], "
                         "w [(Hq+2Hkv)*128, hidden]")
    if block_table.dtype != torch.int32:
        raise TypeError("gemm_qkv_rope_paged: block_table must be int32")
    cs_dtype = {torch.bfloat16: Q3_BF16, torch.float32: Q3_F32}.get(cos.dtype)
    if cs_dtype is None:
        raise TypeError("gemm_qkv_rope_paged: cos/sin must be bf16 or f32")
    num_pages, _, page_tokens, _ = k_pages.shape
    q = torch.empty(B, Hq, S, HEAD_DIM, dtype=torch.bfloat16, device=h.device)
    call("q3_gemm_qkv_rope_paged", _p(h), _p(w), hidden, _p(q_norm_w), _p(k_norm_w), _p(cos),
         _p(sin), cs_dtype, 1 if cs_use_pos else 0, int(cs_offset), int(cs_stride_b), _p(q),
         _p(k_pages), _p(v_pages), B, S, Hq, Hkv, HEAD_DIM, int(start_pos), _p(block_table),
         block_table.shape[1], page_tokens, num_pages, float(eps), _stream())
    return q


def gemm_norm(a: torch.Tensor, norm_w: torch.Tensor, w: torch.Tensor, eps: float = 1e-6,
              epilogue: str = "none", residual: torch.Tensor = None,
              out: torch.Tensor = None) -> torch.Tensor:
    """C = epilogue(rmsnorm(a; norm_w, eps) @ w.T) for decode shapes (1..16 rows)."""
    _cuda("gemm_norm", a, norm_w, w, residual, out)
    _bf16("gemm_norm", a, norm_w, w, residual, out)
    _contig("gemm_norm", a, norm_w, w, residual, out)
    K = a.shape[-1]
    N = w.shape[0]
    M = a.numel() // K
    epi = _EPI[epilogue]
    n_out = N // 2 if epi == Q3_EPI_SWIGLU else N
    if out is None:
        out = torch.empty(*a.shape[:-1], n_out, dtype=torch.bfloat16, device=a.device)
    call("q3_gemm_norm", _p(a), _p(norm_w), float(eps), _p(w), _p(out), M, N, K, epi,
         _p(residual), _stream())
    return out


def gemm_decode(a: torch.Tensor, w: torch.Tensor, epilogue: str = "none",
                residual: torch.Tensor = None, norm_w: torch.Tensor = None, eps: float = 1e-6,
                ss_in: torch.Tensor = None, ss_tiles: int = 0, ss_out: torch.Tensor = None,
                out: torch.Tensor = None) -> torch.Tensor:
    """Decode projection (1..16 rows): C = epilogue(rmsnorm?(a) @ w.T), with the
    norm's sums of squares optionally taken from `ss_in` (ss_tiles x 16 fp32
    partials) and, for the residual epilogue, written for C into `ss_out`."""
    _cuda("gemm_decode", a, w, residual, norm_w, ss_in, ss_out, out)
    _bf16("gemm_decode", a, w, residual, norm_w, out)
    _contig("gemm_decode", a, w, residual, out)
    K = a.shape[-1]
    N = w.shape[0]
    M = a.numel() // K
    epi = _EPI[epilogue]
    n_out = N // 2 if epi == Q3_EPI_SWIGLU else N
    if out is None:
        out = torch.empty(*a.shape[:-1], n_out, dtype=torch.bfloat16, device=a.device)
    for t, need in ((ss_in, ss_tiles * 16), (ss_out, ((N + 63) // 64) * 16)):
        if t is not None and (t.dtype != torch.float32 or t.numel() < need):
            raise ValueError("gemm_decode: sum-of-squares buffers are float32 [tiles, 16]")
    call("q3_gemm_decode", _p(a), _p(w), _p(out), M, N, K, epi, _p(residual), _p(norm_w),
         float(eps), _p(ss_in), int(ss_tiles), _p(ss_out), _stream())
    return out


class DecodeStepPlan:
    """One decode step of every layer in one persistent kernel (q3_decode_step).

    `layers`: per layer a dict of K-major bf16 weights (w_qkv, w_o, w_gate_up
    interleaved, w_down), bf16 norms (input_norm, post_norm, q_norm, k_norm) and
    the layer's bf16 caches (k_cache, v_cache [B, Hkv, max_seq, 128]).  The
    tensors must outlive the plan.  `cos`/`sin`: bf16 [rows, 64] rope tables."""

    def __init__(self, layers, *, batch: int, hidden: int, q_heads: int, kv_heads: int,
                 inter: int, max_seq: int, eps: float, cos: torch.Tensor, sin: torch.Tensor):
        from ._lib import StepLayer
        arr = (StepLayer * len(layers))()
        keep = []
        for i, d in enumerate(layers):
            for name, _ in StepLayer._fields_:
                t = d[name]
                if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
                    raise ValueError(f"DecodeStepPlan: layer {i} {name} must be contiguous "
                                     "bf16 on the GPU")
                setattr(arr[i], name, t.data_ptr())
                keep.append(t)
        _cuda("decode_step", cos, sin)
        _bf16("decode_step", cos, sin)
        handle = ctypes.c_void_p()
        call("q3_decode_step_create", ctypes.cast(arr, ctypes.c_void_p), len(layers), batch,
             hidden, q_heads, kv_heads, inter, int(max_seq), float(eps), _p(cos), _p(sin),
             cos.shape[0], ctypes.byref(handle))
        self.handle = handle
        self.batch, self.hidden = batch, hidden
        self._keep = keep + [cos, sin]

    def run(self, x: torch.Tensor, ss: torch.Tensor, kv_len_dev: torch.Tensor,
            rope_delta: int = 0) -> torch.Tensor:
        """x bf16 [B, hidden] in place: embedded tokens in, last layer out; ss
        float32 [hidden/128, 16] receives the output's per-tile sums of squares."""
        if self.handle is None:
            raise RuntimeError("DecodeStepPlan is closed")
        if x.shape != (self.batch, self.hidden) or x.dtype != torch.bfloat16:
            raise ValueError("decode_step: x must be bf16 [batch, hidden]")
        if ss.dtype != torch.float32 or ss.numel() < (self.hidden // 128) * 16:
            raise ValueError("decode_step: ss must be float32 [hidden/128, 16]")
        if kv_len_dev.dtype != torch.int32:
            raise TypeError("decode_step: kv_len_dev must be int32")
        _contig("decode_step", x, ss)
        call("q3_decode_step", self.handle, _p(x), _p(ss), _p(kv_len_dev), int(rope_delta),
             _stream())
        return x

    def close(self):
        if self.handle is not None:
            call("q3_decode_step_destroy", self.handle)
            self.handle = None
            self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gate_up_granules4(w_il: torch.Tensor) -> torch.Tensor:
    """The step kernel's gate/up row order from the 8-row interleave of
    q3_gemm (rows 16j..16j+7 gate of features 8j.., 16j+8.. up): granules of 8
    rows holding 4 gate rows then the 4 up rows of the same 4 features, so
    every granule a CTA owns carries whole features.  A new tensor."""
    n2 = w_il.shape[0]
    n = torch.arange(n2, device=w_il.device)
    f = (n // 8) * 4 + (n % 4)                     # feature of new row n
    up = (n % 8) >= 4
    src = (f // 8) * 16 + (f % 8) + up.to(torch.long) * 8
    return w_il.index_select(0, src).contiguous()


class DecodeTPPlan:
    """One decode step of every layer, with the tensor-parallel all-reduce
    inside, as one persistent kernel per GPU (q3_decode_tp).  With
    `block_table` the layers' k_cache / v_cache are page pools and the table
    maps each sequence's positions to pages (q3_decode_tp_create_paged).

    `layers` as for DecodeStepPlan (this rank's shards); `comm` an object with
    a `.handle` to a q3_comm_create communicator of this rank's group, opened,
    with max_cols >= hidden, used by this plan only.  The tensors must outlive
    the plan."""

    def __init__(self, layers, *, batch: int, hidden: int, q_heads: int, kv_heads: int,
                 inter: int, max_seq: int, eps: float, cos: torch.Tensor, sin: torch.Tensor,
                 comm, block_table: torch.Tensor = None):
        from ._lib import StepLayer
        arr = (StepLayer * len(layers))()
        keep = []
        for i, d in enumerate(layers):
            d = dict(d)
            d["w_gate_up"] = gate_up_granules4(d["w_gate_up"])   # the kernel's row order
            for name, _ in StepLayer._fields_:
                t = d[name]
                if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
                    raise ValueError(f"DecodeTPPlan: layer {i} {name} must be contiguous "
                                     "bf16 on the GPU")
                setattr(arr[i], name, t.data_ptr())
                keep.append(t)
        _cuda("decode_tp", cos, sin)
        _bf16("decode_tp", cos, sin)
        handle = ctypes.c_void_p()
        if block_table is None:
            call("q3_decode_tp_create", ctypes.cast(arr, ctypes.c_void_p), len(layers), batch,
                 hidden, q_heads, kv_heads, inter, int(max_seq), float(eps), _p(cos), _p(sin),
                 cos.shape[0], comm.handle, ctypes.byref(handle))
        else:
            # paged caches: k_cache / v_cache are page pools [pages, kv_heads, page_tokens, 128]
            if not (block_table.is_cuda and block_table.dtype == torch.int32 and
                    block_table.dim() == 2 and block_table.is_contiguous() and
                    block_table.shape[0] >= batch):
                raise ValueError("DecodeTPPlan: block_table must be contiguous int32 "
                                 "[>= batch, width] on the GPU")
            pool = layers[0]["k_cache"]
            call("q3_decode_tp_create_paged", ctypes.cast(arr, ctypes.c_void_p), len(layers),
                 batch, hidden, q_heads, kv_heads, inter, int(max_seq), float(eps), _p(cos),
                 _p(sin), cos.shape[0], comm.handle, _p(block_table), block_table.shape[1],
                 pool.shape[2], pool.shape[0], ctypes.byref(handle))
            keep.append(block_table)
        self.handle = handle
        self.batch, self.hidden = batch, hidden
        self._keep = keep + [cos, sin, comm]

    def run(self, x: torch.Tensor, kv_len_dev: torch.Tensor, rope_delta: int = 0) -> torch.Tensor:
        """x bf16 [B, hidden] in place: embedded tokens in, last layer out."""
        if self.handle is None:
            raise RuntimeError("DecodeTPPlan is closed")
        if x.shape != (self.batch, self.hidden) or x.dtype != torch.bfloat16:
            raise ValueError("decode_tp: x must be bf16 [batch, hidden]")
        if kv_len_dev.dtype != torch.int32:
            raise TypeError("decode_tp: kv_len_dev must be int32")
        _cuda("decode_tp", x, kv_len_dev)
        _contig("decode_tp", x)
        call("q3_decode_tp", self.handle, _p(x), _p(kv_len_dev), int(rope_delta), _stream())
        return x

    def close(self):
        if self.handle is not None:
            call("q3_decode_tp_destroy", self.handle)
            self.handle = None
            self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_ar(a: torch.Tensor, w: torch.Tensor, comm, residual: torch.Tensor = None,
            out: torch.Tensor = None, ss_out: torch.Tensor = None) -> torch.Tensor:
    """C = residual + all_reduce_sum(a @ w.T) over the communicator's ranks
    (decode shapes: a has 1..16 rows).  Every rank must call this in the same
    order, as with a collective.  `ss_out` (float32, (N/64) x 16) receives the
    per-tile sums of squares of C for a following norm-fused projection."""
    _cuda("gemm_ar", a, w, residual, out, ss_out)
    _bf16("gemm_ar", a, w, residual, out)
    _contig("gemm_ar", a, w, residual, out)
    K = a.shape[-1]
    N = w.shape[0]
    M = a.numel() // K
    if out is None:
        out = torch.empty(*a.shape[:-1], N, dtype=torch.bfloat16, device=a.device)
    if residual is not None and residual.numel() != M * N:
        raise ValueError("gemm_ar: residual must be [M, N]")
    if ss_out is not None and (ss_out.dtype != torch.float32 or ss_out.numel() < (N // 64) * 16):
        raise ValueError("gemm_ar: ss_out must be float32 [N/64, 16]")
    call("q3_gemm_ar", _p(a), _p(w), _p(out), M, N, K, _p(residual), _p(ss_out), comm.handle,
         _stream())
    return out


# ----------------------------------------------------------------------------
# embedding / argmax
# ----------------------------------------------------------------------------
def gemm_allreduce(a: torch.Tensor, w: torch.Tensor, comm, residual: torch.Tensor = None,
                   out: torch.Tensor = None) -> torch.Tensor:
    """Prefill row-parallel projection + all-reduce (+ residual) in one call
    (q3_gemm_allreduce): out = residual + sum over ranks of a @ w.T, with a
    [M, K] (16 < M), w [N, K] this rank's K-major shard.  Collective."""
    _cuda("gemm_allreduce", a, w, residual, out)
    _bf16("gemm_allreduce", a, w, residual, out)
    _contig("gemm_allreduce", a, w, residual, out)
    K = a.shape[-1]
    N = w.shape[0]
    M = a.numel() // K
    if w.shape[1] != K:
        raise ValueError(f"gemm_allreduce: weight [N={N}, K={w.shape[1]}] does not match K={K}")
    if residual is not None and residual.numel() != M * N:
        raise ValueError("gemm_allreduce: residual must be [M, N]")
    if out is None:
        out = torch.empty(*a.shape[:-1], N, dtype=torch.bfloat16, device=a.device)
    call("q3_gemm_allreduce", _p(a), _p(w), _p(out), M, N, K, _p(residual), comm.handle,
         _stream())
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    _cuda("embed", ids, table, out)
    _bf16("embed", table, out)
    ids_c = ids.contiguous()
    if ids_c.dtype != torch.int64:
        ids_c = ids_c.to(torch.int64)
    V, H = table.shape
    if out is None:
        out = torch.empty(*ids.shape, H, dtype=torch.bfloat16, device=table.device)
    call("q3_embed", _p(ids_c), _p(table), _p(out), ids_c.numel(), H, V, _stream())
    return out


def add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """bf16(a + b)."""
    _cuda("add", a, b, out)
    _bf16("add", a, b, out)
    _contig("add", a, b, out)
    if a.shape != b.shape:
        raise ValueError("add: shapes differ")
    out = torch.empty_like(a) if out is None else out
    call("q3_add", _p(a), _p(b), _p(out), a.numel(), _stream())
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    _cuda("argmax", logits, out)
    _bf16("argmax", logits)
    _contig("argmax", logits)
    V = logits.shape[-1]
    rows = logits.numel() // V
    if out is None:
        out = torch.empty(logits.shape[:-1], dtype=torch.int64, device=logits.device)
    call("q3_argmax", _p(logits), rows, V, _p(out), _stream())
    return out


def argmax_key(logits: torch.Tensor, col_offset: int, out: torch.Tensor = None) -> torch.Tensor:
    """Per-row int64 keys of a vocabulary slice whose MAX over ranks encodes the
    global argmax (first index on ties); decode with argmax_key_index."""
    _cuda("argmax_key", logits, out)
    _bf16("argmax_key", logits)
    _contig("argmax_key", logits)
    V = logits.shape[-1]
    rows = logits.numel() // V
    if out is None:
        out = torch.empty(logits.shape[:-1], dtype=torch.int64, device=logits.device)
    call("q3_argmax_key", _p(logits), rows, V, int(col_offset), _p(out), _stream())
    return out


def argmax_key_index(keys: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    _cuda("argmax_key_index", keys, out)
    if keys.dtype != torch.int64 or not keys.is_contiguous():
        raise TypeError("argmax_key_index: contiguous int64 keys")
    if out is None:
        out = torch.empty_like(keys)
    call("q3_argmax_key_index", _p(keys), keys.numel(), _p(out), _stream())
    return out


def lm_head_argmax(h: torch.Tensor, w_lm: torch.Tensor, norm_w: torch.Tensor = None,
                   eps: float = 1e-6, col_offset: int = 0, keys: bool = False,
                   logits: torch.Tensor = None, out: torch.Tensor = None) -> torch.Tensor:
    """Final norm (when norm_w is given; 1..16 rows), lm_head projection and
    greedy argmax in one library call (q3_lm_head_argmax).  h [rows, K];
    w_lm [V, K] K-major, the vocabulary slice starting at col_offset.
    Returns int64 [rows]: indices, or with keys=True the argmax_key keys of the
    slice.  `logits` [rows, V] bf16, when given, receives the logits."""
    _cuda("lm_head_argmax", h, w_lm, norm_w, logits, out)
    _bf16("lm_head_argmax", h, w_lm, norm_w, logits)
    _contig("lm_head_argmax", h, w_lm, logits)
    K = h.shape[-1]
    V = w_lm.shape[0]
    if w_lm.shape[1] != K:
        raise ValueError(f"lm_head_argmax: weight [V={V}, K={w_lm.shape[1]}] does not match K={K}")
    rows = h.numel() // K
    if logits is None:
        logits = torch.empty(rows, V, dtype=torch.bfloat16, device=h.device)
    elif logits.numel() != rows * V:
        raise ValueError("lm_head_argmax: logits must be [rows, V]")
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=h.device)
    call("q3_lm_head_argmax", _p(h), _p(norm_w), float(eps), _p(w_lm), rows, V, K,
         int(col_offset), _p(logits), 1 if keys else 0, _p(out), _stream())
    return out


def l2_prefetch(t: torch.Tensor) -> None:
    """Prefetch a contiguous tensor's bytes into L2 (q3_l2_prefetch), ahead of
    the kernel that reads it."""
    _cuda("l2_prefetch", t)
    _contig("l2_prefetch", t)
    call("q3_l2_prefetch", _p(t), t.numel() * t.element_size(), _stream())


def device_error(clear: bool = True) -> int:
    """Error code recorded by a kernel whose bounded wait timed out (0 = none)."""
    return int(_lib.raw("q3_device_error")(1 if clear else 0))


# device error words of the peer exchanges' bounded waits: the decode
# all-reduce (q3_gemm_ar) and the prefill two-shot exchange (partials, reduced
# tiles)
PEER_TIMEOUT_CODES = (0x501, 0x701, 0x702)


def check_device_error(where: str = "") -> None:
    """Read and clear the device error word; raise Q3Error if a kernel recorded
    one: Q3_ERR_TIMEOUT for a peer exchange whose bounded wait ran out (a rank
    that never delivered), Q3_ERR_CUDA for any other recorded code."""
    code = device_error(clear=True)
    if not code:
        return
    if code in PEER_TIMEOUT_CODES:
        raise _lib.Q3Error(_lib.Q3_ERR_TIMEOUT, where or "device",
                           f"a peer never delivered its partials (code {code:#x})")
    raise _lib.Q3Error(_lib.Q3_ERR_CUDA, where or "device", f"kernel recorded error {code:#x}")

