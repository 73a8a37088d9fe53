"""Qwen3-VL-8B text decoder on B200 -- drop-in for the reference model_fused.py.

Same module/class names and signatures as the reference
(model_fused.py:31-362): RMSNorm, RotaryEmbedding, AttentionBlock,
OProjection, MLPBlock, FusedLinear, DecoderLayer, Qwen3VLDecoderFused.  Weights
arrive in the reference's [in, out] convention; each module keeps one K-major
[out, in] copy for the kernels and exposes the [in, out] view under the
reference's attribute name.  Every op runs on the q3vl sm_100a kernels
(q3vl.ops); CPU tensors raise instead of falling back.

Per layer (forward_layer) the kernels are:
  rmsnorm -> QKV GEMM -> QK-norm+RoPE+KV-write -> prefill/decode attention ->
  o_proj GEMM (+residual) -> [TP all-reduce + fused add+rmsnorm | rmsnorm] ->
  gate_up GEMM with SwiGLU epilogue -> down GEMM (+residual) [-> all-reduce].
Decode runs as a captured CUDA graph per (batch, KV bucket) with the token
and position kept on the device (no per-token host sync).
"""
from __future__ import annotations

import math
import os
import time

import torch
import torch.distributed as dist
import torch.nn as nn

from q3vl import layout, ops
from q3vl._lib import Q3Error
from q3vl.kv_pages import KVPagePool, PagedLayer

KV_BUCKETS = (2048, 4096, 8192)


def _param(t: torch.Tensor) -> nn.Parameter:
    return nn.Parameter(t, requires_grad=False)


class RMSNorm(nn.Module):
    """model_fused.py:31-40."""

    def __init__(self, weight, eps=1e-6):
        super().__init__()
        self.weight = _param(weight)
        self.eps = eps

    def forward(self, x):
        return ops.rmsnorm(x.contiguous(), self.weight, self.eps)


class RotaryEmbedding:
    """model_fused.py:43-58: bf16 cos/sin tables built on the host exactly as the
    reference builds them; device copies stay resident, so `get` slices HBM
    instead of copying from the host every layer."""

    def __init__(self, head_dim, max_seq_len=8192, base=1000000.0):
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        t = torch.arange(max_seq_len, dtype=torch.float32)
        freqs = torch.outer(t, inv_freq)
        self.cos_cached = freqs.cos().to(torch.bfloat16)
        self.sin_cached = freqs.sin().to(torch.bfloat16)
        self.inv_freq = inv_freq
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.base = base
        self._dev = {}

    def tables(self, device):
        key = str(torch.device(device))
        if key not in self._dev:
            self._dev[key] = (self.cos_cached.to(device), self.sin_cached.to(device),
                              self.inv_freq.to(device))
        return self._dev[key]

    def get(self, seq_len, offset=0, device=None):
        if device is None:
            return (self.cos_cached[offset:offset + seq_len],
                    self.sin_cached[offset:offset + seq_len])
        cos, sin, _ = self.tables(device)
        return cos[offset:offset + seq_len], sin[offset:offset + seq_len]


class AttentionBlock(nn.Module):
    """model_fused.py:61-131: norm -> QKV -> per-head QK-norm -> RoPE."""

    def __init__(self, qkv_weight, qkv_bias, o_proj_weight, input_norm_weight, q_norm_weight,
                 k_norm_weight, num_q_heads, num_kv_heads, head_dim, eps=1e-6):
        super().__init__()
        if head_dim != ops.HEAD_DIM:
            raise ValueError(f"head_dim {head_dim} unsupported (kernels are built for 128)")
        self.qkv_weight_km = _param(layout.k_major(qkv_weight))
        self.qkv_bias = _param(qkv_bias) if qkv_bias is not None else None
        self.input_norm_weight = _param(input_norm_weight)
        self.q_norm_weight = _param(q_norm_weight)
        self.k_norm_weight = _param(k_norm_weight)
        self.o_proj_weight_km = _param(layout.k_major(o_proj_weight))
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.q_dim = num_q_heads * head_dim
        self.kv_dim = num_kv_heads * head_dim
        self.eps = eps

    @property
    def qkv_weight(self):
        return self.qkv_weight_km.t()

    @property
    def o_proj_weight(self):
        return self.o_proj_weight_km.t()

    def qkv(self, h2d: torch.Tensor) -> torch.Tensor:
        out = ops.gemm(h2d, self.qkv_weight_km)
        if self.qkv_bias is not None:
            out = ops.add(out, self.qkv_bias.expand_as(out).contiguous())
        return out

    def forward(self, hidden, cos, sin):
        """hidden [B, S, H]; cos/sin [S, D/2] -> q [B,Hq,S,D], k/v [B,Hkv,S,D]."""
        B, S, H = hidden.shape
        h = ops.rmsnorm(hidden.reshape(B * S, H).contiguous(), self.input_norm_weight, self.eps)
        qkv = self.qkv(h)
        return ops.qkv_norm_rope(qkv, self.q_norm_weight, self.k_norm_weight,
                                 cos.contiguous(), sin.contiguous(), B=B, S=S,
                                 Hq=self.num_q_heads, Hkv=self.num_kv_heads, cs_use_pos=False,
                                 want_kv=True, eps=self.eps)


class OProjection(nn.Module):
    """model_fused.py:134-141."""

    def __init__(self, weight):
        super().__init__()
        self.weight_km = _param(layout.k_major(weight))

    @property
    def weight(self):
        return self.weight_km.t()

    def forward(self, x):
        return ops.gemm(x.contiguous(), self.weight_km)


class MLPBlock(nn.Module):
    """model_fused.py:144-172: norm -> gate_up -> SiLU*up -> down (partial sum)."""

    def __init__(self, gate_up_weight, down_weight, post_norm_weight, eps=1e-6):
        super().__init__()
        self.gate_up_weight_il = _param(layout.gate_up_from_fused(gate_up_weight))
        self.down_weight_km = _param(layout.k_major(down_weight))
        self.post_norm_weight = _param(post_norm_weight)
        self.eps = eps

    @property
    def gate_up_weight(self):
        return layout.fused_from_gate_up(self.gate_up_weight_il)

    @property
    def down_weight(self):
        return self.down_weight_km.t()

    def forward(self, hidden):
        shp = hidden.shape
        x = hidden.reshape(-1, shp[-1]).contiguous()
        h = ops.rmsnorm(x, self.post_norm_weight, self.eps)
        act = ops.gemm(h, self.gate_up_weight_il, "swiglu")
        return ops.gemm(act, self.down_weight_km).view(*shp[:-1], -1)


class FusedLinear(nn.Module):
    """model_fused.py:175-186 (lm_head)."""

    def __init__(self, weight, bias=None):
        super().__init__()
        self.weight_km = _param(layout.k_major(weight))
        self.bias = _param(bias) if bias is not None else None

    @property
    def weight(self):
        return self.weight_km.t()

    def forward(self, x):
        shp = x.shape
        out = ops.gemm(x.reshape(-1, shp[-1]).contiguous(), self.weight_km)
        if self.bias is not None:
            out = ops.add(out, self.bias.expand_as(out).contiguous())
        return out.view(*shp[:-1], -1)


class DecoderLayer:
    """model_fused.py:189-194."""

    def __init__(self, attn_block, o_proj, mlp_block):
        self.attn_block = attn_block
        self.o_proj = o_proj
        self.mlp_block = mlp_block


class RowRope:
    """RoPE rows for decode when the rope delta differs per sequence (batched
    multimodal prompts): cos/sin bf16 [B * rows, 64] with row b * rows + t
    holding position t + delta_b, built with RotaryEmbedding's own ops so a
    position's row equals the shared table's."""

    def __init__(self, cos, sin, rows):
        self.cos, self.sin, self.rows = cos, sin, rows


class _DecodeGraph:
    """Captured decode steps for a fixed batch, KV bucket and cache storage:
    `graph` one step (the next tokens land in `tok`), `multi` `steps` steps
    in a row, each writing its tokens to hist[j] and advancing the device
    position counters itself, so the host replays once per `steps` tokens."""

    def __init__(self, graph, tok, pos, kv_len, multi=None, hist=None, steps=1):
        self.graph, self.tok, self.pos, self.kv_len = graph, tok, pos, kv_len
        self.multi, self.hist, self.steps = multi, hist, steps


class Qwen3VLDecoderFused:
    """model_fused.py:197-362 on the q3vl kernels."""

    def __init__(self, layers, lm_head, embed_tokens, final_norm, rotary, tp_size, num_q_heads,
                 num_kv_heads, head_dim, max_seq_len, device):
        self.layers = layers
        self.lm_head = lm_head
        self.embed_tokens = embed_tokens
        self.final_norm = final_norm
        self.rotary = rotary
        self.tp_size = tp_size
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.max_seq_len = max_seq_len
        self.device = torch.device(device)
        self.num_layers = len(layers)
        self.q_dim = num_q_heads * head_dim
        self.scale = 1.0 / math.sqrt(head_dim)
        self.comm = None            # optional in-kernel all-reduce (q3vl.comm)
        self.pcomm = None           # optional prefill two-shot all-reduce (q3vl.comm)
        self._graphs = {}
        self._kv_pool = {}
        self.use_graphs = os.environ.get("Q3VL_DECODE_GRAPHS", "1") != "0"
        # decode: RMSNorms fused into the projections that consume them
        self.fuse_norm = os.environ.get("Q3VL_FUSE_NORM", "1") != "0"
        # decode graphs: every layer in one persistent kernel (q3_decode_step);
        # opt-in until it beats the per-kernel decode step
        self.use_step_kernel = os.environ.get("Q3VL_STEP_KERNEL", "0") == "1"
        # decode at tensor parallelism: every layer of a step in one persistent
        # kernel per GPU with the all-reduce inside (q3_decode_tp).  Default at
        # TP >= 4, where it beats the per-kernel step (measured on B200: TP8
        # 3553 vs 2896 tok/s, TP4 3396 vs 3174); at TP2 the per-kernel step is
        # faster (2631 vs 2369).  Q3VL_TP_KERNEL=1 / 0 forces it on / off.
        tpk = os.environ.get("Q3VL_TP_KERNEL")
        self.use_tp_kernel = (tpk == "1") if tpk in ("0", "1") else self.tp_size >= 4
        self.mk_comm = None
        self._tp_plans = {}
        # decode graphs replay this many steps per launch from the host (the
        # position counters advance inside the graph); 1 replays step by step
        self.graph_steps = max(1, int(os.environ.get("Q3VL_DECODE_GRAPH_STEPS", "8")))
        # prefill: QK-norm, RoPE and the KV write in the QKV GEMM's epilogue
        self.fuse_qkv = os.environ.get("Q3VL_FUSE_QKV", "1") != "0"
        # decode: QK-norm, RoPE and the KV write inside the attention kernel
        # (opt-in: the separate norm/RoPE kernel already hides under the
        # attention kernel's early K/V stream, and measured 0.4% faster)
        self.fuse_attn_qkv = os.environ.get("Q3VL_FUSE_ATTN_QKV", "0") == "1"
        # greedy decoding at TP > 1: MAX all-reduce of per-rank argmax keys
        # instead of the all_gather of every rank's logits
        self.dist_argmax = os.environ.get("Q3VL_DIST_ARGMAX", "1") != "0"
        # prefill attention on the tcgen05 tensor cores (measured on B200, config
        # 2: 578 TFLOP/s for the persistent variant against 147 for the mma.sync
        # kernel); Q3VL_PREFILL_TC=0 selects the mma.sync kernel
        self.prefill_tc = os.environ.get("Q3VL_PREFILL_TC", "1") == "1"
        # decode: weights brought into L2 while the attention kernel, which
        # leaves HBM bandwidth idle, runs (opt-in until measured):
        # "oproj" this layer's o_proj, "qkv" the next layer's QKV projection
        pf = {t.strip() for t in os.environ.get("Q3VL_L2_PREFETCH", "").split(",") if t.strip()}
        self.l2_prefetch_oproj = "oproj" in pf
        self.l2_prefetch_qkv = "qkv" in pf
        self._step_plans = {}
        self._ss_step = None
        self._page_tables = {}
        self._row_ropes = {}

    # ------------------------------------------------------------------ cache
    def init_kv_cache(self, batch_size=1):
        """model_fused.py:224-232: per layer (k, v) [B, Hkv, max_seq_len, D] bf16."""
        cache = []
        for _ in range(self.num_layers):
            k = torch.zeros(batch_size, self.num_kv_heads, self.max_seq_len, self.head_dim,
                            dtype=torch.bfloat16, device=self.device)
            cache.append((k, torch.zeros_like(k)))
        return cache

    # ----------------------------------------------------------------- comm
    def _all_reduce(self, t: torch.Tensor):
        """model_fused.py:267,274 for shapes the in-kernel path does not cover."""
        if self.tp_size > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)

    def enable_peer_allreduce(self, group=None, max_cols: int = 16384):
        """Switch decode-shaped o_proj/down projections (<= 16 tokens) to the
        fused in-kernel all-reduce over NVLink peer memory; prefill keeps
        dist.all_reduce.  Collective: every rank must call it."""
        if self.tp_size > 1 and self.comm is None:
            from q3vl.comm import PeerComm
            self.comm = PeerComm(group=group, max_cols=max_cols, device=self.device)
            self._graphs.clear()
        if self.tp_size > 1 and self.use_tp_kernel and self.mk_comm is None:
            # the step kernel's own exchange buffers (its words must not meet
            # q3_gemm_ar's)
            from q3vl.comm import PeerComm
            H = self.layers[0].attn_block.input_norm_weight.numel()
            self.mk_comm = PeerComm(group=group, max_cols=H, device=self.device)
        rows = os.environ.get("Q3VL_PREFILL_AR", "") == "peer"
        if self.tp_size > 1 and rows and self.pcomm is None:
            self.enable_prefill_allreduce(group=group)
        return self.comm

    def enable_prefill_allreduce(self, group=None, max_rows: int = 8192):
        """Switch prefill-shaped o_proj/down projections (16 < tokens <=
        max_rows) to the two-shot all-reduce over NVLink peer memory
        (q3_gemm_allreduce) in place of dist.all_reduce.  Collective: every
        rank must call it.  Opt-in (Q3VL_PREFILL_AR=peer with
        enable_peer_allreduce) until measured."""
        if self.tp_size > 1 and self.pcomm is None:
            from q3vl.comm import PrefillComm
            hidden = self.layers[0].attn_block.input_norm_weight.numel()
            self.pcomm = PrefillComm(group=group, max_rows=max_rows, max_cols=hidden,
                                     device=self.device)
        return self.pcomm

    def close(self):
        """Release captured graphs and the peer communicator (collective)."""
        self._graphs.clear()
        for plan in self._step_plans.values():
            plan.close()
        self._step_plans.clear()
        for plan in self._tp_plans.values():
            if plan is not None:
                plan.close()
        self._tp_plans.clear()
        if self.mk_comm is not None:
            self.mk_comm.close()
            self.mk_comm = None
        if self.comm is not None:
            self.comm.close()
            self.comm = None
        if self.pcomm is not None:
            self.pcomm.close()
            self.pcomm = None

    @property
    def _eps(self):
        return self.layers[0].attn_block.eps

    # ----------------------------------------------------------------- layer
    def _ss_ok(self, B: int, S: int) -> bool:
        """True when the last layer's down projection left the sums of squares
        of its output rows in _ss_buf(1) (decode at TP1, or with the in-kernel
        all-reduce, whose outputs are identical on every rank)."""
        return (B * S <= 16 and (self.tp_size == 1 or self.comm is not None) and
                self.num_layers > 0 and self.fuse_norm and
                self.layers[-1].attn_block.qkv_bias is None)

    def _ss_buf(self, i: int) -> torch.Tensor:
        """Per-tile sums of squares handed from a residual projection to the
        next projection's fused RMSNorm (0: after o_proj, 1: after down)."""
        if getattr(self, "_ss", None) is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("norm buffers must exist before graph capture")
            self._ss = torch.zeros(2, 256 * 16, dtype=torch.float32, device=self.device)
        return self._ss[i]

    def _layer(self, x, pend, layer_idx, kv_cache, start_pos, S, B, rope=None, pos_dev=None,
               kv_len_dev=None, kv_bound=None, rope_delta=0, ss_valid=False):
        """One decoder layer on the residual stream x [T, H].  `pend` is a partial
        sum still to be added to x (TP>1 keeps the add fused with the next norm).
        `ss_valid` says the previous layer's down projection left the sums of
        squares of x in _ss_buf(1).  Returns (x, pend) in the same convention."""
        L = self.layers[layer_idx]
        ab, mlp = L.attn_block, L.mlp_block
        H = x.shape[-1]
        T = B * S
        decode = T <= 16
        peer = self.tp_size > 1 and self.comm is not None and decode
        # prefill: projection + two-shot all-reduce + residual in the library
        two_shot = (self.tp_size > 1 and self.pcomm is not None and not decode and
                    T <= self.pcomm.max_rows and H <= self.pcomm.max_cols and H % 32 == 0)
        # decode with per-tile sums of squares handed between projections: every
        # RMSNorm runs inside the projection that consumes it
        fast = (decode and (self.tp_size == 1 or peer) and ab.qkv_bias is None and
                H <= 256 * 64 and self.fuse_norm)
        # a paged cache (PagedLayer): K/V rows are written through the block
        # table, and decode attention reads through it
        paged = isinstance(kv_cache[layer_idx], PagedLayer)
        # prefill without a QKV bias: the QKV GEMM's epilogue applies the head
        # norms and RoPE and writes the caches (no qkv tensor)
        fused_qkv = not decode and ab.qkv_bias is None and self.fuse_qkv
        qkv = None
        if pend is not None:
            xn = torch.empty_like(x)
            h = ops.rmsnorm(pend, ab.input_norm_weight, ab.eps, add=x, h_out=xn)
            x = xn
            if not fused_qkv:
                qkv = ab.qkv(h)
        elif decode and ab.qkv_bias is None and self.fuse_norm:
            # decode: the input RMSNorm runs inside the QKV projection
            ss = self._ss_buf(1) if (fast and ss_valid) else None
            qkv = ops.gemm_decode(x, ab.qkv_weight_km, norm_w=ab.input_norm_weight, eps=ab.eps,
                                  ss_in=ss, ss_tiles=H // 64)
        else:
            h = ops.rmsnorm(x, ab.input_norm_weight, ab.eps)
            if not fused_qkv:
                qkv = ab.qkv(h)
        kc, vc = kv_cache[layer_idx]
        if rope is None and isinstance(rope_delta, RowRope):
            cos, sin = rope_delta.cos, rope_delta.sin
            cs_use_pos, cs_stride_b, cs_offset = True, rope_delta.rows, 0
        elif rope is None:
            cos, sin, _ = self.rotary.tables(self.device)
            cs_use_pos, cs_stride_b, cs_offset = True, 0, rope_delta
        else:
            cos, sin = rope
            cs_use_pos, cs_stride_b, cs_offset = False, S, 0
        fused_attn = (S == 1 and rope is None and qkv is not None and self.fuse_attn_qkv and
                      cos.dtype == torch.bfloat16 and not isinstance(rope_delta, RowRope))
        if paged and fused_qkv:
            q = ops.gemm_qkv_rope_paged(h.view(T, H), ab.qkv_weight_km, ab.q_norm_weight,
                                        ab.k_norm_weight, cos, sin, B=B, S=S,
                                        Hq=ab.num_q_heads, Hkv=ab.num_kv_heads, k_pages=kc,
                                        v_pages=vc, block_table=kv_cache[layer_idx].table,
                                        start_pos=start_pos, cs_use_pos=cs_use_pos,
                                        cs_offset=cs_offset, cs_stride_b=cs_stride_b,
                                        eps=ab.eps)
        elif fused_attn:
            q = None  # computed inside the attention kernel from qkv
        elif paged:
            # K/V rows go straight into their pages (no dense copy)
            q = ops.qkv_norm_rope_paged(qkv, ab.q_norm_weight, ab.k_norm_weight, cos, sin, B=B,
                                        S=S, Hq=ab.num_q_heads, Hkv=ab.num_kv_heads, k_pages=kc,
                                        v_pages=vc, block_table=kv_cache[layer_idx].table,
                                        start_pos=start_pos, pos_dev=pos_dev,
                                        cs_use_pos=cs_use_pos, cs_offset=cs_offset,
                                        cs_stride_b=cs_stride_b, eps=ab.eps)
        elif fused_qkv:
            q = ops.gemm_qkv_rope(h.view(T, H), ab.qkv_weight_km, ab.q_norm_weight,
                                  ab.k_norm_weight, cos, sin, B=B, S=S, Hq=ab.num_q_heads,
                                  Hkv=ab.num_kv_heads, k_cache=kc, v_cache=vc,
                                  start_pos=start_pos, cs_use_pos=cs_use_pos, cs_offset=cs_offset,
                                  cs_stride_b=cs_stride_b, eps=ab.eps)
        else:
            q, _, _ = ops.qkv_norm_rope(qkv, ab.q_norm_weight, ab.k_norm_weight, cos, sin, B=B,
                                        S=S, Hq=ab.num_q_heads, Hkv=ab.num_kv_heads,
                                        start_pos=start_pos, pos_dev=pos_dev,
                                        cs_use_pos=cs_use_pos, cs_offset=cs_offset,
                                        cs_stride_b=cs_stride_b, k_cache=kc, v_cache=vc,
                                        eps=ab.eps)
        if S == 1:
            bound = kv_bound if kv_bound is not None else start_pos + 1
            if self.l2_prefetch_oproj:
                ops.l2_prefetch(L.o_proj.weight_km)
            if self.l2_prefetch_qkv and layer_idx + 1 < self.num_layers:
                ops.l2_prefetch(self.layers[layer_idx + 1].attn_block.qkv_weight_km)
            if paged and fused_attn:
                attn = ops.attn_decode_qkv_paged(qkv, ab.q_norm_weight, ab.k_norm_weight, cos,
                                                 sin, kc, vc, kv_cache[layer_idx].table,
                                                 Hq=ab.num_q_heads, Hkv=ab.num_kv_heads,
                                                 kv_len=bound, kv_len_dev=kv_len_dev,
                                                 cs_offset=cs_offset, scale=self.scale,
                                                 eps=ab.eps)
            elif paged:
                attn = ops.attn_decode_paged(q.view(B, ab.num_q_heads, self.head_dim), kc, vc,
                                             kv_cache[layer_idx].table, kv_len=bound,
                                             kv_len_dev=kv_len_dev, scale=self.scale)
            elif fused_attn:
                attn = ops.attn_decode_qkv(qkv, ab.q_norm_weight, ab.k_norm_weight, cos, sin, kc,
                                           vc, Hq=ab.num_q_heads, Hkv=ab.num_kv_heads,
                                           kv_len=bound, kv_len_dev=kv_len_dev,
                                           cs_offset=cs_offset, scale=self.scale, eps=ab.eps)
            else:
                attn = ops.attn_decode(q.view(B, ab.num_q_heads, self.head_dim), kc, vc,
                                       kv_len=bound, kv_len_dev=kv_len_dev, scale=self.scale)
            attn = attn.view(T, ab.q_dim)
        else:
            attn = torch.empty(B, S, ab.num_q_heads, self.head_dim, dtype=torch.bfloat16,
                               device=x.device)
            if paged:
                # this call's K/V rows went into the pages above; earlier
                # positions are there from earlier calls
                if (self.prefill_tc and q.is_contiguous() and kc.shape[2] % 128 == 0 and
                        (ab.num_q_heads // ab.num_kv_heads) % 2 == 0):
                    ops.attn_prefill_tc_paged(q, kc, vc, kv_cache[layer_idx].table,
                                              start_pos=start_pos, causal=True, scale=self.scale,
                                              out=attn.transpose(1, 2))
                else:
                    ops.attn_prefill_paged(q, kc, vc, kv_cache[layer_idx].table,
                                           start_pos=start_pos, causal=True, scale=self.scale,
                                           out=attn.transpose(1, 2))
            elif self.prefill_tc and q.is_contiguous():
                ops.attn_prefill_tc(q, kc, vc, start_pos=start_pos, causal=True,
                                    scale=self.scale, out=attn.transpose(1, 2))
            else:
                ops.attn_prefill(q, kc, vc, start_pos=start_pos, causal=True, scale=self.scale,
                                 out=attn.transpose(1, 2))
            attn = attn.view(T, ab.q_dim)
        if fast:
            # o_proj + residual (emits the sums of squares of x2), gate/up with the
            # post-attention norm fused in, down + residual (emits them for the next
            # layer's input norm); at TP>1 both row-parallel projections all-reduce
            # from inside the kernel
            if peer:
                x2 = ops.gemm_ar(attn, L.o_proj.weight_km, self.comm, residual=x,
                                 ss_out=self._ss_buf(0))
            else:
                x2 = ops.gemm_decode(attn, L.o_proj.weight_km, "residual", residual=x,
                                     ss_out=self._ss_buf(0))
            act = ops.gemm_decode(x2, mlp.gate_up_weight_il, "swiglu",
                                  norm_w=mlp.post_norm_weight, eps=mlp.eps,
                                  ss_in=self._ss_buf(0), ss_tiles=H // 64)
            if peer:
                return ops.gemm_ar(act, mlp.down_weight_km, self.comm, residual=x2,
                                   ss_out=self._ss_buf(1)), None
            return ops.gemm_decode(act, mlp.down_weight_km, "residual", residual=x2,
                                   ss_out=self._ss_buf(1)), None
        h2 = None
        if self.tp_size == 1:
            x2 = ops.gemm(attn, L.o_proj.weight_km, "residual", residual=x)
        elif peer:
            # o_proj partial all-reduced from inside the kernel, residual fused
            x2 = ops.gemm_ar(attn, L.o_proj.weight_km, self.comm, residual=x)
        elif two_shot:
            x2 = ops.gemm_allreduce(attn, L.o_proj.weight_km, self.pcomm, residual=x)
        else:
            part = ops.gemm(attn, L.o_proj.weight_km)
            self._all_reduce(part)
            x2 = torch.empty_like(x)
            h2 = ops.rmsnorm(part, mlp.post_norm_weight, mlp.eps, add=x, h_out=x2)
        if h2 is None and decode and self.fuse_norm:
            # decode: the post-attention RMSNorm runs inside the gate/up projection
            act = ops.gemm_norm(x2, mlp.post_norm_weight, mlp.gate_up_weight_il, mlp.eps,
                                "swiglu")
        else:
            if h2 is None:
                h2 = ops.rmsnorm(x2, mlp.post_norm_weight, mlp.eps)
            act = ops.gemm(h2, mlp.gate_up_weight_il, "swiglu")
        if self.tp_size == 1:
            return ops.gemm(act, mlp.down_weight_km, "residual", residual=x2), None
        if peer:
            return ops.gemm_ar(act, mlp.down_weight_km, self.comm, residual=x2), None
        if two_shot:
            return ops.gemm_allreduce(act, mlp.down_weight_km, self.pcomm, residual=x2), None
        part2 = ops.gemm(act, mlp.down_weight_km)
        self._all_reduce(part2)
        return x2, part2

    def forward_layer(self, hidden, layer_idx, kv_cache, start_pos, seq_len, position_ids=None):
        """model_fused.py:234-277.  position_ids [3, B, S] switches to M-RoPE."""
        B = hidden.shape[0]
        H = hidden.shape[-1]
        x = hidden.reshape(B * seq_len, H).contiguous()
        rope = self._mrope(position_ids) if position_ids is not None else None
        x, pend = self._layer(x, None, layer_idx, kv_cache, start_pos, seq_len, B, rope=rope)
        if pend is not None:
            x = ops.add(x, pend)
        return x.view(B, seq_len, H)

    def _mrope(self, position_ids):
        _, _, inv = self.rotary.tables(self.device)
        pos = position_ids.to(self.device, torch.int64)
        return ops.mrope_cos_sin(pos, inv)

    # vision_config.spatial_merge_size of the Qwen3-VL checkpoints
    spatial_merge_size = 2

    def get_rope_index(self, input_ids, mm_token_type_ids, image_grid_thw=None,
                       video_grid_thw=None, attention_mask=None, **kwargs):
        """Qwen3VLModel.get_rope_index (transformers 5.5.0
        modeling_qwen3_vl.py:1031-1122) on the device: returns position_ids
        int64 [3, B, S] for generate_with_embeds and the rope deltas int64
        [B, 1] (the decode steps' RoPE rows are cache position + delta)."""
        if tuple(mm_token_type_ids.shape) != tuple(input_ids.shape):
            raise ValueError("get_rope_index: mm_token_type_ids must match input_ids")
        return ops.rope_index(mm_token_type_ids.to(self.device), image_grid_thw, video_grid_thw,
                              attention_mask, spatial_merge_size=self.spatial_merge_size)

    # --------------------------------------------------------------- logits
    def _logits(self, x, pend, B, S, ss_valid=False):
        """Full-vocabulary logits [B, 1, V] (model_fused.py:286-292)."""
        local = self._local_logits(x, pend, B, S, ss_valid)
        if self.tp_size == 1:
            return local.view(B, 1, -1)
        return self._gather(local, B).view(B, 1, -1)

    def _greedy(self, x, pend, B, S, ss_valid=False, out=None):
        """Greedy next tokens int64 [B]: argmax of _logits (model_fused.py:310,320).
        At TP > 1 each rank reduces its vocabulary slice to one key per row and
        a MAX all-reduce of B int64 keys replaces the all_gather of the logits;
        the key orders by value, then by lower index (torch.argmax's ties)."""
        local = self._local_logits(x, pend, B, S, ss_valid)
        if self.tp_size == 1 or not self.dist_argmax:
            if self.tp_size > 1:
                local = self._gather(local, B)
            return ops.argmax(local.view(B, -1), out=out)
        keys = ops.argmax_key(local.view(B, -1), self._rank() * local.shape[-1])
        dist.all_reduce(keys, op=dist.ReduceOp.MAX)
        return ops.argmax_key_index(keys, out=out)

    def _gather(self, local, B):
        gathered = torch.empty(self.tp_size, B, local.shape[-1], dtype=local.dtype,
                               device=local.device)
        dist.all_gather_into_tensor(gathered, local)
        return gathered.permute(1, 0, 2).reshape(B, -1)

    def _rank(self):
        return dist.get_rank() if dist.is_initialized() else 0

    def _local_logits(self, x, pend, B, S, ss_valid=False):
        """This rank's vocabulary slice of the last position's logits [B, V/tp]."""
        H = x.shape[-1]
        if S > 1:
            x = x.view(B, S, H)[:, -1].contiguous()
            pend = pend.view(B, S, H)[:, -1].contiguous() if pend is not None else None
            ss_valid = False
        if pend is not None:
            h = ops.rmsnorm(pend, self.final_norm.weight, self.final_norm.eps, add=x)
            local = ops.gemm(h, self.lm_head.weight_km)       # [B, V/tp]
        elif B <= 16 and self.fuse_norm:
            # final norm fused into the lm_head projection
            ss = self._ss_buf(1) if ss_valid else None
            local = ops.gemm_decode(x, self.lm_head.weight_km, norm_w=self.final_norm.weight,
                                    eps=self.final_norm.eps, ss_in=ss, ss_tiles=H // 64)
        else:
            h = ops.rmsnorm(x, self.final_norm.weight, self.final_norm.eps)
            local = ops.gemm(h, self.lm_head.weight_km)
        return local

    def _embed(self, input_ids):
        table = self.embed_tokens.weight if hasattr(self.embed_tokens, "weight") \
            else self.embed_tokens
        return ops.embed(input_ids.to(self.device), table)

    def _run(self, hidden2d, B, S, start_pos, kv_cache, rope=None, deepstack=None,
             visual_mask=None, pos_dev=None, kv_len_dev=None, kv_bound=None, rope_delta=0):
        x, pend = hidden2d, None
        for i in range(self.num_layers):
            # layers after the first find their input norm's sums of squares
            # left by the previous layer's down projection (decode, TP1)
            x, pend = self._layer(x, pend, i, kv_cache, start_pos, S, B, rope=rope,
                                  pos_dev=pos_dev, kv_len_dev=kv_len_dev, kv_bound=kv_bound,
                                  rope_delta=rope_delta, ss_valid=i > 0)
            if deepstack is not None and i < len(deepstack):
                if pend is not None:
                    x = ops.add(x, pend)
                    pend = None
                x = self._deepstack_add(x, B, S, deepstack[i], visual_mask)
        return x, pend

    def _deepstack_add(self, x, B, S, feats, visual_mask):
        """Deepstack injection after an early layer (model_fused.py:339-341):
        hidden[visual positions] += feats.  A 1-D mask [S] addresses batch row 0,
        as the reference does; a [B, S] mask addresses every sequence, with the
        feature rows of all sequences concatenated in (row, position) order."""
        H = x.shape[-1]
        m = visual_mask.to(self.device)
        if m.dim() == 2 and m.shape != (B, S):
            raise ValueError(f"visual_mask must be [S] or [B, S]=[{B}, {S}], got {tuple(m.shape)}")
        flat = x.view(B * S, H)
        idx = torch.nonzero(m.reshape(-1)).flatten()   # row-0 positions for a 1-D mask
        if feats.shape[0] != idx.numel():
            raise ValueError(f"deepstack features: {feats.shape[0]} rows for {idx.numel()} "
                             "visual positions")
        rows = flat.index_select(0, idx).contiguous()
        upd = ops.add(rows, feats.to(self.device, torch.bfloat16).contiguous())
        flat.index_copy_(0, idx, upd)
        return x

    def forward(self, input_ids, start_pos, kv_cache, position_ids=None):
        """model_fused.py:279-293 -> logits [B, 1, V]."""
        B, S = input_ids.shape
        x = self._embed(input_ids).view(B * S, -1)
        rope = self._mrope(position_ids) if position_ids is not None else None
        x, pend = self._run(x, B, S, start_pos, kv_cache, rope=rope)
        return self._logits(x, pend, B, S, ss_valid=self._ss_ok(B, S))

    def prefill(self, input_ids, kv_cache):
        return self.forward(input_ids, start_pos=0, kv_cache=kv_cache)

    def decode_step(self, token_id, pos, kv_cache):
        return self.forward(token_id.view(-1, 1), start_pos=pos, kv_cache=kv_cache)

    # ------------------------------------------------------------- generate
    def _bucket(self, need: int) -> int:
        for b in KV_BUCKETS:
            if need <= b and b <= self.max_seq_len:
                return b
        return self.max_seq_len

    # ------------------------------------------------------ persistent step
    def _step_ok(self, B: int) -> bool:
        """The whole-step kernel covers TP1, head_dim 128, 4 query heads per KV
        head, no QKV bias, up to 16 sequences."""
        H = self.layers[0].attn_block.input_norm_weight.numel() if self.num_layers else 0
        return (self.use_step_kernel and self.tp_size == 1 and self.num_layers > 0 and
                1 <= B <= 16 and self.head_dim == 128 and H % 128 == 0 and
                self.num_q_heads == 4 * self.num_kv_heads and
                all(L.attn_block.qkv_bias is None for L in self.layers))

    def _step_plan(self, B, kv_cache):
        paged = isinstance(kv_cache[0], PagedLayer)
        key = (B, kv_cache[0][0].data_ptr(), kv_cache[0].table.data_ptr() if paged else 0)
        plan = self._step_plans.get(key)
        if plan is None:
            layers = []
            for L, (kc, vc) in zip(self.layers, kv_cache):
                ab, mlp = L.attn_block, L.mlp_block
                layers.append(dict(w_qkv=ab.qkv_weight_km, w_o=L.o_proj.weight_km,
                                   w_gate_up=mlp.gate_up_weight_il, w_down=mlp.down_weight_km,
                                   input_norm=ab.input_norm_weight, post_norm=mlp.post_norm_weight,
                                   q_norm=ab.q_norm_weight, k_norm=ab.k_norm_weight,
                                   k_cache=kc, v_cache=vc))
            cos, sin, _ = self.rotary.tables(self.device)
            mlp0 = self.layers[0].mlp_block
            plan = ops.DecodeStepPlan(
                layers, batch=B, hidden=self.layers[0].attn_block.input_norm_weight.numel(),
                q_heads=self.num_q_heads, kv_heads=self.num_kv_heads,
                inter=mlp0.down_weight_km.shape[1], max_seq=kv_cache[0][0].shape[2],
                eps=self._eps, cos=cos, sin=sin)
            self._step_plans[key] = plan
        return plan

    def _step_logits(self, B, tok, kv_cache, kv_len, rope_delta):
        """One decode step through q3_decode_step; the final RMSNorm runs inside
        the lm_head projection from the step's per-tile sums of squares."""
        plan = self._step_plan(B, kv_cache)
        H = plan.hidden
        if self._ss_step is None:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("step buffers must exist before graph capture")
            self._ss_step = torch.zeros(H // 128, 16, dtype=torch.float32, device=self.device)
        x = self._embed(tok.view(B, 1)).view(B, -1)
        plan.run(x, self._ss_step, kv_len, rope_delta)
        local = ops.gemm_decode(x, self.lm_head.weight_km, norm_w=self.final_norm.weight,
                                eps=self.final_norm.eps, ss_in=self._ss_step, ss_tiles=H // 128)
        return local.view(B, 1, -1)

    # ------------------------------------------- tensor-parallel step kernel
    def _tp_ok(self, B: int, kv_cache, rope_delta) -> bool:
        """The step kernel covers up to 8 sequences, head_dim 128, no QKV bias,
        contiguous caches or pages of a multiple of 64 tokens, and one RoPE
        delta for the batch; at TP > 1 it needs
        its communicator (enable_peer_allreduce with Q3VL_TP_KERNEL=1)."""
        paged_ok = (not isinstance(kv_cache[0], PagedLayer) or
                    kv_cache[0][0].shape[2] % 64 == 0)
        return (self.use_tp_kernel and self.num_layers > 0 and 1 <= B <= 8 and
                self.head_dim == 128 and paged_ok and
                not isinstance(rope_delta, RowRope) and
                all(L.attn_block.qkv_bias is None for L in self.layers) and
                (self.tp_size == 1 or self.mk_comm is not None))

    def _tp_plan(self, B, kv_cache):
        """The step kernel's plan for this batch and cache, or None when the
        library rejects the shapes (then the per-kernel step runs)."""
        paged = isinstance(kv_cache[0], PagedLayer)
        key = (B, kv_cache[0][0].data_ptr(), kv_cache[0].table.data_ptr() if paged else 0)
        if key in self._tp_plans:
            return self._tp_plans[key]
        if self.tp_size == 1 and self.mk_comm is None:
            from q3vl.comm import SoloComm
            H = self.layers[0].attn_block.input_norm_weight.numel()
            self.mk_comm = SoloComm(max_cols=H, device=self.device)
        layers = []
        for L, (kc, vc) in zip(self.layers, kv_cache):
            ab, mlp = L.attn_block, L.mlp_block
            layers.append(dict(w_qkv=ab.qkv_weight_km, w_o=L.o_proj.weight_km,
                               w_gate_up=mlp.gate_up_weight_il, w_down=mlp.down_weight_km,
                               input_norm=ab.input_norm_weight, post_norm=mlp.post_norm_weight,
                               q_norm=ab.q_norm_weight, k_norm=ab.k_norm_weight,
                               k_cache=kc, v_cache=vc))
        cos, sin, _ = self.rotary.tables(self.device)
        mlp0 = self.layers[0].mlp_block
        try:
            plan = ops.DecodeTPPlan(
                layers, batch=B, hidden=self.layers[0].attn_block.input_norm_weight.numel(),
                q_heads=self.num_q_heads, kv_heads=self.num_kv_heads,
                inter=mlp0.down_weight_km.shape[1],
                max_seq=(kv_cache[0].table.shape[1] * kv_cache[0][0].shape[2] if paged
                         else kv_cache[0][0].shape[2]),
                eps=self._eps, cos=cos, sin=sin, comm=self.mk_comm,
                block_table=kv_cache[0].table if paged else None)
        except Q3Error:
            plan = None
        self._tp_plans[key] = plan
        return plan

    def _capture_decode(self, B, kv_cache, bucket, rope_delta=0):
        """Capture one decode step.  Must run before the prefill that fills this
        cache: the warm-up step writes KV slot 0, which the prefill overwrites."""
        key = (B, bucket, kv_cache[0][0].data_ptr(),
               ("rows", rope_delta.cos.data_ptr()) if isinstance(rope_delta, RowRope)
               else rope_delta)
        g = self._graphs.get(key)
        if g is not None:
            return g
        dev = self.device
        tok = torch.zeros(B, dtype=torch.int64, device=dev)
        pos = torch.zeros(1, dtype=torch.int32, device=dev)
        kv_len = torch.ones(1, dtype=torch.int32, device=dev)
        ops.decode_workspace(B, self.num_q_heads, self.num_kv_heads, dev)

        use_step = (self._step_ok(B) and not isinstance(kv_cache[0], PagedLayer) and
                    not isinstance(rope_delta, RowRope))
        tp_plan = self._tp_plan(B, kv_cache) if self._tp_ok(B, kv_cache, rope_delta) else None

        def step():
            """One decode step; the next tokens land in `tok` (read at the start)."""
            if tp_plan is not None:
                x = self._embed(tok.view(B, 1)).view(B, -1)
                tp_plan.run(x, kv_len, int(rope_delta))
                return self._greedy(x, None, B, 1, out=tok)
            if use_step:
                logits = self._step_logits(B, tok, kv_cache, kv_len, rope_delta)
                return ops.argmax(logits.view(B, -1), out=tok)
            x = self._embed(tok.view(B, 1)).view(B, -1)
            x, pend = self._run(x, B, 1, 0, kv_cache, pos_dev=pos, kv_len_dev=kv_len,
                                kv_bound=bucket, rope_delta=rope_delta)
            return self._greedy(x, pend, B, 1, ss_valid=self._ss_ok(B, 1), out=tok)

        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            step()                                  # warm up allocator + tensor maps
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        multi, hist = None, None
        steps = self.graph_steps
        if steps > 1:
            hist = torch.zeros(steps, B, dtype=torch.int64, device=dev)
            multi = torch.cuda.CUDAGraph()
            with torch.cuda.graph(multi):
                for j in range(steps):
                    step()
                    hist[j].copy_(tok)
                    pos.add_(1)
                    kv_len.add_(1)
        g = _DecodeGraph(graph, tok, pos, kv_len, multi, hist, steps if multi is not None else 1)
        self._graphs[key] = g
        return g

    def _decode_rope(self, rope_delta, B, bucket):
        """An int delta as is; per-sequence deltas (a tensor or list of B, as
        get_rope_index returns them) as one int when they agree, else as
        RowRope tables kept per (batch, bucket) so captured graphs read the
        current rows."""
        if isinstance(rope_delta, (int, RowRope)):
            return rope_delta
        d = [int(v) for v in torch.as_tensor(rope_delta).reshape(-1).tolist()]
        if len(d) != B:
            raise ValueError(f"{len(d)} rope deltas for a batch of {B}")
        if all(v == d[0] for v in d):
            return d[0]
        inv = self.rotary.inv_freq
        t = (torch.arange(bucket)[None, :] + torch.tensor(d)[:, None]).reshape(-1).float()
        freqs = torch.outer(t, inv)
        cos, sin = freqs.cos().to(torch.bfloat16), freqs.sin().to(torch.bfloat16)
        key = (B, bucket)
        rr = self._row_ropes.get(key)
        if rr is None:
            rr = RowRope(torch.empty_like(cos, device=self.device),
                         torch.empty_like(sin, device=self.device), bucket)
            self._row_ropes[key] = rr
        rr.cos.copy_(cos)
        rr.sin.copy_(sin)
        return rr

    def _paged_kv(self, pool: KVPagePool, B, bucket, slots=None):
        """Per-layer PagedLayer views of `pool` for a batch: every slot grows to
        cover the bucket, and the block table goes into a device tensor kept per
        (pool, batch) so that captured decode graphs read its current rows."""
        if len(pool.k) != self.num_layers:
            raise ValueError(f"page pool holds {len(pool.k)} layers, the decoder {self.num_layers}")
        slots = list(range(B)) if slots is None else [int(sl) for sl in slots]
        if len(slots) != B:
            raise ValueError(f"{len(slots)} slots for a batch of {B}")
        if pool.max_pages_per_seq * pool.page_tokens < bucket:
            raise ValueError(f"page pool covers {pool.max_pages_per_seq * pool.page_tokens} "
                             f"positions per sequence, the KV bucket is {bucket}")
        for sl in slots:
            pool.reserve(sl, bucket)
        key = (id(pool), B)
        table = self._page_tables.get(key)
        if table is None:
            table = torch.empty(B, pool.max_pages_per_seq, dtype=torch.int32, device=self.device)
            self._page_tables[key] = table
        pool.device_table(slots, out=table)
        return pool.layers(table)

    def _kv_for(self, B, bucket):
        key = (B, bucket)
        kv = self._kv_pool.get(key)
        if kv is None:
            kv = []
            for _ in range(self.num_layers):
                k = torch.zeros(B, self.num_kv_heads, bucket, self.head_dim,
                                dtype=torch.bfloat16, device=self.device)
                kv.append((k, torch.zeros_like(k)))
            self._kv_pool[key] = kv
        return kv

    @torch.no_grad()
    def generate_tokens(self, input_ids=None, max_new_tokens=256, eos_token_id=151645,
                        inputs_embeds=None, position_ids=None, deepstack_embeds=None,
                        visual_mask=None, rope_delta=0, eos_check_every=32,
                        prefill_done=None, kv_pages: KVPagePool = None, slots=None,
                        health=None):
        """Batched greedy generation with a device-resident decode loop.

        Returns int64 [B, T] (T <= max_new_tokens): generation stops once every row
        has produced EOS; rows that stop early keep producing tokens after their
        EOS, which callers cut (see generate).  `prefill_done` (a CUDA event) is
        recorded on the current stream between prefill and decode.

        With `kv_pages` (a KVPagePool holding this decoder's layers), the KV
        cache lives in that pool's pages: row b uses slot slots[b] (default b),
        which is grown to the KV bucket here and left to the caller to release.

        With `health` (a q3vl.health.RankHealth), every eos_check_every decode
        steps each rank records its progress and waits (bounded) for its peers
        before launching more steps, so a dead peer raises RankFailure on the
        host instead of being met by the kernels' bounded waits."""
        if inputs_embeds is not None:
            B, P, _ = inputs_embeds.shape
        else:
            B, P = input_ids.shape
        need = P + max_new_tokens
        if need > self.max_seq_len:
            raise ValueError(f"prompt {P} + {max_new_tokens} new tokens exceeds max_seq_len "
                             f"{self.max_seq_len}")
        bucket = self._bucket(need)
        rope_delta = self._decode_rope(rope_delta, B, bucket)
        if kv_pages is not None:
            kv = self._paged_kv(kv_pages, B, bucket, slots)
        else:
            kv = self._kv_for(B, bucket)
        g = None
        if self.use_graphs and max_new_tokens > 1:
            g = self._capture_decode(B, kv, bucket, rope_delta)
        if inputs_embeds is not None:
            x = inputs_embeds.to(self.device, torch.bfloat16).reshape(B * P, -1).contiguous()
        else:
            x = self._embed(input_ids).view(B * P, -1)
        rope = self._mrope(position_ids) if position_ids is not None else None
        x, pend = self._run(x, B, P, 0, kv, rope=rope, deepstack=deepstack_embeds,
                            visual_mask=visual_mask)
        out = torch.empty(B, max_new_tokens, dtype=torch.int64, device=self.device)
        out[:, 0] = self._greedy(x, pend, B, P)
        if prefill_done is not None:
            prefill_done.record(torch.cuda.current_stream(self.device))
        if max_new_tokens == 1:
            return out
        # cache positions continue at P; RoPE rows at P + rope_delta (M-RoPE text)
        if g is not None:
            g.tok.copy_(out[:, 0])
            g.pos.fill_(P)
            g.kv_len.fill_(P + 1)
            done_at = max_new_tokens
            i = 1                                   # tokens 0 .. i-1 are in `out`
            next_check = 1 + eos_check_every
            while i < max_new_tokens:
                if g.multi is not None and max_new_tokens - i >= g.steps:
                    g.multi.replay()                # steps tokens, counters advanced inside
                    out[:, i:i + g.steps].copy_(g.hist.t())
                    i += g.steps
                else:
                    g.graph.replay()
                    out[:, i].copy_(g.tok)
                    g.pos.add_(1)
                    g.kv_len.add_(1)
                    i += 1
                if i >= next_check:
                    next_check = i + eos_check_every
                    if health is not None:
                        torch.cuda.current_stream(self.device).synchronize()
                        health.wait_for_peers(health.tick())
                    if eos_token_id is not None and \
                            bool((out[:, :i] == eos_token_id).any(dim=1).all()):
                        done_at = i
                        break
            return out[:, :done_at]
        tok = out[:, 0]
        for i in range(1, max_new_tokens):
            pos = P + i - 1
            x = self._embed(tok.view(B, 1)).view(B, -1)
            x, pend = self._run(x, B, 1, pos, kv, rope_delta=rope_delta)
            tok = self._greedy(x, pend, B, 1, ss_valid=self._ss_ok(B, 1))
            out[:, i] = tok
        return out

    @staticmethod
    def _cut_at_eos(row, eos):
        toks = []
        for t in row:
            if t == eos:
                break
            toks.append(t)
        return toks

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens=256, eos_token_id=151645, verbose=False):
        """model_fused.py:302-328: greedy, returns list[int] for batch 1 (a list
        of lists for batch > 1).  The first token is always kept; later tokens
        stop before the first EOS, as in the reference."""
        t0 = time.time()
        toks = self.generate_tokens(input_ids, max_new_tokens, eos_token_id).tolist()
        if verbose and (not dist.is_initialized() or dist.get_rank() == 0):
            print(f"    generate: {time.time() - t0:.3f}s for {len(toks[0])} tokens")
        rows = [[r[0]] + self._cut_at_eos(r[1:], eos_token_id) for r in toks]
        return rows[0] if len(rows) == 1 else rows

    @torch.no_grad()
    def generate_with_embeds(self, inputs_embeds, max_new_tokens=256, eos_token_id=151645,
                             deepstack_embeds=None, visual_mask=None, position_ids=None,
                             rope_delta=0):
        """model_fused.py:330-362 (+ optional 3-axis M-RoPE position_ids, and a
        rope delta that is one int or one per sequence, as get_rope_index
        returns them)."""
        toks = self.generate_tokens(None, max_new_tokens, eos_token_id,
                                    inputs_embeds=inputs_embeds, position_ids=position_ids,
                                    deepstack_embeds=deepstack_embeds, visual_mask=visual_mask,
                                    rope_delta=rope_delta).tolist()
        rows = [[r[0]] + self._cut_at_eos(r[1:], eos_token_id) for r in toks]
        return rows[0] if len(rows) == 1 else rows
