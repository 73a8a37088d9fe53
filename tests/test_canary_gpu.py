"""Unwritten outputs and stray writes, at ragged shapes.

Every output is a contiguous view inside a buffer poisoned with NaN (int64
outputs: a sentinel), with a guard region before and after it.  After the
call the whole view must be written (finite) and both guards untouched.
Caches start filled with finite stale values: a cache write must change only
its own rows.  Shapes are deliberately off the tile sizes (1, 3, 17, 63, 65,
129, ...)."""
import math

import pytest
import torch

from q3vl import ops
from tests.helpers import compare

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF16 = torch.bfloat16
SENTINEL = -0x5A5A5A5A


class Canvas:
    def __init__(self, shape, dtype=BF16, guard=4096):
        self.n = math.prod(shape)
        self.guard = guard
        fill = float("nan") if dtype.is_floating_point else SENTINEL
        self.buf = torch.full((guard + self.n + guard,), fill, dtype=dtype, device=DEV)
        self.view = self.buf[guard:guard + self.n].view(shape)

    def check(self, name):
        head, tail = self.buf[:self.guard], self.buf[self.guard + self.n:]
        if self.buf.dtype.is_floating_point:
            assert torch.isnan(head).all() and torch.isnan(tail).all(), f"{name}: stray write"
            assert torch.isfinite(self.view).all(), f"{name}: part of the output unwritten"
        else:
            assert (head == SENTINEL).all() and (tail == SENTINEL).all(), f"{name}: stray write"
            assert (self.view != SENTINEL).all(), f"{name}: part of the output unwritten"


def rnd(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(BF16).to(DEV)


@pytest.mark.parametrize("rows", [1, 3, 17, 129])
def test_rmsnorm(rows):
    x, a, w = rnd(rows, 4096, seed=1), rnd(rows, 4096, seed=2), rnd(4096, seed=3) + 1
    out, h = Canvas((rows, 4096)), Canvas((rows, 4096))
    ops.rmsnorm(x, w, 1e-6, add=a, h_out=h.view, out=out.view)
    out.check("rmsnorm out")
    h.check("rmsnorm h_out")
    hf = (x.float() + a.float()).to(BF16).float()
    ref = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(BF16).float() * w.float()
    compare("rmsnorm", out.view.float(), ref, max_abs=3e-2, rel_scale=True, min_cos=0.9999)


@pytest.mark.parametrize("M,N,K", [(1, 48, 96), (5, 272, 4096), (17, 272, 96), (129, 4096, 512),
                                   (300, 48, 4096)])
@pytest.mark.parametrize("epi", ["none", "residual", "swiglu"])
def test_gemm(M, N, K, epi):
    x, w = rnd(M, K, seed=4), rnd(N, K, seed=5, scale=0.05)
    r = rnd(M, N, seed=6) if epi == "residual" else None
    n_out = N // 2 if epi == "swiglu" else N
    out = Canvas((M, n_out))
    ops.gemm(x, w, epi, residual=r, out=out.view)
    out.check(f"gemm {epi}")
    acc = x.float() @ w.float().t()
    if epi == "residual":
        ref = r.float() + acc.to(BF16).float()
    elif epi == "swiglu":
        gu = acc.view(M, N // 16, 2, 8)
        ref = (torch.nn.functional.silu(gu[:, :, 0]) * gu[:, :, 1]).reshape(M, n_out)
    else:
        ref = acc
    compare(f"gemm {epi}", out.view.float(), ref, max_abs=3e-2, rel_scale=True, min_cos=0.999)


@pytest.mark.parametrize("M,N", [(1, 4096), (7, 1088), (16, 4160)])
def test_gemm_decode_sums_of_squares(M, N):
    K = 4096
    x, w, r = rnd(M, K, seed=7), rnd(N, K, seed=8, scale=0.02), rnd(M, N, seed=9)
    # the residual projections (o_proj, down) emit the sums of squares the
    # next RMSNorm needs; a normalising projection cannot also emit them
    out = Canvas((M, N))
    ss = Canvas(((N + 63) // 64, 16), dtype=torch.float32)
    ops.gemm_decode(x, w, "residual", residual=r, ss_out=ss.view, out=out.view)
    out.check("gemm_decode out")
    # only the first M token columns of each tile's 16 carry sums; the rest are
    # written as zeros
    ss.check("gemm_decode ss_out")
    want = out.view.float().pow(2).view(M, -1, 64).sum(-1).t()
    compare("sums of squares", ss.view[:, :M], want, max_abs=1e-3, rel_scale=True)


@pytest.mark.parametrize("L", [1, 63, 64, 65, 1000])
@pytest.mark.parametrize("dtype", [torch.float32, BF16])
def test_attn_decode(L, dtype):
    B, Hq, Hkv, max_seq = 3, 8, 2, 1024
    q = rnd(B, Hq, 128, seed=11).to(dtype)
    k = rnd(B, Hkv, max_seq, 128, seed=12).to(dtype)
    v = rnd(B, Hkv, max_seq, 128, seed=13).to(dtype)
    out = Canvas((B, Hq, 128), dtype=dtype)
    ops.attn_decode(q, k, v, kv_len=L, out=out.view)
    out.check("attn_decode")
    kk = k[:, :, :L].float().repeat_interleave(Hq // Hkv, 1)
    vv = v[:, :, :L].float().repeat_interleave(Hq // Hkv, 1)
    p = torch.softmax((q.float()[:, :, None] @ kk.transpose(-2, -1)) / math.sqrt(128), -1)
    ref = (p @ vv)[:, :, 0]
    compare("attn_decode", out.view.float(), ref, max_abs=2e-2, min_cos=0.9999)


@pytest.mark.parametrize("S,start", [(1, 0), (127, 0), (129, 37), (200, 0)])
def test_attn_prefill(S, start):
    B, Hq, Hkv = 2, 8, 2
    rows = start + S
    q = rnd(B, Hq, S, 128, seed=14)
    k, v = rnd(B, Hkv, rows, 128, seed=15), rnd(B, Hkv, rows, 128, seed=16)
    out = Canvas((B, Hq, S, 128))
    ops.attn_prefill(q, k, v, start_pos=start, out=out.view)
    out.check("attn_prefill")


def test_qkv_norm_rope_writes_only_its_cache_rows():
    B, S, Hq, Hkv, start, max_seq = 2, 5, 8, 2, 13, 64
    qkv = rnd(B * S, (Hq + 2 * Hkv) * 128, seed=17)
    kc, vc = rnd(B, Hkv, max_seq, 128, seed=18), rnd(B, Hkv, max_seq, 128, seed=19)
    k0, v0 = kc.clone(), vc.clone()
    t = torch.arange(max_seq, dtype=torch.float32)
    inv = 1.0 / (5e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    f = torch.outer(t, inv)
    cos, sin = f.cos().to(BF16).to(DEV), f.sin().to(BF16).to(DEV)
    ones = torch.ones(128, dtype=BF16, device=DEV)
    q, _, _ = ops.qkv_norm_rope(qkv, ones, ones, cos, sin, B=B, S=S, Hq=Hq, Hkv=Hkv,
                                start_pos=start, k_cache=kc, v_cache=vc)
    assert torch.isfinite(q.float()).all()
    inside = torch.zeros(max_seq, dtype=torch.bool, device=DEV)
    inside[start:start + S] = True
    for name, c, c0 in (("k", kc, k0), ("v", vc, v0)):
        assert torch.equal(c[:, :, ~inside], c0[:, :, ~inside]), f"{name} cache: stray write"
        assert not torch.equal(c[:, :, inside], c0[:, :, inside]), f"{name} cache: not written"
    # v rows are the projection's v columns, unchanged
    vq = qkv.view(B, S, Hq + 2 * Hkv, 128)[:, :, Hq + Hkv:].transpose(1, 2)
    assert torch.equal(vc[:, :, start:start + S], vq)


@pytest.mark.parametrize("n", [1, 13, 129])
def test_embed_argmax_add(n):
    V, H = 1000, 4096
    table = rnd(V, H, seed=20)
    ids = torch.randint(0, V, (n,), generator=torch.Generator().manual_seed(n)).to(DEV)
    out = Canvas((n, H))
    ops.embed(ids, table, out=out.view)
    out.check("embed")
    assert torch.equal(out.view, table[ids])
    logits = rnd(n, 18992, seed=21)
    idx = Canvas((n,), dtype=torch.int64)
    ops.argmax(logits, out=idx.view)
    idx.check("argmax")
    assert torch.equal(idx.view.cpu(), logits.float().cpu().argmax(-1))
    a, b = rnd(n, 24, seed=22), rnd(n, 24, seed=23)
    s = Canvas((n, 24))
    ops.add(a, b, out=s.view)
    s.check("add")
    assert torch.equal(s.view, (a.float() + b.float()).to(BF16))
