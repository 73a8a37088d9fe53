"""The arithmetic of the tcgen05 prefill attention kernels (csrc/attn_prefill_tc.cu),
restated in torch tile by tile, against fp32 attention at the tolerance of
the GPU parity tests (max-abs <= 2e-2, cosine >= 0.9999).

Variant 0: per 64-key tile, P = exp2(x - m_new) in bf16 with the running
maximum moved every tile, O_j = P V_j accumulated in fp32 and folded into the
output as o = o * exp2(m_old - m_new) + O_j.  Variant 1: P relative to a base
that moves only when a row's maximum exceeds it by more than 8 (log2 units),
so P <= 256; O accumulates across tiles and is scaled by exp2(base_old -
base_new) only when the base moves.  Both sum l from the unrounded P.  This
checks the scheme, not the kernels; the kernels' own parity tests run on the
GPU.  CPU only."""
import math

import pytest
import torch

BF16 = torch.bfloat16
LOG2E = 1.4426950408889634


def flash(q, k, v, variant, causal=True, start=0, tile=64, threshold=8.0):
    """q [S, D], k/v [L, D] (bf16) -> [S, D] fp32, one head."""
    S, D = q.shape
    L = k.shape[0]
    qf, kf, vf = q.float(), k.float(), v.float()
    m = torch.full((S,), -math.inf)
    l = torch.zeros(S)
    o = torch.zeros(S, D)
    qpos = start + torch.arange(S)
    for j in range(0, L, tile):
        s = (qf @ kf[j:j + tile].t()) * (LOG2E / math.sqrt(D))
        keys = j + torch.arange(s.shape[1])
        if causal:
            s = s.masked_fill(keys[None, :] > qpos[:, None], -math.inf)
        mx = s.max(dim=1).values
        if variant == 0:
            m_new = torch.maximum(m, mx)
            base = torch.where(m_new == -math.inf, torch.zeros_like(m_new), m_new)
            corr = torch.exp2(m - base)
            p = torch.exp2(s - base[:, None])
            o_j = p.to(BF16).float() @ vf[j:j + tile]
            o = o * corr[:, None] + o_j
            l = l * corr + p.sum(1)
            m = m_new
        else:
            m_new = torch.maximum(m, mx)
            move = m_new > m + threshold
            corr = torch.where(move, torch.exp2(m - m_new), torch.ones_like(m))
            corr = torch.where(torch.isnan(corr), torch.zeros_like(corr), corr)
            o = o * corr[:, None]
            l = l * corr
            m = torch.where(move, m_new, m)
            base = torch.where(m == -math.inf, torch.zeros_like(m), m)
            p = torch.exp2(s - base[:, None])
            assert float(p.max()) <= 2.0 ** threshold * (1 + 1e-6)
            o = o + p.to(BF16).float() @ vf[j:j + tile]
            l = l + p.sum(1)
    return o / l[:, None]


def fp32_attention(q, k, v, causal=True, start=0):
    s = (q.float() @ k.float().t()) / math.sqrt(q.shape[1])
    if causal:
        S, L = s.shape
        s = s.masked_fill(torch.arange(L)[None, :] > (start + torch.arange(S))[:, None],
                          -math.inf)
    return torch.softmax(s, -1) @ v.float()


def check(got, want):
    diff = (got - want).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.flatten().double(),
                                                want.flatten().double(), dim=0).item()
    assert diff <= 2e-2 and cos >= 0.9999, (diff, cos)


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("S,start,causal", [(200, 0, True), (130, 70, True), (96, 0, False),
                                            (1, 37, True)])
def test_tile_scheme_matches_fp32(variant, S, start, causal):
    g = torch.Generator().manual_seed(S + start)
    L = start + S
    q = torch.randn(S, 128, generator=g).to(BF16)
    k = torch.randn(L, 128, generator=g).to(BF16)
    v = torch.randn(L, 128, generator=g).to(BF16)
    check(flash(q, k, v, variant, causal, start), fp32_attention(q, k, v, causal, start))


def test_lazy_rescale_on_growing_scores():
    """Scores growing along the keys (the GPU test's construction) move the
    base many times; the lazily rescaled sum still matches fp32."""
    S = 640
    g = torch.Generator().manual_seed(36)
    q = torch.randn(S, 128, generator=g)
    k = torch.randn(S, 128, generator=g) * 0.2
    d = q.mean(0)
    k = k + (torch.arange(S, dtype=torch.float32) / 4.0)[:, None] * d / d.norm()
    v = torch.randn(S, 128, generator=g)
    q, k, v = q.to(BF16), k.to(BF16), v.to(BF16)
    want = fp32_attention(q, k, v)
    check(flash(q, k, v, 1), want)
    check(flash(q, k, v, 0), want)
