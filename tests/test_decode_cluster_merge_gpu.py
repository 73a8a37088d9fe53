"""Decode attention's split merge inside a thread-block cluster (2-8 splits of
one (sequence, KV head) merged by cluster rank 0 through distributed shared
memory) against the workspace + combine-kernel merge and an fp32 torch
reference of model_fused.py:252-262 at S = 1.  The split count comes from the
plan (about one CTA per SM over B x Hkv pairs), so the shapes below give 2,
4, 6, 7 and 8 splits on 148 SMs; past 8 (B = 1 here) a cluster would exceed
the portable size and the combine kernel stays in both modes.  The cluster
merge is opt-in (Q3VL_DECODE_CLUSTER_MERGE=1): it measured slower than the
combine kernel on B200."""
import os

import pytest
import torch

from q3vl import _lib, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _ref(q, kc, vc, L):
    B, Hq, D = q.shape
    G = Hq // kc.shape[1]
    k = kc[:, :, :L].float().repeat_interleave(G, 1)
    v = vc[:, :, :L].float().repeat_interleave(G, 1)
    s = (q.float().unsqueeze(2) @ k.transpose(-1, -2)) / D ** 0.5
    return (torch.softmax(s, -1) @ v).squeeze(2)


def _planned_splits(pairs, bound):
    """The host plan of the tensor-core kernel: about one CTA per SM over the
    pairs, chunks in whole 64-position tiles (attn_decode.cu)."""
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    sp = max(1, min(sms // pairs, (bound + 63) // 64))
    ch = -(-bound // sp)
    ch = -(-ch // 64) * 64
    return -(-bound // ch)


def test_plan_gives_the_split_counts_the_cases_name():
    assert [_planned_splits(p, 2048) for p in (64, 32, 24, 20, 16, 8)] == [2, 4, 6, 7, 8, 16]


def _run(mode, fn):
    old = os.environ.get("Q3VL_DECODE_CLUSTER_MERGE")
    os.environ["Q3VL_DECODE_CLUSTER_MERGE"] = mode
    try:
        n0 = _lib.raw("q3_launch_count")()
        out = fn()
        torch.cuda.synchronize()
        return out, _lib.raw("q3_launch_count")() - n0
    finally:
        if old is None:
            del os.environ["Q3VL_DECODE_CLUSTER_MERGE"]
        else:
            os.environ["Q3VL_DECODE_CLUSTER_MERGE"] = old


@pytest.mark.parametrize("B,Hq,Hkv,L", [(8, 32, 8, 1152), (4, 32, 8, 1000), (3, 32, 8, 777),
                                        (5, 16, 4, 2047), (8, 32, 8, 65), (2, 32, 8, 1500),
                                        (1, 32, 8, 1999)])
def test_cluster_merge_matches_combine_and_reference(B, Hq, Hkv, L):
    g = torch.Generator(device=DEV).manual_seed(B * 1000 + L)
    S = 2048
    q = torch.randn(B, Hq, 128, device=DEV, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, S, 128, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, 128, device=DEV, generator=g).to(torch.bfloat16)
    Ld = torch.tensor([L], dtype=torch.int32, device=DEV)
    fn = lambda: ops.attn_decode(q, kc, vc, kv_len=S, kv_len_dev=Ld)  # noqa: E731
    a, na = _run("1", fn)
    b, nb = _run("0", fn)
    ref = _ref(q, kc, vc, L)
    for name, o in (("cluster", a), ("combine", b)):
        err = (o.float() - ref).abs().max().item()
        assert err < 2e-2, (name, err)
    # the two merges differ only in fp32 rounding of the rescale factors
    assert (a.float() - b.float()).abs().max().item() < 1e-2
    if 1 < _planned_splits(B * Hkv, S) <= 8:
        assert (na, nb) == (1, 2), (na, nb)   # no combine kernel in cluster mode
    else:
        assert na == nb


def test_cluster_merge_paged_matches_contiguous():
    B, Hq, Hkv, L, page = 8, 32, 8, 1152, 256
    g = torch.Generator(device=DEV).manual_seed(7)
    S = 2048
    q = torch.randn(B, Hq, 128, device=DEV, generator=g).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, S, 128, device=DEV, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, S, 128, device=DEV, generator=g).to(torch.bfloat16)
    per = S // page
    perm = torch.randperm(B * per, generator=torch.Generator().manual_seed(3)).to(DEV)
    table = perm.view(B, per).to(torch.int32)
    kp = torch.zeros(B * per, Hkv, page, 128, dtype=torch.bfloat16, device=DEV)
    vp = torch.zeros_like(kp)
    for b in range(B):
        for j in range(per):
            kp[table[b, j]] = kc[b, :, j * page:(j + 1) * page]
            vp[table[b, j]] = vc[b, :, j * page:(j + 1) * page]
    Ld = torch.tensor([L], dtype=torch.int32, device=DEV)
    a, na = _run("1", lambda: ops.attn_decode_paged(q, kp, vp, table, kv_len=S, kv_len_dev=Ld))
    b, _ = _run("1", lambda: ops.attn_decode(q, kc, vc, kv_len=S, kv_len_dev=Ld))
    assert na == 1
    assert torch.equal(a, b)   # same kernel arithmetic, rows read through the table
    assert (a.float() - _ref(q, kc, vc, L)).abs().max().item() < 2e-2
