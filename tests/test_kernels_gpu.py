"""Kernel parity: the CUDA path (through the C ABI) vs the CPU oracle and the
golden fixtures made from the reference.  Tolerances are stated per test:
bf16 outputs are compared by max-abs and cosine; the fp32 decode attention of
config 1 by max-abs <= 1e-5."""
import math

import pytest
import torch

from oracle import ref as oref
from q3vl import layout, ops
from tests.golden import cases
from tests.helpers import as_tensor, compare, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF16 = torch.bfloat16


def rnd(*shape, seed=0, dtype=BF16, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(dtype)


# --------------------------------------------------------------------------- a1
@pytest.mark.parametrize("rows,hidden", [(1, 4096), (37, 4096), (8, 2048), (5, 520), (3, 1024)])
def test_rmsnorm(rows, hidden):
    x, w = rnd(rows, hidden, seed=1), (1 + rnd(hidden, seed=2, std=0.1)).to(BF16)
    y = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6).cpu()
    compare("rmsnorm", y, oref.rmsnorm(x, w), max_abs=1.6e-2, min_cos=0.99999)
    mism = (y.view(torch.int16) != oref.rmsnorm(x, w).view(torch.int16)).float().mean().item()
    assert mism < 1e-3, f"rmsnorm: {mism:.4%} of elements differ from the oracle bit pattern"


def test_rmsnorm_fused_residual():
    x, a = rnd(9, 4096, seed=3), rnd(9, 4096, seed=4)
    w = (1 + rnd(4096, seed=5, std=0.1)).to(BF16)
    h = torch.empty(9, 4096, dtype=BF16, device=DEV)
    y = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6, add=a.to(DEV), h_out=h)
    assert torch.equal(h.cpu(), x + a)
    compare("add+rmsnorm", y.cpu(), oref.rmsnorm(x + a, w), max_abs=1.6e-2, min_cos=0.99999)


# --------------------------------------------------------------------------- a9
def test_rope_kat_bit_exact():
    """kernels/rope.py semantics on the reference test's seed-42 inputs (S=256, N=4)."""
    g = load_golden("kernels_kat")
    x, cos, sin, *_ = cases.kernels_kat_inputs()
    cs = torch.cat([cos, sin], dim=-1).float()
    out = ops.rope(x.to(DEV), cs.to(DEV)).cpu()
    assert torch.equal(out, as_tensor(g["rope"]))


# --------------------------------------------------------------------------- a4
def test_mrope_tables_config2():
    pos = oref.config2_position_ids()             # [3, 1, 2048]
    inv = oref.inv_freq(128, 5e6)
    cos, sin = ops.mrope_cos_sin(pos.to(DEV), inv.to(DEV))
    f = oref.mrope_freqs(pos, inv)[0]             # [2048, 64] fp32 angles
    compare("mrope cos", cos.cpu(), f.cos(), max_abs=2e-6)
    compare("mrope sin", sin.cpu(), f.sin(), max_abs=2e-6)
    g = load_golden("mrope_cfg2")                 # HF tables (bf16) for the first 512 rows
    compare("mrope vs HF", cos[:cases.MROPE_ROWS].cpu().to(BF16), as_tensor(g["cos"]),
            max_abs=8e-3)


# --------------------------------------------------------------------------- a3 epilogue
def _attn_block_qkv(c):
    h = oref.rmsnorm(c["hidden"], c["in_norm"])
    return h @ c["qkv_w"]                         # bf16 [B, S, (Hq+2Hkv)*D]


def test_qkv_norm_rope_matches_reference_attention_block():
    """Epilogue on the reference AttentionBlock's own QKV product (1-D bf16 tables)."""
    g = load_golden("attn_block")
    c = cases.attn_block_case()
    qkv = _attn_block_qkv(c)
    cos, sin = oref.rotary_tables(128, c["max_seq"], 5e6)
    B, S, Hq, Hkv = c["B"], c["S"], c["Hq"], c["Hkv"]
    kc = torch.zeros(B, Hkv, c["max_seq"], 128, dtype=BF16, device=DEV)
    vc = torch.zeros_like(kc)
    q, k, v = ops.qkv_norm_rope(qkv.to(DEV).contiguous(), c["q_norm"].to(DEV),
                                c["k_norm"].to(DEV), cos.to(DEV), sin.to(DEV), B=B, S=S,
                                Hq=Hq, Hkv=Hkv, start_pos=c["start"], k_cache=kc, v_cache=vc,
                                want_kv=True)
    for name, got in (("q", q), ("k", k), ("v", v)):
        want = as_tensor(g[name])
        compare(f"qkv epilogue {name}", got.cpu(), want, max_abs=3.2e-2, min_cos=0.99999)
        mism = (got.cpu().view(torch.int16) != want.view(torch.int16)).float().mean().item()
        assert mism < 2e-3, f"{name}: {mism:.4%} differ bitwise from the reference"
    st = c["start"]
    assert torch.equal(kc[:, :, st:st + S].cpu(), k.cpu())
    assert torch.equal(vc[:, :, st:st + S].cpu(), v.cpu())
    assert kc[:, :, :st].abs().sum().item() == 0 and kc[:, :, st + S:].abs().sum().item() == 0


def test_qkv_norm_rope_device_position_and_mrope():
    c = cases.attn_block_case()
    qkv = _attn_block_qkv(c)
    B, S, Hq, Hkv = c["B"], c["S"], c["Hq"], c["Hkv"]
    # per-token f32 M-RoPE rows (b-stride S), positions from the config-2 layout
    pos = oref.config2_position_ids(seq=S + 100)[:, :, 100:100 + S].expand(3, B, S)
    inv = oref.inv_freq(128, 5e6)
    cosf, sinf = ops.mrope_cos_sin(pos.contiguous().to(DEV), inv.to(DEV))
    q, k, v = ops.qkv_norm_rope(qkv.to(DEV).contiguous(), c["q_norm"].to(DEV),
                                c["k_norm"].to(DEV), cosf, sinf, B=B, S=S, Hq=Hq, Hkv=Hkv,
                                cs_use_pos=False, cs_stride_b=S, want_kv=True)
    hc, hs = oref.mrope_cos_sin(pos, inv)          # bf16 [B, S, 128]
    rq, rk, rv = oref.attention_block(c["hidden"], c["qkv_w"], None, c["in_norm"], c["q_norm"],
                                      c["k_norm"], hc[:, None], hs[:, None], Hq, Hkv)
    compare("mrope q", q.cpu(), rq, max_abs=3.2e-2, min_cos=0.99999)
    compare("mrope k", k.cpu(), rk, max_abs=3.2e-2, min_cos=0.99999)
    # device-resident position (graph replay path) == host position
    pos_dev = torch.tensor([c["start"]], dtype=torch.int32, device=DEV)
    cos, sin = oref.rotary_tables(128, c["max_seq"], 5e6)
    q1, _, _ = ops.qkv_norm_rope(qkv.to(DEV).contiguous(), c["q_norm"].to(DEV),
                                 c["k_norm"].to(DEV), cos.to(DEV), sin.to(DEV), B=B, S=S, Hq=Hq,
                                 Hkv=Hkv, start_pos=c["start"])
    q2, _, _ = ops.qkv_norm_rope(qkv.to(DEV).contiguous(), c["q_norm"].to(DEV),
                                 c["k_norm"].to(DEV), cos.to(DEV), sin.to(DEV), B=B, S=S, Hq=Hq,
                                 Hkv=Hkv, start_pos=0, pos_dev=pos_dev)
    assert torch.equal(q1, q2)


# --------------------------------------------------------------------------- a6/a8 decode
def test_decode_attention_config1_fp32_vs_reference():
    """Config 1 (B1, Hq32, Hkv8, D128, L1024, fp32): max-abs <= 1e-5 vs the
    reference forward_layer's eager attention (golden)."""
    g = load_golden("decode_cfg1")
    q, k, v = cases.decode_cfg1_inputs()
    out = ops.attn_decode(q.to(DEV), k.to(DEV), v.to(DEV), kv_len=1024).cpu()
    compare("decode cfg1", out, as_tensor(g["out"]), max_abs=1e-5, min_cos=0.999999)


@pytest.mark.parametrize("B,Hq,Hkv,L,maxS", [(3, 8, 2, 777, 1024), (8, 32, 8, 1100, 2048),
                                            (2, 4, 1, 1, 64), (1, 4, 1, 64, 64),
                                            (2, 16, 16, 300, 512), (1, 16, 2, 4096, 4096)])
def test_decode_attention_bf16(B, Hq, Hkv, L, maxS):
    q = rnd(B, Hq, 128, seed=7)
    kc = rnd(B, Hkv, maxS, 128, seed=8)
    vc = rnd(B, Hkv, maxS, 128, seed=9)
    out = ops.attn_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), kv_len=L).cpu()
    want = oref.decode_attention_fp32(q.float(), kc[:, :, :L].float(), vc[:, :, :L].float())
    compare("decode bf16", out, want, max_abs=1e-2, min_cos=0.9999)
    # the reference's own bf16 eager path (rounded scores/probabilities)
    eager = oref.eager_attention(q[:, :, None], kc[:, :, :L], vc[:, :, :L], L - 1)[:, :, 0]
    compare("decode vs eager bf16", out, eager, max_abs=2e-2, min_cos=0.9999)


def test_decode_attention_device_length():
    q = rnd(2, 8, 128, seed=10)
    kc, vc = rnd(2, 2, 2048, 128, seed=11), rnd(2, 2, 2048, 128, seed=12)
    qd, kd, vd = q.to(DEV), kc.to(DEV), vc.to(DEV)
    for L in (1, 513, 2048):
        Ld = torch.tensor([L], dtype=torch.int32, device=DEV)
        a = ops.attn_decode(qd, kd, vd, kv_len=2048, kv_len_dev=Ld).cpu()
        b = ops.attn_decode(qd, kd, vd, kv_len=L).cpu()
        compare(f"decode dev len {L}", a, b, max_abs=2e-3, min_cos=0.99999)


@pytest.mark.parametrize("dtype", [BF16, torch.float32])
def test_decode_attention_device_length_decode_graph_shape(dtype):
    """The decode graph's call: grid planned for the KV bucket (2048), actual
    length read on the device; the splits share the present positions.  bf16:
    max-abs <= 1e-2, cosine >= 0.9999 vs the fp32 oracle; fp32: max-abs <= 1e-5."""
    B, Hq, Hkv, S = 8, 32, 8, 2048
    q = rnd(B, Hq, 128, seed=13).to(dtype)
    kc, vc = rnd(B, Hkv, S, 128, seed=14).to(dtype), rnd(B, Hkv, S, 128, seed=15).to(dtype)
    qd, kd, vd = q.to(DEV), kc.to(DEV), vc.to(DEV)
    for L in (1, 63, 65, 1152, 1279, 2048):
        Ld = torch.tensor([L], dtype=torch.int32, device=DEV)
        got = ops.attn_decode(qd, kd, vd, kv_len=S, kv_len_dev=Ld).cpu()
        want = oref.decode_attention_fp32(q.float(), kc[:, :, :L].float(), vc[:, :, :L].float())
        if dtype == BF16:
            compare(f"graph-shape decode L={L}", got, want, max_abs=1e-2, min_cos=0.9999)
        else:
            compare(f"graph-shape decode fp32 L={L}", got, want, max_abs=1e-5)


@pytest.mark.parametrize("B,Hq,Hkv,L,dev_len,offset", [(8, 32, 8, 1152, True, 0),
                                                       (8, 32, 8, 65, True, 3),
                                                       (8, 32, 8, 1, False, 0),
                                                       (1, 4, 1, 40, False, 5),
                                                       (3, 8, 1, 300, True, 0),
                                                       (16, 32, 8, 2048, True, 0)])
def test_decode_attention_from_qkv_matches_norm_rope_then_attention(B, Hq, Hkv, L, dev_len,
                                                                     offset):
    """q3_attn_decode_qkv == q3_qkv_norm_rope (new row written at L-1) followed
    by q3_attn_decode: the new K/V cache rows bit-identical; the attention
    output max-abs <= 2e-2 of its scale, cosine >= 0.9999 (the new row's
    probability is not rounded to bf16 before P.V here)."""
    D, S = 128, 2048
    qkv = rnd(B, (Hq + 2 * Hkv) * D, seed=80)
    qn = (1 + rnd(D, seed=81, std=0.1)).to(BF16)
    kn = (1 + rnd(D, seed=82, std=0.1)).to(BF16)
    cos, sin = oref.rotary_tables(D, S + 16, 5e6)
    kc = rnd(B, Hkv, S, D, seed=83)
    vc = rnd(B, Hkv, S, D, seed=84)
    kc1, vc1, kc2, vc2 = kc.to(DEV), vc.to(DEV), kc.to(DEV), vc.to(DEV)
    qkvd, qnd, knd, cd, sd = qkv.to(DEV), qn.to(DEV), kn.to(DEV), cos.to(DEV), sin.to(DEV)
    pos = L - 1
    Ld = torch.tensor([L], dtype=torch.int32, device=DEV) if dev_len else None
    bound = S if dev_len else L
    got = ops.attn_decode_qkv(qkvd, qnd, knd, cd, sd, kc1, vc1, Hq=Hq, Hkv=Hkv, kv_len=bound,
                              kv_len_dev=Ld, cs_offset=offset)
    q, _, _ = ops.qkv_norm_rope(qkvd, qnd, knd, cd, sd, B=B, S=1, Hq=Hq, Hkv=Hkv,
                                start_pos=pos, cs_offset=offset, k_cache=kc2, v_cache=vc2)
    want = ops.attn_decode(q.view(B, Hq, D), kc2, vc2, kv_len=L)
    torch.cuda.synchronize()
    assert torch.equal(kc1[:, :, pos].cpu(), kc2[:, :, pos].cpu()), "new k row differs"
    assert torch.equal(vc1[:, :, pos].cpu(), vc2[:, :, pos].cpu()), "new v row differs"
    assert torch.equal(kc1.cpu(), kc2.cpu()) and torch.equal(vc1.cpu(), vc2.cpu())
    compare(f"attn from qkv B={B} L={L}", got.cpu(), want.cpu(), max_abs=2e-2, rel_scale=True,
            min_cos=0.9999)


@pytest.mark.parametrize("B,Hq,Hkv,L,page,offset", [(8, 32, 8, 1152, 256, 0),
                                                     (4, 32, 8, 257, 128, 2),
                                                     (3, 8, 1, 64, 64, 0),
                                                     (2, 16, 4, 2048, 512, 1)])
def test_paged_decode_attention_from_qkv_matches_norm_rope_then_attention(B, Hq, Hkv, L, page,
                                                                           offset):
    """q3_attn_decode_qkv_paged == q3_qkv_norm_rope_paged (new row into its
    page) followed by q3_attn_decode_paged, over pages dealt in a shuffled
    order: both pools bit-identical after the call (the new rows land in the
    same page slots), the outputs within the tolerance of the contiguous case."""
    D, S = 128, 2048
    per = S // page
    qkv = rnd(B, (Hq + 2 * Hkv) * D, seed=90)
    qn = (1 + rnd(D, seed=91, std=0.1)).to(BF16)
    kn = (1 + rnd(D, seed=92, std=0.1)).to(BF16)
    cos, sin = oref.rotary_tables(D, S + 16, 5e6)
    kp = rnd(B * per + 3, Hkv, page, D, seed=93)
    vp = rnd(B * per + 3, Hkv, page, D, seed=94)
    perm = torch.randperm(B * per + 3, generator=torch.Generator().manual_seed(5))[:B * per]
    table = perm.view(B, per).to(torch.int32).to(DEV)
    kp1, vp1, kp2, vp2 = kp.to(DEV), vp.to(DEV), kp.to(DEV), vp.to(DEV)
    qkvd, qnd, knd, cd, sd = qkv.to(DEV), qn.to(DEV), kn.to(DEV), cos.to(DEV), sin.to(DEV)
    pos = L - 1
    Ld = torch.tensor([L], dtype=torch.int32, device=DEV)
    Pd = torch.tensor([pos], dtype=torch.int32, device=DEV)
    got = ops.attn_decode_qkv_paged(qkvd, qnd, knd, cd, sd, kp1, vp1, table, Hq=Hq, Hkv=Hkv,
                                    kv_len=S, kv_len_dev=Ld, cs_offset=offset)
    q = ops.qkv_norm_rope_paged(qkvd, qnd, knd, cd, sd, B=B, S=1, Hq=Hq, Hkv=Hkv, k_pages=kp2,
                                v_pages=vp2, block_table=table, start_pos=0, pos_dev=Pd,
                                cs_offset=offset)
    want = ops.attn_decode_paged(q.view(B, Hq, D), kp2, vp2, table, kv_len=S, kv_len_dev=Ld)
    torch.cuda.synchronize()
    assert torch.equal(kp1.cpu(), kp2.cpu()) and torch.equal(vp1.cpu(), vp2.cpu())
    compare(f"paged attn from qkv B={B} L={L}", got.cpu(), want.cpu(), max_abs=2e-2,
            rel_scale=True, min_cos=0.9999)


# --------------------------------------------------------------------------- a6/a7 prefill
def test_prefill_kat_vs_reference_attention_ref():
    """kernels/prefill_attention.py layouts (q [Hq,D,S], k [Hkv,D,S], v [Hkv,S,D])."""
    g = load_golden("kernels_kat")
    _, _, _, q, k, v = cases.kernels_kat_inputs()
    qd = q.transpose(1, 2)[None].to(DEV)          # strided views with unit d stride
    kd = k.transpose(1, 2).contiguous()[None].to(DEV)
    vd = v[None].contiguous().to(DEV)
    out = ops.attn_prefill(qd.contiguous(), kd, vd, causal=True)[0].cpu()
    compare("prefill KAT", out, as_tensor(g["attn"]), max_abs=2e-2, min_cos=0.9999)


@pytest.mark.parametrize("B,Hq,Hkv,S,start,causal", [(1, 32, 8, 2048, 0, True),
                                                     (2, 8, 2, 200, 0, True),
                                                     (1, 4, 1, 130, 70, True),
                                                     (1, 8, 8, 96, 0, False),
                                                     (3, 4, 4, 1, 37, True)])
def test_prefill_attention(B, Hq, Hkv, S, start, causal):
    q = rnd(B, Hq, S, 128, seed=20)
    k = rnd(B, Hkv, start + S, 128, seed=21)
    v = rnd(B, Hkv, start + S, 128, seed=22)
    out = ops.attn_prefill(q.to(DEV), k.to(DEV), v.to(DEV), start_pos=start, causal=causal).cpu()
    if causal:
        want = oref.causal_attention_fp32(q, k, v, start)
    else:
        rep = Hq // Hkv
        s = q.float() @ k.float().repeat_interleave(rep, 1).transpose(-2, -1) / math.sqrt(128)
        want = torch.softmax(s, -1) @ v.float().repeat_interleave(rep, 1)
    compare("prefill", out, want, max_abs=2e-2, min_cos=0.9999)


def test_prefill_attention_output_layout_bshd():
    """Writing straight into the [B, S, Hq*D] layout o_proj consumes."""
    B, Hq, Hkv, S = 2, 8, 2, 160
    q, k, v = rnd(B, Hq, S, 128, seed=23), rnd(B, Hkv, S, 128, seed=24), rnd(B, Hkv, S, 128, seed=25)
    o = torch.empty(B, S, Hq, 128, dtype=BF16, device=DEV)
    ops.attn_prefill(q.to(DEV), k.to(DEV), v.to(DEV), out=o.transpose(1, 2))
    want = oref.causal_attention_fp32(q, k, v).transpose(1, 2)
    compare("prefill bshd", o.cpu(), want, max_abs=2e-2, min_cos=0.9999)


# --------------------------------------------------------------------------- GEMMs
def _mm_ref(a, w):
    return (a.float() @ w.float().t()).to(BF16)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (5, 768, 4096), (8, 6144, 4096),
                                   (16, 4096, 1536), (9, 18992, 512), (17, 768, 4096),
                                   (128, 512, 512), (300, 1024, 4096), (1024, 3072, 4096),
                                   (2048, 4096, 1536), (256, 272, 256)])
def test_gemm_plain(M, N, K):
    a = rnd(M, K, seed=30)
    w = rnd(N, K, seed=31, std=0.02)
    c = ops.gemm(a.to(DEV), w.to(DEV)).cpu()
    compare(f"gemm {M}x{N}x{K}", c, _mm_ref(a, w), max_abs=1e-2, rel_scale=True,
            min_cos=0.99999)


@pytest.mark.parametrize("M", [4, 200])
def test_gemm_residual(M):
    N, K = 4096, 1536
    a, w, r = rnd(M, K, seed=32), rnd(N, K, seed=33, std=0.02), rnd(M, N, seed=34)
    c = ops.gemm(a.to(DEV), w.to(DEV), "residual", residual=r.to(DEV)).cpu()
    compare("gemm+residual", c, r + _mm_ref(a, w), max_abs=1e-2, rel_scale=True,
            min_cos=0.99999)


@pytest.mark.parametrize("M", [3, 16, 130, 512])
def test_gemm_swiglu(M):
    I, H = 1536, 4096
    a = rnd(M, H, seed=35)
    gate, up = rnd(I, H, seed=36, std=0.02), rnd(I, H, seed=37, std=0.02)
    w = layout.interleave_gate_up(gate, up)
    c = ops.gemm(a.to(DEV), w.to(DEV), "swiglu").cpu()
    gu = a @ torch.cat([gate, up], 0).t()        # reference: fused [gate | up] product
    g_, u_ = gu.chunk(2, dim=-1)
    want = torch.nn.functional.silu(g_) * u_
    compare("gemm+swiglu", c, want, max_abs=2e-2, rel_scale=True, min_cos=0.9999)


# ------------------------------------- prefill QKV with norm + RoPE in the epilogue
@pytest.mark.parametrize("B,S,Hq,Hkv,H,start,mrope", [(1, 40, 4, 1, 512, 0, False),
                                                      (2, 300, 32, 8, 4096, 17, False),
                                                      (2, 100, 8, 2, 1024, 0, True),
                                                      (3, 129, 4, 1, 2048, 5, False)])
def test_gemm_qkv_rope_matches_gemm_then_norm_rope(B, S, Hq, Hkv, H, start, mrope):
    """q3_gemm_qkv_rope == q3_gemm followed by q3_qkv_norm_rope (the same
    rounding points; the head norm's sum runs in another order, so a bf16 value
    may differ by one rounding step): max-abs <= 2e-2 of the output scale,
    cosine >= 0.99999, at most 1% of elements differing."""
    D, maxS = 128, 512
    h = rnd(B * S, H, seed=70)
    w = rnd((Hq + 2 * Hkv) * D, H, seed=71, std=0.02)
    qn = (1 + rnd(D, seed=72, std=0.1)).to(BF16)
    kn = (1 + rnd(D, seed=73, std=0.1)).to(BF16)
    if mrope:   # per-token f32 rows, as M-RoPE builds them
        ang = torch.rand(B * S, 64, generator=torch.Generator().manual_seed(74)) * 50
        cos, sin = ang.cos(), ang.sin()
        kw = dict(cs_use_pos=False, cs_offset=0, cs_stride_b=S)
    else:       # bf16 tables indexed by position, as RotaryEmbedding builds them
        cos, sin = oref.rotary_tables(D, maxS + 8, 5e6)
        kw = dict(cs_use_pos=True, cs_offset=3, cs_stride_b=0)
    dv = dict(device=DEV)
    hd, wd, cd, sd = h.to(DEV), w.to(DEV), cos.to(DEV), sin.to(DEV)
    caches = [torch.zeros(B, Hkv, maxS, D, dtype=BF16, **dv) for _ in range(4)]
    q1 = ops.gemm_qkv_rope(hd, wd, qn.to(DEV), kn.to(DEV), cd, sd, B=B, S=S, Hq=Hq, Hkv=Hkv,
                           k_cache=caches[0], v_cache=caches[1], start_pos=start, **kw)
    qkv = ops.gemm(hd, wd)
    q2, _, _ = ops.qkv_norm_rope(qkv, qn.to(DEV), kn.to(DEV), cd, sd, B=B, S=S, Hq=Hq, Hkv=Hkv,
                                 start_pos=start, k_cache=caches[2], v_cache=caches[3], **kw)
    for name, a, b in (("q", q1, q2), ("k cache", caches[0], caches[2]),
                       ("v cache", caches[1], caches[3])):
        compare(f"fused qkv {name}", a.cpu(), b.cpu(), max_abs=2e-2, rel_scale=True,
                min_cos=0.99999)
        diff = (a.view(torch.int16) != b.view(torch.int16)).float().mean().item()
        assert diff < 0.01, f"fused qkv {name}: {diff:.3%} of elements differ"
    # rows outside start .. start + S - 1 untouched
    assert torch.count_nonzero(caches[0][:, :, :start]) == 0
    assert torch.count_nonzero(caches[0][:, :, start + S:]) == 0


# ------------------------------------------------- decode projections, norm fused
@pytest.mark.parametrize("M,N,K,epi", [(1, 6144, 4096, "none"), (8, 6144, 4096, "none"),
                                       (13, 4096, 4096, "none"), (16, 2048, 544, "none"),
                                       (8, 3072, 4096, "swiglu"), (11, 3072, 4096, "swiglu"),
                                       (8, 4096, 4096, "residual")])
def test_gemm_norm_matches_norm_then_gemm(M, N, K, epi):
    """q3_gemm_norm == rmsnorm (model_fused.py:37-40) followed by the projection;
    bf16 tolerance: max-abs 1e-2 of the output scale, cosine >= 0.99999."""
    a = rnd(M, K, seed=50)
    nw = (1 + rnd(K, seed=51, std=0.1)).to(BF16)
    w = rnd(N, K, seed=52, std=0.02)
    r = rnd(M, N, seed=53)
    h = oref.rmsnorm(a, nw, 1e-6)
    c = ops.gemm_norm(a.to(DEV), nw.to(DEV), w.to(DEV), 1e-6, epi,
                      residual=r.to(DEV) if epi == "residual" else None).cpu()
    if epi == "swiglu":
        want = ops.gemm(h.to(DEV), w.to(DEV), "swiglu").cpu()
        compare("gemm_norm swiglu", c, want, max_abs=2e-2, rel_scale=True, min_cos=0.9999)
        return
    want = _mm_ref(h, w)
    if epi == "residual":
        want = r + want
    compare(f"gemm_norm {M}x{N}x{K} {epi}", c, want, max_abs=1e-2, rel_scale=True,
            min_cos=0.99999)


@pytest.mark.parametrize("M", [8, 16])
def test_gemm_decode_sum_of_squares_chain(M):
    """o_proj-like residual projection emits per-tile sums of squares; the next
    projection's fused norm consumes them instead of re-reading its input."""
    H, Kin, N2 = 4096, 1024, 3072
    a = rnd(M, Kin, seed=60)
    w1 = rnd(H, Kin, seed=61, std=0.02)
    x = rnd(M, H, seed=62)
    nw = (1 + rnd(H, seed=63, std=0.1)).to(BF16)
    w2 = rnd(N2, H, seed=64, std=0.02)
    ss = torch.full((H // 64, 16), float("nan"), device=DEV)
    x2 = ops.gemm_decode(a.to(DEV), w1.to(DEV), "residual", residual=x.to(DEV), ss_out=ss)
    x2h = x2.cpu()
    compare("residual projection", x2h, x + _mm_ref(a, w1), max_abs=1e-2, rel_scale=True,
            min_cos=0.99999)
    tot = ss[:, :M].sum(0).cpu()
    want_ss = (x2h.float() ** 2).sum(-1)
    assert torch.allclose(tot, want_ss, rtol=1e-4), (tot, want_ss)
    c = ops.gemm_decode(x2, w2.to(DEV), norm_w=nw.to(DEV), eps=1e-6, ss_in=ss,
                        ss_tiles=H // 64).cpu()
    c_re = ops.gemm_decode(x2, w2.to(DEV), norm_w=nw.to(DEV), eps=1e-6).cpu()
    want = _mm_ref(oref.rmsnorm(x2h, nw, 1e-6), w2)
    compare("norm from ss_in", c, want, max_abs=1e-2, rel_scale=True, min_cos=0.99999)
    compare("norm recomputed", c_re, want, max_abs=1e-2, rel_scale=True, min_cos=0.99999)


# --------------------------------------------------------------------------- a13
def test_embed_and_argmax():
    V, H = 1000, 512
    table = rnd(V, H, seed=40)
    ids = torch.tensor([[0, 5, 999], [17, 17, 3]])
    out = ops.embed(ids.to(DEV), table.to(DEV)).cpu()
    assert torch.equal(out, table[ids])
    logits = rnd(4, 151936, seed=41)
    logits[2, 77] = 100.0
    logits[2, 9000] = 100.0  # tie -> first index
    idx = ops.argmax(logits.to(DEV)).cpu()
    assert idx.tolist() == logits.float().argmax(-1).tolist()
    assert idx[2].item() == 77


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_distributed_argmax_keys_match_gathered_argmax(tp):
    """Per-rank keys of the vocabulary slices, MAX-reduced (emulated here by
    an elementwise max over the slices' keys), decode to torch.argmax of the
    concatenated logits, first index on ties: ties inside a slice, across
    slices, negative maxima, an all-equal row and -inf entries."""
    V = 151936
    logits = rnd(8, V, seed=42)
    n = V // tp
    logits[0, n // 2] = 50.0
    logits[0, n + 3] = 50.0                      # same value in a later slice
    logits[1] = -3.0                             # all equal -> index 0
    logits[2] = -float("inf")
    logits[2, V - 1] = -1e30                     # only finite entry, last slice
    logits[3, 17] = 9.0
    logits[3, 18] = 9.0                          # tie inside one slice
    logits[4] = -(logits[4].abs() + 1)           # every value negative
    logits[5, n - 1] = 30.0
    logits[5, n] = 30.0                          # tie across a slice boundary
    d = logits.to(DEV)
    keys = torch.stack([ops.argmax_key(d[:, r * n:(r + 1) * n].contiguous(), r * n)
                        for r in range(tp)])
    idx = ops.argmax_key_index(keys.max(dim=0).values.contiguous()).cpu()
    assert idx.tolist() == logits.float().argmax(-1).tolist()
    assert idx[0].item() == n // 2 and idx[1].item() == 0 and idx[2].item() == V - 1
    assert idx[3].item() == 17 and idx[5].item() == n - 1


def test_device_error_word_clear():
    assert ops.device_error(clear=True) == 0
