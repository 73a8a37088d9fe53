"""Vision tower on the GPU vs the CPU oracle (oracle/vision.py, itself pinned
bit-exact to transformers' Qwen3VLVisionModel) and the golden fixture.

Tolerances, per test: bias-epilogue linears max-abs <= 6.25e-2 and cosine
>= 0.9999 against an fp32-accumulated reference with the same rounding
points; LayerNorm max-abs <= 3.2e-2; position embeddings bit-exact; RoPE
max-abs <= 1.6e-2 (the cos/sin implementations may differ in the last fp32
bit); attention max-abs <= 2e-2 and cosine >= 0.9999 against fp32 attention;
whole tower cosine >= 0.999 on every output."""
import pytest
import torch
import torch.nn.functional as F

from oracle import vision as ovis
from q3vl import ops
from q3vl.vision_tower import VisionPlan, VisionTower
from tests.golden import cases
from tests.helpers import as_tensor, compare, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF16 = torch.bfloat16


def rnd(*shape, seed=0, std=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std).to(BF16)


def linear_ref(a, w, b, epi, r=None):
    v = (a.float() @ w.float().t() + b.float()).to(BF16)
    if epi == "bias_gelu_tanh":
        v = F.gelu(v.float(), approximate="tanh").to(BF16)
    elif epi == "bias_gelu":
        v = F.gelu(v.float()).to(BF16)
    elif epi == "bias_residual":
        v = (r.float() + v.float()).to(BF16)
    return v


@pytest.mark.parametrize("M,N,K", [(300, 152, 144), (1024, 1152, 4304), (17, 4608, 4608),
                                   (5, 72, 64)])
@pytest.mark.parametrize("epi", ["bias", "bias_gelu_tanh", "bias_gelu", "bias_residual"])
def test_gemm_bias_epilogues(M, N, K, epi):
    a, w = rnd(M, K, seed=1), rnd(N, K, seed=2, std=K ** -0.5)
    b, r = rnd(N, seed=3, std=0.1), rnd(M, N, seed=4)
    got = ops.gemm_bias(a.to(DEV), w.to(DEV), b.to(DEV), epi,
                        residual=r.to(DEV) if epi == "bias_residual" else None).cpu()
    compare(f"gemm_bias {epi}", got, linear_ref(a, w, b, epi, r), max_abs=6.25e-2,
            min_cos=0.9999)


def test_gemm_bias_residual_in_place():
    a, w, b, r = rnd(200, 1152, seed=5), rnd(1152, 1152, seed=6, std=0.03), \
        rnd(1152, seed=7), rnd(200, 1152, seed=8)
    h = r.to(DEV)
    ops.gemm_bias(a.to(DEV), w.to(DEV), b.to(DEV), "bias_residual", residual=h, out=h)
    compare("in place", h.cpu(), linear_ref(a, w, b, "bias_residual", r), max_abs=6.25e-2,
            min_cos=0.9999)


@pytest.mark.parametrize("rows,cols", [(37, 1152), (9, 4608), (300, 144)])
def test_layernorm(rows, cols):
    x = rnd(rows, cols, seed=9, std=2.0) + 0.5
    w, b = (1 + rnd(cols, seed=10, std=0.1).float()).to(BF16), rnd(cols, seed=11, std=0.1)
    got = ops.layernorm(x.to(DEV), w.to(DEV), b.to(DEV), 1e-6).cpu()
    want = F.layer_norm(x, (cols,), w, b, 1e-6)
    compare("layernorm", got, want, max_abs=3.2e-2, min_cos=0.99999)


GRIDS = [[1, 8, 12], [2, 6, 4], [1, 34, 46]]


def test_position_embeddings_bit_exact():
    grid = torch.tensor(GRIDS)
    table = rnd(48 * 48, 1152, seed=12, std=0.5)
    plan = VisionPlan(grid, 2, DEV)
    got = ops.vision_pos_embed(table.to(DEV), plan.imgs, plan.imgs_host, 2, plan.n_tok).cpu()
    assert torch.equal(got, ovis.pos_embed_interpolate(table, grid, 2))


def test_vision_rope_matches_oracle():
    grid = torch.tensor(GRIDS)
    plan = VisionPlan(grid, 2, DEV)
    heads, hd = 16, 72
    qkv = rnd(plan.n_tok, 3 * heads * hd, seed=13)
    dim = hd // 2
    inv = 1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
    dev = qkv.to(DEV)
    ops.vision_rope(dev, heads, inv.to(DEV), plan.imgs, plan.imgs_host, 2)
    got = dev.cpu().view(plan.n_tok, 3, heads, hd)
    cos, sin = ovis.rotary_cos_sin(grid, hd, 2)
    c, s = cos[:, None, :], sin[:, None, :]
    src = qkv.view(plan.n_tok, 3, heads, hd)
    for part in (0, 1):
        x = src[:, part].float()
        want = (x * c + ovis._rotate_half(x) * s).to(BF16)
        compare(f"rope part {part}", got[:, part], want, max_abs=1.6e-2, min_cos=0.99999)
    assert torch.equal(got[:, 2], src[:, 2])           # v untouched


def test_frame_attention_matches_fp32():
    grid = torch.tensor(GRIDS)
    plan = VisionPlan(grid, 2, DEV)
    heads, hd = 16, 72
    qkv = rnd(plan.n_tok, 3 * heads * hd, seed=14)
    got = ops.vision_attention(qkv.to(DEV), heads, plan.blocks, plan.blocks_host).cpu()
    q, k, v = qkv.float().view(plan.n_tok, 3, heads, hd).unbind(1)
    outs = []
    cu = ovis.frame_bounds(grid)
    for a, b in zip(cu[:-1], cu[1:]):
        sc = torch.einsum("qhd,khd->hqk", q[a:b], k[a:b]) * hd ** -0.5
        outs.append(torch.einsum("hqk,khd->qhd", torch.softmax(sc, -1), v[a:b]))
    want = torch.cat(outs).reshape(plan.n_tok, heads * hd)
    compare("frame attention", got, want, max_abs=2e-2, min_cos=0.9999)


def _check_tower(tower, x, grid, pooler, deep, last):
    p, d, h = tower(x.to(DEV), grid)
    compare("pooler", p.cpu(), pooler, max_abs=5e-2, rel_scale=True, min_cos=0.999)
    compare("last hidden", h.cpu(), last, max_abs=5e-2, rel_scale=True, min_cos=0.999)
    assert len(d) == len(deep)
    for j, (a, b) in enumerate(zip(d, deep)):
        compare(f"deepstack {j}", a.cpu(), b, max_abs=5e-2, rel_scale=True, min_cos=0.999)


def test_tiny_tower_matches_hf_fixture():
    g = load_golden("vision_tiny")
    x, grid = cases.vision_tiny_inputs()
    tower = VisionTower(cases.vision_tiny_weights(), cases.VISION_TINY, DEV)
    deep = [as_tensor(g["bf16_deepstack0"]), as_tensor(g["bf16_deepstack1"])]
    _check_tower(tower, x, grid, as_tensor(g["bf16_pooler"]), deep, as_tensor(g["bf16_last"]))


def test_full_width_block_matches_oracle():
    """hidden 1152, 16 heads, MLP 4304, merger to 4096 (the 8B tower's widths),
    one block with a deepstack merger, an image and a two-frame clip."""
    c = dict(cases.VISION_TINY, depth=1, hidden_size=1152, num_heads=16,
             intermediate_size=4304, out_hidden_size=4096, num_position_embeddings=2304,
             deepstack_visual_indexes=[0])
    w = cases.vision_weights(c, seed=41)
    grid = torch.tensor([[1, 16, 16], [2, 8, 12]])
    n = int((grid[:, 0] * grid[:, 1] * grid[:, 2]).sum())
    x = torch.randn(n, 1536, generator=torch.Generator().manual_seed(42))
    pooler, deep, last = ovis.vision_forward(x, grid, w, depth=1, heads=16, merge=2,
                                             deepstack=(0,), dtype=BF16)
    _check_tower(VisionTower(w, c, DEV), x, grid, pooler, deep, last)


@pytest.mark.parametrize("name", cases.DROPIN_CASES)
def test_dropin_prepare_vision_embeds_matches_the_reference(name):
    """The drop-in vision.prepare_vision_embeds on the GPU against the
    reference's own prepare_vision_embeds (fixture) on the same seeded
    transformers model: text rows and the visual mask identical, visual rows
    and deepstack levels within the tower's tolerance."""
    import vision
    g = load_golden("vision_dropin")
    model = cases.dropin_hf_model()
    emb, deep, mask = vision.prepare_vision_embeds(model, None, cases.dropin_inputs(name), DEV)
    want_mask = torch.from_numpy(g[name + "_mask"])
    assert torch.equal(mask.cpu(), want_mask)
    want = as_tensor(g[name + "_embeds"])
    assert torch.equal(emb[0, ~mask].cpu(), want[0, ~want_mask])
    compare("visual rows", emb[0, mask].cpu(), want[0, want_mask], max_abs=5e-2, rel_scale=True,
            min_cos=0.999)
    assert len(deep) == int(g[name + "_levels"])
    for j, d in enumerate(deep):
        compare(f"deepstack {j}", d.cpu(), as_tensor(g[f"{name}_deepstack{j}"]), max_abs=5e-2,
                rel_scale=True, min_cos=0.999)
