"""Seeded inputs shared by the fixture generator and the tests.

Everything here is regenerated deterministically from CPU torch RNG seeds, so
the fixtures only need to store outputs (and input checksums).
"""
from __future__ import annotations

import math

import torch

from oracle import decoder as odec
from oracle import ref as oref

BF16 = torch.bfloat16


# ---- test_kernels.py:34,113-123,171-175: seed 42, S=256, 4 q heads, 1 kv head ----
def kernels_kat_inputs():
    g = torch.Generator().manual_seed(42)
    x = torch.randn(256, 4, 128, dtype=BF16, generator=g)
    inv = 1.0 / (1000000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    freqs = torch.outer(torch.arange(256, dtype=torch.float32), inv)
    cos, sin = freqs.cos(), freqs.sin()
    q = torch.randn(4, 128, 256, dtype=BF16, generator=g)
    k = torch.randn(1, 128, 256, dtype=BF16, generator=g)
    v = torch.randn(1, 256, 128, dtype=BF16, generator=g)
    return x, cos, sin, q, k, v


# ---- config 1: B1, 32 q heads, 8 kv heads, D128, L1024, fp32, N(0,1) ----
def decode_cfg1_inputs(seed: int = 0, B: int = 1, Hq: int = 32, Hkv: int = 8, L: int = 1024):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, 128, generator=g)
    k = torch.randn(B, Hkv, L, 128, generator=g)
    v = torch.randn(B, Hkv, L, 128, generator=g)
    return q, k, v


# ---- a3: AttentionBlock on small shapes (TP8-like 4:1 GQA, nonzero offset) ----
def attn_block_case(seed: int = 3):
    g = torch.Generator().manual_seed(seed)
    H, Hq, Hkv, S, B = 512, 4, 1, 32, 2

    def rn(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(BF16)

    return dict(
        H=H, Hq=Hq, Hkv=Hkv, S=S, B=B, start=16, max_seq=128,
        qkv_w=rn(H, (Hq + 2 * Hkv) * 128), o_w=rn(Hq * 128, H),
        in_norm=(1 + torch.randn(H, generator=g) * 0.1).to(BF16),
        q_norm=(1 + torch.randn(128, generator=g) * 0.1).to(BF16),
        k_norm=(1 + torch.randn(128, generator=g) * 0.1).to(BF16),
        hidden=torch.randn(B, S, H, generator=g).to(BF16))


# ---- one Qwen3-VL-8B-shape layer at TP1 ----
def layer8b_case(seed: int = 1):
    spec = odec.Spec(layers=1, vocab=16, max_seq=64)
    w = odec.make_weights(spec, seed=seed, random_norms=True)
    g = torch.Generator().manual_seed(seed + 100)
    hidden = torch.randn(1, 8, 4096, generator=g).to(BF16)
    hidden_dec = torch.randn(1, 1, 4096, generator=g).to(BF16)
    return dict(spec=spec, weights=w, hidden=hidden, hidden_dec=hidden_dec, S=8, max_seq=64)


# ---- config 3: one Qwen3-VL-8B-shape layer at TP8 sharding ----
# N(0, 0.02) bf16 weights (norms 1.0), hidden states N(0, 1): prefill of
# 4 x 512 tokens, then 128 decode steps of 4 x 1 fresh N(0, 1) states.  The
# fixture keeps a fingerprint of every output (the layer's contribution,
# out - in, projected on 16 seeded directions) and a few whole rows.
LAYER_TP8 = dict(seed=5, B=4, S=512, steps=128, tp=8, max_seq=1024, proj_dim=16,
                 pre_tokens=(0, 1, 200, 511), dec_steps=(0, 64, 127))


def layer_tp8_case():
    c = LAYER_TP8
    spec = odec.Spec(layers=1, vocab=16, max_seq=c["max_seq"])
    w = odec.make_weights(spec, seed=c["seed"])
    g = torch.Generator().manual_seed(c["seed"] + 100)
    hidden = torch.randn(c["B"], c["S"], 4096, generator=g).to(BF16)
    dec_in = torch.randn(c["steps"], c["B"], 1, 4096, generator=g).to(BF16)
    return dict(spec=spec, weights=w, hidden=hidden, dec_in=dec_in)


def fingerprint_matrix(dim: int = 16, hidden: int = 4096, seed: int = 999) -> torch.Tensor:
    """Seeded directions [hidden, dim] (unit scale) for output fingerprints."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(hidden, dim, generator=g) / math.sqrt(hidden)


def layer_fingerprint(out: torch.Tensor, inp: torch.Tensor, R: torch.Tensor) -> torch.Tensor:
    """fp32 projection of a layer's contribution (out - in) on R's directions."""
    return (out.float().cpu() - inp.float().cpu()) @ R


# ---- config 4: the 36-layer Qwen3-VL-8B-shape decoder at TP8 sharding ----
# N(0, 0.02) bf16 weights (norms 1.0) with a peaky lm_head, batch 8 prompts
# of 1024 uniform random ids, greedy tokens over the first 32 steps.
DECODER8B_TP8 = dict(seed=21, B=8, prompt_len=1024, new_tokens=32, tp=8, max_seq=2048, topk=8)


def decoder8b_spec() -> "odec.Spec":
    return odec.Spec(max_seq=DECODER8B_TP8["max_seq"])


def decoder8b_weights(on_layer=None) -> dict:
    """The config-4 weights (8B shape, 36 layers); on_layer as in
    oracle.decoder.make_weights, so a rank can keep only its shards."""
    c = DECODER8B_TP8
    w = odec.make_weights(decoder8b_spec(), seed=c["seed"], on_layer=on_layer)
    w["lm_head"] = peaky(w["lm_head"], c["seed"])
    return w


def decoder8b_prompt() -> torch.Tensor:
    c = DECODER8B_TP8
    g = torch.Generator().manual_seed(c["seed"] + 1)
    return torch.randint(0, decoder8b_spec().vocab, (c["B"], c["prompt_len"]), generator=g)


# ---- tiny full decoders (reference generate), TP1 and TP2 ----
DECODER_CASES = {
    "decoder_tiny_tp1": dict(
        spec=odec.Spec(hidden=512, q_heads=4, kv_heads=1, inter=1024, vocab=1024, layers=2,
                       max_seq=256),
        tp=1, seed=11, prompt_len=40, new_tokens=32, max_seq=256),
    "decoder_tiny_tp2": dict(
        spec=odec.Spec(hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=1024, layers=2,
                       max_seq=256),
        tp=2, seed=12, prompt_len=40, new_tokens=32, max_seq=256),
    # the TP2 case's weights and prompt at TP1: a greedy sequence that changes
    # token from step to step, checkable on one GPU
    "decoder_tiny8_tp1": dict(
        spec=odec.Spec(hidden=512, q_heads=8, kv_heads=2, inter=1024, vocab=1024, layers=2,
                       max_seq=256),
        tp=1, seed=12, prompt_len=40, new_tokens=32, max_seq=256),
}


def peaky(lm_head: torch.Tensor, seed: int) -> torch.Tensor:
    """Scale lm_head rows by lognormal factors so greedy argmax has clear margins
    (random-init logits otherwise sit within bf16 rounding of each other)."""
    g = torch.Generator().manual_seed(seed + 7)
    f = torch.exp(torch.randn(lm_head.shape[0], 1, generator=g) * 1.0)
    return (lm_head.float() * f).to(BF16)


def decoder_weights(name: str):
    c = DECODER_CASES[name]
    w = odec.make_weights(c["spec"], seed=c["seed"], random_norms=True)
    w["lm_head"] = peaky(w["lm_head"], c["seed"])
    return w


def decoder_prompt(name: str) -> torch.Tensor:
    c = DECODER_CASES[name]
    g = torch.Generator().manual_seed(c["seed"] + 1)
    return torch.randint(0, c["spec"].vocab, (1, c["prompt_len"]), generator=g)


def weights_checksum(w: dict) -> float:
    s = 0.0
    for lw in w["layers"]:
        for t in lw.values():
            s += float(t.double().abs().sum())
    for k in ("embed", "final_norm", "lm_head"):
        s += float(w[k].double().abs().sum())
    return s


# ---- config 2 M-RoPE: HF rotary on the 3-axis positions (first 512 tokens) ----
MROPE_ROWS = 512


def mrope_q_input(seed: int = 5):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(1, 1, MROPE_ROWS, 128, generator=g).to(BF16)


def hf_mrope_reference():
    """transformers 5.5.0 Qwen3VLTextRotaryEmbedding + apply_rotary_pos_emb."""
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import (Qwen3VLTextRotaryEmbedding,
                                                                apply_rotary_pos_emb)
    cfg = Qwen3VLTextConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8,
                            head_dim=128,
                            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                             "mrope_section": [24, 20, 20],
                                             "mrope_interleaved": True})
    rot = Qwen3VLTextRotaryEmbedding(cfg)
    pos = oref.config2_position_ids()            # [3, 1, 2048]
    q = mrope_q_input()
    cos, sin = rot(q, pos[:, :, :MROPE_ROWS])     # [1, S, 128] bf16
    qe, _ = apply_rotary_pos_emb(q, q, cos, sin)
    return cos[0, :, :64].contiguous(), sin[0, :, :64].contiguous(), qe


def attention_scale() -> float:
    return 1.0 / math.sqrt(128)


# ---- multimodal position ids (get_rope_index): seeded token-type layouts ----
def _vision_tokens(t, h, w, merge):
    return t * (h // merge) * (w // merge)


def rope_index_layout(seed: int, B: int, runs: int, merge: int = 2, pad_max: int = 6,
                      max_side: int = 10, holes: bool = True):
    """B sequences of alternating text and vision runs, left-padded to one length.

    Text runs are 1..12 tokens.  An image run takes a grid (t, h, w) with
    t in {1, 2} and h, w in merge*[1, max_side] (+1 now and then, which the
    // merge floors away).  A video is t frames of one (h, w) grid, each frame
    run preceded by a 1..3 token text run (the timestamp).  Grids are listed
    in batch order, as the model consumes them.  Padding tokens have random
    types (masked tokens are dropped before grouping); with `holes`, a few
    masked tokens also sit inside text runs.  Returns a dict of numpy arrays:
    types [B, S] int32, mask [B, S] int32, image_thw [Ni, 3], video_thw [Nv, 3]
    (int64, possibly with zero rows)."""
    import random
    import numpy as np
    rnd = random.Random(seed)
    seqs, masks, imgs, vids = [], [], [], []
    for _ in range(B):
        ty, mk = [], []

        def text(n):
            for _ in range(n):
                ty.append(0)
                mk.append(1)
                if holes and rnd.random() < 0.03:
                    ty.append(rnd.randrange(3))
                    mk.append(0)
        text(rnd.randint(1, 12))
        for _ in range(runs):
            side = lambda: merge * rnd.randint(1, max_side) + (1 if rnd.random() < 0.2 else 0)
            if rnd.random() < 0.6:
                g = (rnd.choice((1, 1, 2)), side(), side())
                imgs.append(g)
                n = _vision_tokens(*g, merge)
                ty += [1] * n
                mk += [1] * n
            else:
                t, h, w = rnd.randint(1, 4), side(), side()
                vids.append((t, h, w))
                for f in range(t):
                    if f:
                        text(rnd.randint(1, 3))
                    n = _vision_tokens(1, h, w, merge)
                    ty += [2] * n
                    mk += [1] * n
            text(rnd.randint(1, 12))
        seqs.append(ty)
        masks.append(mk)
    S = max(len(s) for s in seqs) + rnd.randint(0, pad_max)
    types = np.zeros((B, S), dtype=np.int32)
    mask = np.zeros((B, S), dtype=np.int32)
    for b, (ty, mk) in enumerate(zip(seqs, masks)):
        off = S - len(ty)
        types[b, :off] = [rnd.randrange(3) for _ in range(off)]
        types[b, off:] = ty
        mask[b, off:] = mk
    return {"types": types, "mask": mask,
            "image_thw": np.array(imgs, dtype=np.int64).reshape(-1, 3),
            "video_thw": np.array(vids, dtype=np.int64).reshape(-1, 3)}


def rope_index_fixture_cases():
    """(name, layout, merge) of the get_rope_index fixture."""
    import numpy as np
    text_only = {"types": np.zeros((1, 37), np.int32), "mask": None,
                 "image_thw": np.zeros((0, 3), np.int64), "video_thw": np.zeros((0, 3), np.int64)}
    two_images = {"types": np.array([[0] * 5 + [1] * 24 + [0] * 3 + [1] * 6 + [0] * 7], np.int32),
                  "mask": None, "image_thw": np.array([[1, 8, 12], [1, 6, 4]], np.int64),
                  "video_thw": np.zeros((0, 3), np.int64)}
    return [("text_only", text_only, 2),
            ("two_images", two_images, 2),
            ("mixed_b2", rope_index_layout(11, 2, 3), 2),
            ("mixed_b3_nohole", rope_index_layout(12, 3, 4, holes=False), 2),
            ("mixed_b4_merge1", rope_index_layout(13, 4, 2, merge=1, max_side=5), 1),
            ("mixed_b2_long", rope_index_layout(14, 2, 12), 2)]


def hf_rope_index(layout, merge):
    """transformers 5.5.0 Qwen3VLModel.get_rope_index, called on an object that
    carries only what the method reads (config.vision_config.spatial_merge_size
    and get_vision_position_ids), so no model weights are built."""
    import functools
    import types as pytypes
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLModel
    host = pytypes.SimpleNamespace(
        config=pytypes.SimpleNamespace(
            vision_config=pytypes.SimpleNamespace(spatial_merge_size=merge)))
    host.get_vision_position_ids = functools.partial(Qwen3VLModel.get_vision_position_ids, host)
    ty = torch.from_numpy(layout["types"]).long()
    mask = None if layout["mask"] is None else torch.from_numpy(layout["mask"]).long()
    img = torch.from_numpy(layout["image_thw"]) if len(layout["image_thw"]) else None
    vid = torch.from_numpy(layout["video_thw"]).clone() if len(layout["video_thw"]) else None
    ids = torch.zeros_like(ty)
    pos, delta = Qwen3VLModel.get_rope_index(host, ids, ty, img, vid, mask)
    return pos, delta.reshape(-1)


def rope_index_checksum() -> int:
    """Position-weighted sum over every fixture layout (catches a changed generator)."""
    import numpy as np
    total = 0
    for _, lay, merge in rope_index_fixture_cases():
        for a in (lay["types"], lay["mask"], lay["image_thw"], lay["video_thw"]):
            if a is not None and a.size:
                w = np.arange(1, a.size + 1, dtype=np.int64)
                total += int((a.reshape(-1).astype(np.int64) * w).sum())
        total += merge
    return total


# ---- vision tower: a small Qwen3VLVisionModel with the real head_dim (72) ----
VISION_TINY = dict(depth=3, hidden_size=144, num_heads=2, intermediate_size=256,
                   out_hidden_size=128, num_position_embeddings=64, patch_size=16,
                   temporal_patch_size=2, in_channels=3, spatial_merge_size=2,
                   deepstack_visual_indexes=[0, 2])
VISION_GRIDS = [[1, 8, 12], [2, 6, 4]]     # an image and a two-frame clip


def vision_tiny_weights(seed: int = 31) -> dict:
    """Seeded fp32 weights of VISION_TINY (see vision_weights)."""
    return vision_weights(VISION_TINY, seed)


def vision_weights(c: dict, seed: int) -> dict:
    """Seeded fp32 weights named as Qwen3VLVisionModel.state_dict() for config
    dict `c` (N(0, 0.05) matrices, N(0, 0.02) biases, LayerNorm weights near 1)."""
    g = torch.Generator().manual_seed(seed)
    H, I, O = c["hidden_size"], c["intermediate_size"], c["out_hidden_size"]
    M = H * c["spatial_merge_size"] ** 2
    inp = c["in_channels"] * c["temporal_patch_size"] * c["patch_size"] ** 2

    def mat(o, i, std=0.05):
        return torch.randn(o, i, generator=g) * std

    def vec(n, std=0.02, base=0.0):
        return base + torch.randn(n, generator=g) * std

    p = {"patch_embed.proj.weight": mat(H, inp, 0.03).view(H, c["in_channels"],
                                                           c["temporal_patch_size"],
                                                           c["patch_size"], c["patch_size"]),
         "patch_embed.proj.bias": vec(H),
         "pos_embed.weight": torch.randn(c["num_position_embeddings"], H, generator=g) * 0.5}
    for i in range(c["depth"]):
        b = f"blocks.{i}."
        p.update({b + "norm1.weight": vec(H, 0.1, 1.0), b + "norm1.bias": vec(H),
                  b + "norm2.weight": vec(H, 0.1, 1.0), b + "norm2.bias": vec(H),
                  b + "attn.qkv.weight": mat(3 * H, H), b + "attn.qkv.bias": vec(3 * H),
                  b + "attn.proj.weight": mat(H, H), b + "attn.proj.bias": vec(H),
                  b + "mlp.linear_fc1.weight": mat(I, H), b + "mlp.linear_fc1.bias": vec(I),
                  b + "mlp.linear_fc2.weight": mat(H, I), b + "mlp.linear_fc2.bias": vec(H)})
    mergers = ["merger."] + [f"deepstack_merger_list.{j}."
                             for j in range(len(c["deepstack_visual_indexes"]))]
    for j, m in enumerate(mergers):
        n = H if j == 0 else M
        p.update({m + "norm.weight": vec(n, 0.1, 1.0), m + "norm.bias": vec(n),
                  m + "linear_fc1.weight": mat(M, M), m + "linear_fc1.bias": vec(M),
                  m + "linear_fc2.weight": mat(O, M), m + "linear_fc2.bias": vec(O)})
    return p


def vision_tiny_inputs(seed: int = 32):
    """Flattened patches [N, C*T*P*P] ~ N(0, 1) and grid_thw int64 [2, 3]."""
    c = VISION_TINY
    grid = torch.tensor(VISION_GRIDS, dtype=torch.int64)
    n = int((grid[:, 0] * grid[:, 1] * grid[:, 2]).sum())
    g = torch.Generator().manual_seed(seed)
    inp = c["in_channels"] * c["temporal_patch_size"] * c["patch_size"] ** 2
    return torch.randn(n, inp, generator=g), grid


def hf_vision_tiny(dtype=torch.float32):
    """transformers 5.5.0 Qwen3VLVisionModel (eager attention) on the seeded
    weights and inputs: (pooler_output, deepstack features, last_hidden_state)."""
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionModel
    cfg = Qwen3VLVisionConfig(**VISION_TINY)
    cfg._attn_implementation = "eager"
    model = Qwen3VLVisionModel(cfg).eval()
    missing, unexpected = model.load_state_dict(vision_tiny_weights(), strict=True)
    assert not missing and not unexpected
    model = model.to(dtype)
    # from_pretrained(dtype=bf16), as the reference loads the model
    # (loader_fused.py:56-58), keeps this buffer fp32 (_init_weights
    # computes it in float); .to(dtype) would round it
    rot = model.rotary_pos_emb
    rot.inv_freq = 1.0 / (rot.theta ** (torch.arange(0, rot.dim, 2, dtype=torch.float) / rot.dim))
    x, grid = vision_tiny_inputs()
    with torch.no_grad():
        out = model(x.to(dtype), grid_thw=grid)
    return out.pooler_output, list(out.deepstack_features), out.last_hidden_state


# ---- the drop-in vision.py: the reference's prepare_vision_embeds end to end ----
DROPIN_TEXT = dict(hidden_size=128, num_attention_heads=1, num_key_value_heads=1, head_dim=128,
                   intermediate_size=256, num_hidden_layers=1, vocab_size=151936,
                   rms_norm_eps=1e-6,
                   rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                    "mrope_section": [24, 20, 20], "mrope_interleaved": True})
DROPIN_CASES = ("image", "video_short", "image_video")
IMAGE_TOKEN, VIDEO_TOKEN = 151655, 151656


def dropin_embed_table(seed: int = 41) -> torch.Tensor:
    """bf16 [151936, 128] text embeddings of the drop-in model."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(DROPIN_TEXT["vocab_size"], 128, generator=g) * 0.5).to(BF16)


def dropin_hf_model():
    """A seeded transformers 5.5.0 Qwen3VLForConditionalGeneration in bf16 with
    eager attention: VISION_TINY's tower (out width 128) over a one-layer text
    model with the real vocabulary, so the image / video token ids embed.
    Only the tower and the embeddings are used by prepare_vision_embeds."""
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration
    cfg = Qwen3VLConfig(text_config=dict(DROPIN_TEXT), vision_config=dict(VISION_TINY))
    for c in (cfg, cfg.text_config, cfg.vision_config):
        c._attn_implementation = "eager"
    model = Qwen3VLForConditionalGeneration(cfg).eval()
    missing, unexpected = model.model.visual.load_state_dict(vision_tiny_weights(), strict=True)
    assert not missing and not unexpected
    model = model.to(BF16)
    with torch.no_grad():
        model.model.language_model.embed_tokens.weight.copy_(dropin_embed_table())
    # from_pretrained(dtype=bf16) keeps this buffer fp32
    rot = model.model.visual.rotary_pos_emb
    rot.inv_freq = 1.0 / (rot.theta ** (torch.arange(0, rot.dim, 2, dtype=torch.float) / rot.dim))
    return model


def dropin_inputs(name: str) -> dict:
    """Processor-style inputs: input_ids [1, S] with <image> / <video> runs,
    flattened patches and grids (VISION_TINY's image and clip).  video_short
    has 10 <video> positions for the clip's 12 features (the reference fills
    10 and cuts the deepstack rows to 10)."""
    x, grid = vision_tiny_inputs()
    img_px, vid_px = x[:96], x[96:]
    g = torch.Generator().manual_seed(43 + DROPIN_CASES.index(name))

    def text(n):
        return torch.randint(0, 151000, (n,), generator=g)

    def run(tok, n):
        return torch.full((n,), tok, dtype=torch.int64)

    if name == "image":
        ids = torch.cat([text(5), run(IMAGE_TOKEN, 24), text(7)])
        return dict(input_ids=ids[None], pixel_values=img_px, image_grid_thw=grid[:1])
    if name == "video_short":
        ids = torch.cat([text(3), run(VIDEO_TOKEN, 10), text(4)])
        return dict(input_ids=ids[None], pixel_values_videos=vid_px, video_grid_thw=grid[1:])
    if name == "image_video":
        ids = torch.cat([text(2), run(IMAGE_TOKEN, 24), text(3), run(VIDEO_TOKEN, 12), text(5)])
        return dict(input_ids=ids[None], pixel_values=img_px, image_grid_thw=grid[:1],
                    pixel_values_videos=vid_px, video_grid_thw=grid[1:])
    raise KeyError(name)


# ---- a4 + a12: one text decoder layer with interleaved M-RoPE (transformers) ----
MROPE_LAYER_SPEC = odec.Spec(hidden=512, q_heads=4, kv_heads=1, inter=1024, vocab=64, layers=1,
                             max_seq=512)
MROPE_LAYER_S = 300


def mrope_layer_case(seed: int = 17):
    """Seeded layer weights (HF [out, in] convention, random norms), hidden
    states [1, 300, 512] and the text / 16x16 image / text position ids."""
    w = odec.make_weights(MROPE_LAYER_SPEC, seed=seed, std=0.05, random_norms=True)
    g = torch.Generator().manual_seed(seed + 1)
    hidden = torch.randn(1, MROPE_LAYER_S, 512, generator=g).to(BF16)
    pos = oref.config2_position_ids(seq=MROPE_LAYER_S)
    return w["layers"][0], hidden, pos


def hf_mrope_layer(dtype=torch.float32):
    """transformers 5.5.0 Qwen3VLTextDecoderLayer (eager attention, causal mask)
    with Qwen3VLTextRotaryEmbedding on mrope_layer_case()'s inputs."""
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import (Qwen3VLTextDecoderLayer,
                                                                Qwen3VLTextRotaryEmbedding)
    s = MROPE_LAYER_SPEC
    cfg = Qwen3VLTextConfig(hidden_size=s.hidden, num_attention_heads=s.q_heads,
                            num_key_value_heads=s.kv_heads, head_dim=128,
                            intermediate_size=s.inter, rms_norm_eps=s.eps,
                            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                                             "mrope_section": [24, 20, 20],
                                             "mrope_interleaved": True})
    cfg._attn_implementation = "eager"
    lw, hidden, pos = mrope_layer_case()
    layer = Qwen3VLTextDecoderLayer(cfg, 0).eval()
    sd = {"self_attn.q_proj.weight": lw["q"], "self_attn.k_proj.weight": lw["k"],
          "self_attn.v_proj.weight": lw["v"], "self_attn.o_proj.weight": lw["o"],
          "self_attn.q_norm.weight": lw["q_norm"], "self_attn.k_norm.weight": lw["k_norm"],
          "mlp.gate_proj.weight": lw["gate"], "mlp.up_proj.weight": lw["up"],
          "mlp.down_proj.weight": lw["down"], "input_layernorm.weight": lw["input_norm"],
          "post_attention_layernorm.weight": lw["post_norm"]}
    layer.load_state_dict({k: v.float() for k, v in sd.items()}, strict=True)
    layer = layer.to(dtype)
    rot = Qwen3VLTextRotaryEmbedding(cfg)
    x = hidden.to(dtype)
    cos, sin = rot(x, pos)
    S = x.shape[1]
    mask = torch.full((S, S), float("-inf"), dtype=dtype).triu(1)[None, None]
    with torch.no_grad():
        out = layer(x, position_embeddings=(cos, sin), attention_mask=mask)
    return out, cos, sin


# ---- a4 + a13 + 8(f)2: multimodal prefill and one decode step (transformers) ----
MM_PROMPT = dict(text0=6, grid=(1, 12, 12), text1=18)   # 6 + 36 image tokens + 18 = 60


def mm_decode_case(seed: int = 23):
    """Inputs of the multimodal prefill + decode fixture on the tiny TP1
    decoder's weights: inputs_embeds [1, 60, 512] (text rows from the
    embedding, image rows random), 3-axis position ids and rope delta (from
    the oracle's get_rope_index), the visual mask and two deepstack levels."""
    import numpy as np
    w = decoder_weights("decoder_tiny_tp1")
    t0, (gt, gh, gw), t1 = MM_PROMPT["text0"], MM_PROMPT["grid"], MM_PROMPT["text1"]
    n_img = gt * (gh // 2) * (gw // 2)
    P = t0 + n_img + t1
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 1024, (1, P), generator=g)
    emb = w["embed"][ids].clone()
    types = np.zeros((1, P), np.int32)
    types[0, t0:t0 + n_img] = 1
    mask = torch.from_numpy(types[0] == 1)
    emb[0, mask] = (torch.randn(n_img, 512, generator=g) * 0.05).to(BF16)
    deep = [(torch.randn(n_img, 512, generator=g) * 0.05).to(BF16) for _ in range(2)]
    pos, delta = oref.rope_index(types, None, np.array([[gt, gh, gw]]), None, 2)
    return w, emb, pos, int(delta[0]), mask, deep


def hf_mm_decode():
    """transformers 5.5.0 Qwen3VLTextModel (eager, bf16) on mm_decode_case():
    the multimodal prefill with deepstack, then one cached decode step at
    position P + delta on all three axes.  Greedy tokens use the decoder's
    lm_head on the returned hidden states."""
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel
    spec = DECODER_CASES["decoder_tiny_tp1"]["spec"]
    w, emb, pos, delta, mask, deep = mm_decode_case()
    cfg = Qwen3VLTextConfig(hidden_size=spec.hidden, num_attention_heads=spec.q_heads,
                            num_key_value_heads=spec.kv_heads, head_dim=128,
                            intermediate_size=spec.inter, num_hidden_layers=spec.layers,
                            vocab_size=spec.vocab, rms_norm_eps=spec.eps,
                            rope_parameters={"rope_type": "default", "rope_theta": spec.rope_theta,
                                             "mrope_section": [24, 20, 20],
                                             "mrope_interleaved": True})
    cfg._attn_implementation = "eager"
    model = Qwen3VLTextModel(cfg).eval()
    sd = {"embed_tokens.weight": w["embed"], "norm.weight": w["final_norm"]}
    for i, lw in enumerate(w["layers"]):
        p = f"layers.{i}."
        sd.update({p + "self_attn.q_proj.weight": lw["q"], p + "self_attn.k_proj.weight": lw["k"],
                   p + "self_attn.v_proj.weight": lw["v"], p + "self_attn.o_proj.weight": lw["o"],
                   p + "self_attn.q_norm.weight": lw["q_norm"],
                   p + "self_attn.k_norm.weight": lw["k_norm"],
                   p + "mlp.gate_proj.weight": lw["gate"], p + "mlp.up_proj.weight": lw["up"],
                   p + "mlp.down_proj.weight": lw["down"],
                   p + "input_layernorm.weight": lw["input_norm"],
                   p + "post_attention_layernorm.weight": lw["post_norm"]})
    model.load_state_dict({k: v.float() for k, v in sd.items()}, strict=True)
    model = model.to(BF16)
    # keep the rotary frequencies fp32, as from_pretrained(dtype=bf16) leaves them
    inv = model.rotary_emb.inv_freq
    model.rotary_emb.inv_freq = 1.0 / (spec.rope_theta ** (
        torch.arange(0, 128, 2, dtype=torch.float) / 128))
    assert inv.shape == model.rotary_emb.inv_freq.shape
    P = emb.shape[1]
    with torch.no_grad():
        out = model(inputs_embeds=emb, position_ids=pos, use_cache=True,
                    visual_pos_masks=mask[None], deepstack_visual_embeds=deep)
        h_pre = out.last_hidden_state
        t0 = int((h_pre[0, -1] @ w["lm_head"].t()).float().argmax())
        x1 = w["embed"][torch.tensor([[t0]])]
        p1 = torch.full((3, 1, 1), P + delta, dtype=torch.long)
        out1 = model(inputs_embeds=x1, position_ids=p1, past_key_values=out.past_key_values,
                     use_cache=True)
        h_dec = out1.last_hidden_state
        t1 = int((h_dec[0, -1] @ w["lm_head"].t()).float().argmax())
    return h_pre, h_dec, [t0, t1]
