"""Qwen3-VL vision tower on the q3vl kernels.

The reference runs transformers' Qwen3VLVisionModel eagerly (vision.py:51-53,
:74-76).  This module takes that model's weights (its state_dict, or the module
itself) and runs the same computation (transformers 5.5.0
modeling_qwen3_vl.py:616-823) on the library's sm_100a kernels:

  patch embed + position embeddings   q3_vision_pos_embed, then q3_gemm_bias
                                      (the Conv3d as a GEMM, bias and the
                                      position-embedding add in its epilogue)
  27 blocks                           q3_layernorm -> q3_gemm_bias(qkv) ->
                                      q3_vision_rope (in place) ->
                                      q3_vision_attention -> q3_gemm_bias(proj,
                                      + residual) -> q3_layernorm ->
                                      q3_gemm_bias(fc1, gelu tanh) ->
                                      q3_gemm_bias(fc2, + residual)
  mergers (final, deepstack)          q3_layernorm + two q3_gemm_bias (erf GELU)

The per-call plan (which token belongs to which image and frame, and the
128-row query blocks of every frame) is built on the host from grid_thw, as
the reference does, and uploaded once per forward.  Everything else runs on
the device; there is no CPU fallback.
"""
from __future__ import annotations

import torch

from . import ops

_DEFAULTS = dict(depth=27, hidden_size=1152, num_heads=16, intermediate_size=4304,
                 out_hidden_size=4096, num_position_embeddings=2304, patch_size=16,
                 temporal_patch_size=2, in_channels=3, spatial_merge_size=2,
                 deepstack_visual_indexes=(8, 16, 24))


def _cfg_get(cfg, name):
    if cfg is None:
        return _DEFAULTS[name]
    if isinstance(cfg, dict):
        return cfg.get(name, _DEFAULTS[name])
    return getattr(cfg, name, _DEFAULTS[name])


def shard_images(grid_thw, world: int, rank: int, merge: int = 2):
    """Contiguous split of the images over `world` ranks, balanced by patch
    count.  Returns (first image, end image, first patch, end patch, merged
    token offsets of every rank's share) for `rank`; the offsets list has
    world + 1 entries (merged tokens = patches / merge^2)."""
    grid = [tuple(int(v) for v in g) for g in
            (grid_thw.tolist() if hasattr(grid_thw, "tolist") else grid_thw)]
    sizes = [t * h * w for t, h, w in grid]
    total = sum(sizes)
    bounds, acc, img = [0], 0, 0
    for r in range(1, world):
        target = total * r / world
        while img < len(sizes) and acc + sizes[img] / 2 <= target:
            acc += sizes[img]
            img += 1
        bounds.append(img)
    bounds.append(len(sizes))
    patch_off = [0]
    for s in sizes:
        patch_off.append(patch_off[-1] + s)
    mm = merge * merge
    merged = [patch_off[b] // mm for b in bounds]
    i0, i1 = bounds[rank], bounds[rank + 1]
    return i0, i1, patch_off[i0], patch_off[i1], merged


def gather_rows(local: torch.Tensor, merged_offsets, group=None) -> torch.Tensor:
    """All-gather every rank's rows [n_r, width] into [sum n_r, width] in rank
    order (shares differ in size: rows are padded to the largest share)."""
    import torch.distributed as dist
    world = len(merged_offsets) - 1
    counts = [merged_offsets[r + 1] - merged_offsets[r] for r in range(world)]
    pad = max(counts)
    buf = torch.zeros(pad, local.shape[1], dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([parts[r][:counts[r]] for r in range(world)])


class VisionPlan:
    """Host-built token layout of one forward: image table [n_img, 4] =
    (t, h, w, first token) and query blocks [n_blocks, 3] = (frame first
    token, frame length, first query row), on the host and the device."""

    def __init__(self, grid_thw, merge: int, device):
        grid = [tuple(int(v) for v in g) for g in
                (grid_thw.tolist() if hasattr(grid_thw, "tolist") else grid_thw)]
        imgs, blocks, first = [], [], 0
        for t, h, w in grid:
            if h % merge or w % merge:
                raise ValueError(f"vision grid {t}x{h}x{w} is not a multiple of merge {merge}")
            imgs.append((t, h, w, first))
            for f in range(t):
                f0 = first + f * h * w
                for q0 in range(0, h * w, 128):
                    blocks.append((f0, h * w, q0))
            first += t * h * w
        self.n_tok = first
        self.imgs_host = torch.tensor(imgs, dtype=torch.int32).reshape(-1, 4)
        self.blocks_host = torch.tensor(blocks, dtype=torch.int32).reshape(-1, 3)
        both = torch.cat([self.imgs_host.reshape(-1), self.blocks_host.reshape(-1)])
        dev = both.to(device, non_blocking=False)
        self.imgs = dev[:self.imgs_host.numel()].view(-1, 4)
        self.blocks = dev[self.imgs_host.numel():].view(-1, 3)


class VisionTower:
    """Qwen3VLVisionModel forward on the q3vl kernels (bf16).

    `weights` is a state_dict with the HF module's names; `config` any object
    or dict with the HF vision config fields."""

    def __init__(self, weights: dict, config=None, device="cuda"):
        g = lambda n: _cfg_get(config, n)  # noqa: E731
        self.depth, self.hidden, self.heads = g("depth"), g("hidden_size"), g("num_heads")
        self.merge = g("spatial_merge_size")
        self.deepstack = tuple(g("deepstack_visual_indexes"))
        self.head_dim = self.hidden // self.heads
        if self.head_dim != 72:
            raise ValueError(f"vision head_dim {self.head_dim} unsupported (kernels are built "
                             f"for 72)")
        self.device = torch.device(device)
        dev, bf = self.device, torch.bfloat16

        def w(name):
            return weights[name].to(dev, bf).contiguous()

        pw = weights["patch_embed.proj.weight"]
        self.patch_w = pw.reshape(pw.shape[0], -1).to(dev, bf).contiguous()
        self.patch_b = w("patch_embed.proj.bias")
        self.pos_table = w("pos_embed.weight")
        # rotary frequencies as the HF module computes them (fp32)
        dim = self.head_dim // 2
        self.inv_freq = (1.0 / (10000.0 ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
                         ).to(dev)
        names = ("norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias", "attn.qkv.weight",
                 "attn.qkv.bias", "attn.proj.weight", "attn.proj.bias", "mlp.linear_fc1.weight",
                 "mlp.linear_fc1.bias", "mlp.linear_fc2.weight", "mlp.linear_fc2.bias")
        self.blocks = [{n: w(f"blocks.{i}.{n}") for n in names} for i in range(self.depth)]
        mnames = ("norm.weight", "norm.bias", "linear_fc1.weight", "linear_fc1.bias",
                  "linear_fc2.weight", "linear_fc2.bias")
        self.merger = {n: w("merger." + n) for n in mnames}
        self.ds_mergers = [{n: w(f"deepstack_merger_list.{j}.{n}") for n in mnames}
                           for j in range(len(self.deepstack))]

    @classmethod
    def from_hf(cls, visual, device=None):
        """Build from a transformers Qwen3VLVisionModel instance."""
        dev = device if device is not None else next(visual.parameters()).device
        return cls({k: v.detach() for k, v in visual.state_dict().items()}, visual.config, dev)

    def _merge(self, x, m, postshuffle):
        width = self.hidden * self.merge * self.merge
        if postshuffle:
            y = ops.layernorm(x.view(-1, width), m["norm.weight"], m["norm.bias"])
        else:
            y = ops.layernorm(x, m["norm.weight"], m["norm.bias"]).view(-1, width)
        f = ops.gemm_bias(y, m["linear_fc1.weight"], m["linear_fc1.bias"], "bias_gelu")
        return ops.gemm_bias(f, m["linear_fc2.weight"], m["linear_fc2.bias"], "bias")

    @torch.no_grad()
    def forward(self, pixel_values: torch.Tensor, grid_thw):
        """pixel_values [N, C*T*P*P] (the processor's flattened patches), grid_thw
        [n, 3] -> (pooler_output [N / merge^2, out], [deepstack features],
        last_hidden_state [N, hidden]), all bf16 on the device."""
        plan = VisionPlan(grid_thw, self.merge, self.device)
        n = plan.n_tok
        if pixel_values.shape[0] != n:
            raise ValueError(f"pixel_values has {pixel_values.shape[0]} patches, grid_thw {n}")
        x = pixel_values.to(self.device, torch.bfloat16).contiguous()
        pos = ops.vision_pos_embed(self.pos_table, plan.imgs, plan.imgs_host, self.merge, n)
        h = ops.gemm_bias(x, self.patch_w, self.patch_b, "bias_residual", residual=pos)
        feats = []
        for i, b in enumerate(self.blocks):
            t = ops.layernorm(h, b["norm1.weight"], b["norm1.bias"])
            qkv = ops.gemm_bias(t, b["attn.qkv.weight"], b["attn.qkv.bias"], "bias")
            ops.vision_rope(qkv, self.heads, self.inv_freq, plan.imgs, plan.imgs_host, self.merge)
            o = ops.vision_attention(qkv, self.heads, plan.blocks, plan.blocks_host)
            h = ops.gemm_bias(o, b["attn.proj.weight"], b["attn.proj.bias"], "bias_residual",
                              residual=h, out=h)
            t = ops.layernorm(h, b["norm2.weight"], b["norm2.bias"])
            f = ops.gemm_bias(t, b["mlp.linear_fc1.weight"], b["mlp.linear_fc1.bias"],
                              "bias_gelu_tanh")
            h = ops.gemm_bias(f, b["mlp.linear_fc2.weight"], b["mlp.linear_fc2.bias"],
                              "bias_residual", residual=h, out=h)
            if i in self.deepstack:
                feats.append(self._merge(h, self.ds_mergers[self.deepstack.index(i)], True))
        return self._merge(h, self.merger, False), feats, h

    @torch.no_grad()
    def forward_sharded(self, pixel_values: torch.Tensor, grid_thw, group=None):
        """forward() with the images split over the ranks of `group` (data
        parallel: each rank encodes its share, then the merged outputs are
        all-gathered).  Every rank returns the full pooler output and
        deepstack features, as forward() would; the last hidden state is
        this rank's share only."""
        import torch.distributed as dist
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        if world == 1:
            return self.forward(pixel_values, grid_thw)
        rank = dist.get_rank(group)
        grid = grid_thw.tolist() if hasattr(grid_thw, "tolist") else list(grid_thw)
        i0, i1, p0, p1, merged = shard_images(grid, world, rank, self.merge)
        if i1 > i0:
            pooler, feats, last = self.forward(pixel_values[p0:p1], grid[i0:i1])
        else:
            out_w = self.merger["linear_fc2.weight"].shape[0]
            pooler = torch.empty(0, out_w, dtype=torch.bfloat16, device=self.device)
            feats = [torch.empty(0, out_w, dtype=torch.bfloat16, device=self.device)
                     for _ in self.deepstack]
            last = torch.empty(0, self.hidden, dtype=torch.bfloat16, device=self.device)
        pooler = gather_rows(pooler, merged, group)
        feats = [gather_rows(f, merged, group) for f in feats]
        return pooler, feats, last

    __call__ = forward
