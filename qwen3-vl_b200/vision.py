"""Vision encoder integration for Qwen3-VL with deepstack: drop-in for the
reference's vision.py.

prepare_vision_embeds(hf_model, processor, inputs, device) has the reference's
signature and return values (vision.py:15-140): merged input embeddings
[1, S, H], the deepstack feature list (one [n_visual, H] tensor per level) and
the visual-token mask [S].  The vision tower runs on the q3vl kernels
(q3vl.vision_tower.VisionTower, built once from hf_model's vision module), and
the text embeddings on the q3vl embedding kernel, instead of transformers'
eager modules.

The merge rules are the reference's, kept for parity of the returned tensors:
  - batch row 0 only; image features fill the <image> positions (151655) when
    the features cover them (vision.py:57-70);
  - video features fill the first n = min(features, <video> positions) of the
    <video> positions (151656), and the video deepstack rows are cut to the
    same n (vision.py:95-109);
  - with both images and video, each deepstack level is rebuilt over all
    visual positions, image rows at image positions and video rows at the
    filled video positions (vision.py:110-129).
"""
from __future__ import annotations

import os

import torch

from q3vl import ops
from q3vl.vision_tower import VisionTower

IMAGE_TOKEN_ID = 151655
VIDEO_TOKEN_ID = 151656


def vision_tower_for(hf_model, device) -> VisionTower:
    """The q3vl tower for hf_model's vision module (built on first use)."""
    visual = hf_model.model.visual if hasattr(hf_model.model, "visual") else hf_model.visual
    dev = torch.device(device)
    tower = getattr(visual, "_q3vl_tower", None)
    if tower is None or tower.device != dev:
        tower = VisionTower.from_hf(visual, dev)
        visual._q3vl_tower = tower
    return tower


def _encode(tower, pixels, grid):
    """The tower on every rank (replicated, as the reference runs it), or with
    Q3VL_VISION_DP=1 and a process group of several ranks, data parallel: each
    rank encodes its share of the images and the outputs are all-gathered
    (every rank must then call prepare_vision_embeds, as SPMD serving does)."""
    import torch.distributed as dist
    if (os.environ.get("Q3VL_VISION_DP", "0") == "1" and dist.is_initialized()
            and dist.get_world_size() > 1):
        return tower.forward_sharded(pixels, grid)
    return tower(pixels, grid)


def _embed_table(hf_model):
    emb = hf_model.model.language_model.embed_tokens
    return emb.weight if hasattr(emb, "weight") else emb


def prepare_vision_embeds(hf_model, processor, inputs, device):
    """Run the vision tower and merge its embeddings into the text sequence.

    Returns (inputs_embeds [1, S, H], deepstack_embeds list or None,
    visual_mask [S] bool or None), as the reference does."""
    input_ids = inputs["input_ids"].to(device)
    pixel_values = inputs.get("pixel_values")
    image_grid_thw = inputs.get("image_grid_thw")
    pixel_values_videos = inputs.get("pixel_values_videos")
    video_grid_thw = inputs.get("video_grid_thw")

    table = _embed_table(hf_model).to(device)
    inputs_embeds = ops.embed(input_ids, table.to(torch.bfloat16).contiguous())
    image = video = None
    if pixel_values is not None and image_grid_thw is not None:
        feats, deep, _ = _encode(vision_tower_for(hf_model, device), pixel_values,
                                 image_grid_thw)
        image = (feats, deep)
    if pixel_values_videos is not None and video_grid_thw is not None:
        feats, deep, _ = _encode(vision_tower_for(hf_model, device), pixel_values_videos,
                                 video_grid_thw)
        video = (feats, deep)
    return merge_vision(inputs_embeds, input_ids[0], image, video)


def merge_vision(inputs_embeds, ids0, image=None, video=None):
    """The reference's merge of the tower outputs into batch row 0 of the text
    embeddings (vision.py:57-129).  image / video: (features [n, H], deepstack
    levels) from one tower call each, or None.  inputs_embeds is updated in
    place.  Returns (inputs_embeds, deepstack list or None, visual_mask or
    None)."""
    device = inputs_embeds.device
    dtype = inputs_embeds.dtype
    visual_mask = torch.zeros(ids0.shape[-1], dtype=torch.bool, device=device)
    deepstack = []

    if image is not None:
        feats, img_deep = image
        image_mask = ids0 == IMAGE_TOKEN_ID
        n_img = int(image_mask.sum())
        if n_img > 0 and feats.shape[0] >= n_img:
            inputs_embeds[0, image_mask] = feats[:n_img].to(dtype)
            visual_mask |= image_mask
            deepstack = [d[:n_img].to(dtype) for d in img_deep]

    if video is not None:
        vfeats, vid_deep = video
        video_mask = ids0 == VIDEO_TOKEN_ID
        n_fill = min(int(vfeats.shape[0]), int(video_mask.sum()))
        if n_fill > 0:
            vid_pos = video_mask.nonzero(as_tuple=True)[0][:n_fill]
            fill = torch.zeros_like(video_mask)
            fill[vid_pos] = True
            inputs_embeds[0, fill] = vfeats[:n_fill].to(dtype)
            visual_mask |= fill
            if vid_deep:
                if deepstack:
                    deepstack = _combine_levels(deepstack, vid_deep, ids0, visual_mask, vid_pos,
                                                dtype, device)
                else:
                    deepstack = [d[:n_fill].to(dtype) for d in vid_deep]

    return (inputs_embeds, deepstack if deepstack else None,
            visual_mask if bool(visual_mask.any()) else None)


def _combine_levels(img_levels, vid_levels, ids0, visual_mask, vid_pos, dtype, device):
    """Deepstack levels over every visual position: image rows at the image
    positions, video rows at the filled video positions (rows past a level's
    length stay zero), as vision.py:110-129 builds them."""
    vis = visual_mask.nonzero(as_tuple=True)[0]
    row_of = torch.full((ids0.shape[-1],), -1, dtype=torch.long, device=device)
    row_of[vis] = torch.arange(vis.numel(), device=device)
    img_pos = (ids0 == IMAGE_TOKEN_ID).nonzero(as_tuple=True)[0]
    out = list(img_levels)
    for idx, vlevel in enumerate(vid_levels):
        combined = torch.zeros(vis.numel(), vlevel.shape[-1], dtype=dtype, device=device)
        if idx < len(img_levels):
            lvl = img_levels[idx]
            n = min(img_pos.numel(), lvl.shape[0])
            rows = row_of[img_pos[:n]]
            keep = rows >= 0
            combined[rows[keep]] = lvl[:n][keep]
        n = min(vid_pos.numel(), vlevel.shape[0])
        rows = row_of[vid_pos[:n]]
        keep = rows >= 0
        combined[rows[keep]] = vlevel[:n][keep].to(dtype)
        if idx < len(out):
            out[idx] = combined
        else:
            out.append(combined)
    return out
