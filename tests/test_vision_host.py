"""Host-side parts of the vision path (no GPU): the per-call plan built from
grid_thw, the deepstack level merge of prepare_vision_embeds, and argument
checks of the vision entry points."""
import ctypes

import pytest
import torch

from q3vl import _lib
from q3vl.vision_tower import VisionPlan


def test_plan_lists_images_and_128_row_blocks_of_every_frame():
    plan = VisionPlan(torch.tensor([[1, 8, 12], [2, 6, 4], [1, 16, 18]]), 2, "cpu")
    assert plan.n_tok == 96 + 48 + 288
    assert plan.imgs_host.tolist() == [[1, 8, 12, 0], [2, 6, 4, 96], [1, 16, 18, 144]]
    blocks = plan.blocks_host.tolist()
    assert blocks[:1] == [[0, 96, 0]]                     # one block: 96 rows
    assert blocks[1:3] == [[96, 24, 0], [120, 24, 0]]     # two frames of 24
    assert blocks[3:] == [[144, 288, 0], [144, 288, 128], [144, 288, 256]]
    assert torch.equal(plan.imgs.cpu(), plan.imgs_host)


def test_plan_rejects_grids_off_the_merge_size():
    with pytest.raises(ValueError, match="merge"):
        VisionPlan([[1, 7, 8]], 2, "cpu")


def _reference_combine(img_levels, vid_levels, ids0, visual_mask, vid_pos, dtype):
    """The loops of the reference's vision.py:110-129, transcribed for the check."""
    vis = visual_mask.nonzero(as_tuple=True)[0]
    img_pos = (ids0 == 151655).nonzero(as_tuple=True)[0]
    out = list(img_levels)
    for idx in range(len(vid_levels)):
        combined = torch.zeros(vis.shape[0], vid_levels[idx].shape[-1], dtype=dtype)
        pos_to_row = {int(p): r for r, p in enumerate(vis.tolist())}
        for j, pos in enumerate(img_pos.tolist()):
            r = pos_to_row.get(pos)
            if r is not None and idx < len(out) and j < img_levels[idx].shape[0]:
                combined[r] = img_levels[idx][j]
        for j, pos in enumerate(vid_pos.tolist()):
            r = pos_to_row.get(pos)
            if r is not None and j < vid_levels[idx].shape[0]:
                combined[r] = vid_levels[idx][j].to(dtype)
        if idx < len(out):
            out[idx] = combined
        else:
            out.append(combined)
    return out


def test_deepstack_levels_combine_like_the_reference():
    import vision
    g = torch.Generator().manual_seed(0)
    ids = torch.tensor([1, 151655, 151655, 151655, 2, 151656, 151656, 151656, 151656, 3])
    mask = torch.zeros(10, dtype=torch.bool)
    mask[1:4] = True                                    # images filled
    vid_pos = torch.tensor([5, 6, 7])                   # three of four video slots filled
    mask[vid_pos] = True
    img = [torch.randn(3, 4, generator=g), torch.randn(2, 4, generator=g)]  # level 1 short
    vid = [torch.randn(3, 4, generator=g), torch.randn(5, 4, generator=g),
           torch.randn(3, 4, generator=g)]              # one more level than the images
    got = vision._combine_levels(img, vid, ids, mask, vid_pos, torch.float32, "cpu")
    want = _reference_combine(img, vid, ids, mask, vid_pos, torch.float32)
    assert len(got) == len(want) == 3
    for a, b in zip(got, want):
        assert torch.equal(a, b)


def test_vision_entry_points_reject_bad_arguments_on_the_host():
    lib = _lib.load()
    one = ctypes.c_void_p(16)
    # linears: K must keep 16-byte rows
    rc = lib.q3_gemm_bias(one, one, one, one, 64, 128, 100, _lib.Q3_EPI_BIAS, None, None)
    assert rc == _lib.Q3_ERR_INVALID and b"multiple of 8" in lib.q3_last_error()
    rc = lib.q3_gemm_bias(one, one, one, one, 64, 128, 96, _lib.Q3_EPI_NONE, None, None)
    assert rc == _lib.Q3_ERR_INVALID and b"not a bias epilogue" in lib.q3_last_error()
    rc = lib.q3_gemm_bias(one, one, one, one, 64, 128, 96, _lib.Q3_EPI_BIAS_RESIDUAL, None, None)
    assert rc == _lib.Q3_ERR_INVALID and b"aux" in lib.q3_last_error()
    # image table checked against n_tok before any launch
    imgs = (ctypes.c_int32 * 4)(1, 8, 12, 0)
    rc = lib.q3_vision_pos_embed(one, 48, 1152, one, imgs, 1, 2, 95, one, None)
    assert rc == _lib.Q3_ERR_INVALID and b"96 tokens" in lib.q3_last_error()
    bad = (ctypes.c_int32 * 4)(1, 7, 12, 0)
    rc = lib.q3_vision_rope(one, 16, 72, one, one, bad, 1, 2, 84, None)
    assert rc == _lib.Q3_ERR_INVALID and b"merge" in lib.q3_last_error()
    rc = lib.q3_vision_rope(one, 16, 64, one, one, imgs, 1, 2, 96, None)
    assert rc == _lib.Q3_ERR_INVALID and b"head_dim" in lib.q3_last_error()
    # attention blocks must be 128-row blocks inside the tokens
    blocks = (ctypes.c_int32 * 3)(0, 96, 64)
    rc = lib.q3_vision_attention(one, one, 16, 72, one, blocks, 1, 96, None)
    assert rc == _lib.Q3_ERR_INVALID and b"128-row block" in lib.q3_last_error()
    blocks = (ctypes.c_int32 * 3)(0, 200, 0)
    rc = lib.q3_vision_attention(one, one, 16, 72, one, blocks, 1, 96, None)
    assert rc == _lib.Q3_ERR_INVALID
    rc = lib.q3_layernorm(one, one, one, one, 4, 100, 1e-6, None)
    assert rc == _lib.Q3_ERR_INVALID


def test_shard_images_balances_patches_and_covers_every_image():
    from q3vl.vision_tower import shard_images
    grid = [[1, 28, 28]] * 16
    shares = [shard_images(grid, 8, r) for r in range(8)]
    assert [(i0, i1) for i0, i1, *_ in shares] == [(2 * r, 2 * r + 2) for r in range(8)]
    uneven = [[1, 40, 40], [1, 8, 8], [2, 16, 16], [1, 8, 12], [1, 32, 32]]
    for world in (2, 3, 7):
        shares = [shard_images(uneven, world, r) for r in range(world)]
        assert shares[0][0] == 0 and shares[-1][1] == len(uneven)
        for a, b in zip(shares, shares[1:]):
            assert a[1] == b[0] and a[3] == b[2]
        merged = shares[0][4]
        assert merged[-1] == sum(t * h * w for t, h, w in uneven) // 4


def _sharded_worker(rank, world, port, q):
    import os
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen3-vl_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from q3vl.vision_tower import VisionTower

    class StandIn(VisionTower):
        """forward() replaced by a function of (image, merged token): the
        sharding and the gather are what is under test."""

        def forward(self, pixel_values, grid_thw):
            rows, off = [], 0
            for t, h, w in (grid_thw.tolist() if hasattr(grid_thw, "tolist") else grid_thw):
                img = int(pixel_values[off, 0])           # image index stored in its patches
                n = t * h * w // 4
                rows.append(torch.stack([torch.full((n,), float(img)),
                                         torch.arange(n, dtype=torch.float)], dim=1))
                off += t * h * w
            pooler = (torch.cat(rows) if rows else torch.empty(0, 2)).to(torch.bfloat16)
            return pooler, [pooler * 2, pooler * 3], torch.empty(0, 2, dtype=torch.bfloat16)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tower = StandIn.__new__(StandIn)
        tower.merge, tower.deepstack, tower.hidden = 2, (0, 1), 2
        tower.device = torch.device("cpu")
        tower.merger = {"linear_fc2.weight": torch.zeros(2, 2)}
        results = []
        for grid in ([[1, 8, 8], [2, 4, 4], [1, 16, 8], [1, 4, 12]], [[1, 8, 8]]):
            n = sum(t * h * w for t, h, w in grid)
            pix = torch.zeros(n, 3)
            off = 0
            for i, (t, h, w) in enumerate(grid):
                pix[off:off + t * h * w, 0] = i          # image index in every patch
                off += t * h * w
            full = StandIn.forward(tower, pix, grid)
            got = tower.forward_sharded(pix, torch.tensor(grid))
            results.append(torch.equal(got[0], full[0]) and
                           all(torch.equal(a, b) for a, b in zip(got[1], full[1])))
        if rank == 0:
            q.put(results)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put(repr(e))
        raise
    finally:
        dist.destroy_process_group()


def test_data_parallel_tower_gathers_every_image_in_order():
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [True, True]
