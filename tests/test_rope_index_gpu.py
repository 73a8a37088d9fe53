"""Multimodal 3-axis position ids on the device (q3_rope_index) vs the
fixtures of transformers' Qwen3VLModel.get_rope_index and the CPU oracle.
Integer work: every comparison is bit-exact."""
import numpy as np
import pytest
import torch

from oracle import ref as oref
from q3vl import ops
from tests.golden import cases
from tests.helpers import as_tensor, load_golden

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def run(lay, merge):
    ty = torch.from_numpy(np.ascontiguousarray(lay["types"])).to(DEV)
    mask = None if lay["mask"] is None else torch.from_numpy(lay["mask"]).to(DEV)
    img = torch.from_numpy(lay["image_thw"]).to(DEV)
    vid = torch.from_numpy(lay["video_thw"]).to(DEV)
    pos, delta = ops.rope_index(ty, img, vid, mask, spatial_merge_size=merge)
    return pos.cpu(), delta.cpu().view(-1)


@pytest.mark.parametrize("idx", range(len(cases.rope_index_fixture_cases())))
def test_rope_index_matches_get_rope_index_fixture(idx):
    name, lay, merge = cases.rope_index_fixture_cases()[idx]
    g = load_golden("rope_index")
    pos, delta = run(lay, merge)
    assert torch.equal(pos, as_tensor(g[name + "_pos"])), name
    assert torch.equal(delta, as_tensor(g[name + "_delta"])), name


@pytest.mark.parametrize("seed,B,runs,merge", [(21, 1, 80, 2), (22, 4, 40, 2), (23, 3, 60, 1),
                                               (24, 9, 6, 2)])
def test_rope_index_multi_chunk_layouts_match_oracle(seed, B, runs, merge):
    """Sequences of several 4096-token chunks: the scan carries cross chunks
    inside runs, including vision runs."""
    lay = cases.rope_index_layout(seed, B, runs, merge=merge, max_side=12)
    pos, delta = run(lay, merge)
    want_pos, want_delta = oref.rope_index(lay["types"], lay["mask"], lay["image_thw"],
                                           lay["video_thw"], merge)
    assert torch.equal(pos, want_pos)
    assert torch.equal(delta, want_delta)


def test_rope_index_rejects_what_the_reference_rejects():
    lay = dict(cases.rope_index_fixture_cases()[1][1])
    bad = [
        ({"image_thw": lay["image_thw"][:1]}, "more vision runs"),
        ({"image_thw": np.array([[1, 8, 12], [1, 6, 6]])}, "differs from its grid"),   # short
        ({"image_thw": np.array([[1, 8, 12], [1, 6, 2]])}, "differs from its grid"),   # long
        ({"mask": np.zeros_like(lay["types"])}, "no kept token"),
        ({"types": np.where(lay["types"] == 1, 1, 5).astype(np.int32)}, "outside"),
    ]
    for change, msg in bad:
        case = dict(lay, **change)
        with pytest.raises(ValueError, match=msg):
            run(case, 2)
    # the device stays usable after a rejected call
    pos, _ = run(lay, 2)
    assert torch.equal(pos, as_tensor(load_golden("rope_index")["two_images_pos"]))


def test_model_get_rope_index_feeds_mrope_tables():
    """Qwen3VLDecoderFused.get_rope_index (HF signature) -> the M-RoPE rows of
    prefill: the tables built from device-made positions equal those built
    from the fixture positions."""
    from model_fused import Qwen3VLDecoderFused, RotaryEmbedding
    name, lay, merge = cases.rope_index_fixture_cases()[2]
    m = Qwen3VLDecoderFused.__new__(Qwen3VLDecoderFused)
    m.device = torch.device(DEV)
    m.rotary = RotaryEmbedding(128, max_seq_len=4096, base=5e6)
    ids = torch.zeros(lay["types"].shape, dtype=torch.int64)
    pos, delta = m.get_rope_index(ids, torch.from_numpy(lay["types"]),
                                  torch.from_numpy(lay["image_thw"]),
                                  torch.from_numpy(lay["video_thw"]),
                                  torch.from_numpy(lay["mask"]))
    g = load_golden("rope_index")
    assert delta.shape == (2, 1)
    cos, sin = m._mrope(pos)
    cos_w, sin_w = m._mrope(as_tensor(g[name + "_pos"]))
    assert torch.equal(cos, cos_w) and torch.equal(sin, sin_w)
