"""loader_fused.load_model on a local HF checkpoint (loader_fused.py:38-237):
a tiny Qwen3-VL saved by transformers 5.5.0 is loaded at TP1 and TP2, and
every decoder weight of the rank is compared with the HF model's own tensors
through the modules' [in, out] views: q/k/v fused and column-sharded, o and
down row-sharded, gate/up fused, lm_head sharded by vocabulary rows, norms and
embeddings as is.  The processor comes from the checkpoint's files in the
reference; no tokenizer is available here, so AutoProcessor is replaced by a
stand-in.  CPU only: the modules are built on the CPU and no kernel runs."""
import pytest
import torch

import loader_fused
from tests.golden import cases

BF16 = torch.bfloat16
TEXT = dict(hidden_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
            intermediate_size=1024, num_hidden_layers=2, vocab_size=1024, rms_norm_eps=1e-6,
            rope_parameters={"rope_type": "default", "rope_theta": 5e6,
                             "mrope_section": [24, 20, 20], "mrope_interleaved": True})


def tiny_checkpoint(path, text=None):
    """Writes a seeded tiny Qwen3VLForConditionalGeneration to `path`."""
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration
    text = dict(TEXT if text is None else text)
    vision = dict(cases.VISION_TINY, out_hidden_size=text["hidden_size"])
    cfg = Qwen3VLConfig(text_config=text, vision_config=vision)
    torch.manual_seed(0)
    model = Qwen3VLForConditionalGeneration(cfg)
    with torch.no_grad():     # norms away from 1 so a swapped norm shows
        for n, p in model.named_parameters():
            if n.endswith("norm.weight"):
                p.uniform_(0.5, 1.5)
    model.save_pretrained(str(path))
    return path


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    return tiny_checkpoint(tmp_path_factory.mktemp("qwen3vl_tiny"))


@pytest.fixture
def no_processor(monkeypatch):
    import transformers
    monkeypatch.setattr(transformers.AutoProcessor, "from_pretrained",
                        classmethod(lambda cls, path, **kw: ("processor", str(path))))


@pytest.mark.parametrize("world,rank", [(1, 0), (2, 1)])
def test_load_model_shards_the_checkpoint_weights(checkpoint, no_processor, world, rank):
    dec, vision, processor, hf = loader_fused.load_model(str(checkpoint), rank, world, "cpu")
    assert processor == ("processor", str(checkpoint))
    assert vision is hf.model.visual
    lang = hf.model.language_model
    assert dec.num_layers == 2 and dec.tp_size == world
    hq, hkv, D = 4 // world, 2 // world, 128

    def col(w, n):  # rows of this rank's column shard
        return w[rank * n:(rank + 1) * n]

    def row(w, n):  # columns of this rank's row shard
        return w[:, rank * n:(rank + 1) * n]

    for i, layer in enumerate(dec.layers):
        a, m = lang.layers[i].self_attn, lang.layers[i].mlp
        ab, mb = layer.attn_block, layer.mlp_block
        qkv = torch.cat([col(a.q_proj.weight, hq * D), col(a.k_proj.weight, hkv * D),
                         col(a.v_proj.weight, hkv * D)]).t()
        assert torch.equal(ab.qkv_weight, qkv)
        assert torch.equal(ab.o_proj_weight, row(a.o_proj.weight, hq * D).t())
        assert torch.equal(layer.o_proj.weight, row(a.o_proj.weight, hq * D).t())
        assert torch.equal(ab.q_norm_weight, a.q_norm.weight)
        assert torch.equal(ab.k_norm_weight, a.k_norm.weight)
        assert torch.equal(ab.input_norm_weight, lang.layers[i].input_layernorm.weight)
        inter = 1024 // world
        gu = torch.cat([col(m.gate_proj.weight, inter), col(m.up_proj.weight, inter)]).t()
        assert torch.equal(mb.gate_up_weight, gu)
        assert torch.equal(mb.down_weight, row(m.down_proj.weight, inter).t())
        assert torch.equal(mb.post_norm_weight, lang.layers[i].post_attention_layernorm.weight)
        assert ab.num_q_heads == hq and ab.num_kv_heads == hkv and ab.head_dim == D
    V = 1024 // world
    assert torch.equal(dec.lm_head.weight, col(hf.lm_head.weight, V).t())
    assert torch.equal(dec.final_norm.weight, lang.norm.weight)
    table = dec.embed_tokens.weight if hasattr(dec.embed_tokens, "weight") else dec.embed_tokens
    assert torch.equal(table, lang.embed_tokens.weight)
    assert dec.rotary.inv_freq.shape == (64,)
    assert torch.allclose(dec.rotary.inv_freq,
                          1.0 / (5e6 ** (torch.arange(0, 128, 2, dtype=torch.float) / 128)))


def test_head_dim_comes_from_the_config(tmp_path, no_processor):
    """A config whose head_dim differs from hidden // heads (hidden 384 with 4
    heads of 128) loads with head_dim 128, as the checkpoint's shapes need."""
    text = dict(TEXT, hidden_size=384)
    path = tiny_checkpoint(tmp_path / "odd", text)
    dec, _, _, hf = loader_fused.load_model(str(path), 0, 1, "cpu")
    ab = dec.layers[0].attn_block
    assert ab.head_dim == 128 and ab.num_q_heads == 4
    assert ab.qkv_weight.shape == (384, (4 + 2 * 2) * 128)


def test_missing_checkpoint_raises_instead_of_serving_random_weights(tmp_path):
    """A mistyped model path must fail, not quietly build a random-init model;
    random weights come only from an explicit 'random' / 'random:<seed>'."""
    with pytest.raises(FileNotFoundError, match="does not exist"):
        loader_fused.load_model(str(tmp_path / "no_such_checkpoint"), 0, 1, "cpu")
    with pytest.raises(FileNotFoundError):
        loader_fused.load_model(None, 0, 1, "cpu")
