"""The one-call entry points of the C ABI (q3_gate_up_swiglu, q3_lm_head_argmax,
q3_init_comm) against the kernels they are made of: identical bits to
q3_gemm / q3_gemm_norm with the SwiGLU epilogue, to q3_gemm_norm followed by
q3_argmax / q3_argmax_key, and the communicator checks on one GPU."""
import ctypes

import pytest
import torch

from q3vl import _lib, ops
from tests.helpers import compare

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF16 = torch.bfloat16


def rnd(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(BF16).to(DEV)


@pytest.mark.parametrize("M", [1, 8, 16, 300])
def test_gate_up_swiglu_is_the_swiglu_projection(M):
    K, inter = 4096, 1536                       # one TP8 rank of the 8B MLP
    x, w = rnd(M, K, seed=1), rnd(2 * inter, K, seed=2, scale=0.02)
    got = ops.gate_up_swiglu(x, w)
    want = ops.gemm(x, w, "swiglu")
    assert torch.equal(got, want)
    if M <= 16:
        nw = rnd(K, seed=3, scale=0.1) + 1
        got = ops.gate_up_swiglu(x, w, norm_w=nw, eps=1e-6)
        want = ops.gemm_decode(x, w, "swiglu", norm_w=nw, eps=1e-6)
        assert torch.equal(got, want)
        # and within bf16 tolerance of the unfused fp32 formula
        h = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
        h = h.to(BF16).float() * nw.float()
        gu = h.to(BF16).float() @ w.float().t()
        gu = gu.view(M, inter // 8, 2, 8)
        ref = torch.nn.functional.silu(gu[:, :, 0]) * gu[:, :, 1]
        compare("gate_up_swiglu", got.float().cpu(), ref.reshape(M, inter).cpu(), max_abs=5e-2,
                min_cos=0.999, rel_scale=True)


@pytest.mark.parametrize("rows", [1, 8])
def test_lm_head_argmax_is_norm_projection_argmax(rows):
    K, V = 4096, 18992                          # one TP8 rank's vocabulary slice
    h, w = rnd(rows, K, seed=4), rnd(V, K, seed=5, scale=0.02)
    nw = rnd(K, seed=6, scale=0.1) + 1
    logits = torch.empty(rows, V, dtype=BF16, device=DEV)
    idx = ops.lm_head_argmax(h, w, norm_w=nw, eps=1e-6, logits=logits)
    want_logits = ops.gemm_decode(h, w, norm_w=nw, eps=1e-6)
    assert torch.equal(logits, want_logits)
    assert torch.equal(idx, ops.argmax(want_logits))
    assert torch.equal(idx.cpu(), want_logits.float().cpu().argmax(-1))
    keys = ops.lm_head_argmax(h, w, norm_w=nw, eps=1e-6, col_offset=3 * V, keys=True)
    assert torch.equal(keys, ops.argmax_key(want_logits, 3 * V))
    assert torch.equal(ops.argmax_key_index(keys), idx + 3 * V)
    # without the fused norm: the rows are used as given (any row count)
    hn = rnd(40, K, seed=7)
    idx2 = ops.lm_head_argmax(hn, w)
    assert torch.equal(idx2, ops.argmax(ops.gemm(hn, w)))
    assert ops.device_error(clear=True) == 0


def test_init_comm_checks_rank_and_world():
    lib = _lib.load()
    torch.cuda.set_device(0)
    comm = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(lib.q3_comm_handle_bytes())
    assert lib.q3_comm_create(0, 1, 4096, ctypes.byref(comm), handle) == _lib.Q3_OK
    try:
        rc = lib.q3_init_comm(comm, 1, 2, handle)
        assert rc == _lib.Q3_ERR_INVALID and b"created for rank 0 of 1" in lib.q3_last_error()
        assert lib.q3_init_comm(comm, 0, 1, handle) == _lib.Q3_OK
        assert lib.q3_init_comm(comm, 0, 1, handle) == _lib.Q3_ERR_INVALID   # already open
    finally:
        lib.q3_comm_destroy(comm)


def test_l2_prefetch_changes_no_result():
    """q3_l2_prefetch writes nothing: eager and inside a graph, and the tiny
    decoder with o_proj and next-layer QKV weights prefetched before each
    decode attention generates the reference's golden tokens, with and
    without graphs."""
    import loader_fused
    from tests.golden import cases
    from tests.helpers import load_golden
    w = rnd(4096, 4096, seed=8)
    before = w.clone()
    ops.l2_prefetch(w)
    ops.l2_prefetch(w[:1])
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.l2_prefetch(w)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(w, before)
    name = "decoder_tiny_tp1"
    gold = load_golden(name)
    c = cases.DECODER_CASES[name]
    s = c["spec"]
    spec = loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                 inter=s.inter, vocab=s.vocab, layers=s.layers,
                                 rope_theta=s.rope_theta, eps=s.eps)
    wt = cases.decoder_weights(name)
    dec = loader_fused.build_decoder(wt["layers"], wt["embed"], wt["final_norm"], wt["lm_head"],
                                     spec, 0, 1, DEV, c["max_seq"])
    dec.l2_prefetch_oproj = dec.l2_prefetch_qkv = True
    ids = cases.decoder_prompt(name).to(DEV)
    for graphs in (False, True):
        dec.use_graphs = graphs
        toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
        assert toks == gold["tokens"].tolist(), graphs
    assert ops.device_error(clear=True) == 0
