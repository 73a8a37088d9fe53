"""Tensor-parallel decoder on 2 GPUs (one process per GPU, NCCL): greedy
tokens and prefill logits vs the reference decoder run at TP2 (fixture
decoder_tiny_tp2).  Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen3-vl_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    import loader_fused
    from tests.golden import cases

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        name = "decoder_tiny_tp2"
        c = cases.DECODER_CASES[name]
        s = c["spec"]
        w = cases.decoder_weights(name)
        spec = loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                     inter=s.inter, vocab=s.vocab, layers=s.layers,
                                     rope_theta=s.rope_theta, eps=s.eps)
        dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"],
                                         w["lm_head"], spec, rank, world, dev, c["max_seq"])
        ids = cases.decoder_prompt(name).to(dev)
        logits = dec.forward(ids, 0, dec.init_kv_cache(1)).float().cpu()
        toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
        if rank == 0:
            q.put((logits.numpy(), toks))
        dec._graphs.clear()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_decoder_matches_reference():
    import torch.multiprocessing as mp

    from tests.golden import cases
    from tests.helpers import as_tensor, compare, load_golden
    g = load_golden("decoder_tiny_tp2")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    logits, toks = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    compare("tp2 logits", torch.from_numpy(logits), as_tensor(g["logits"]).float(),
            max_abs=5e-2, rel_scale=True, min_cos=0.999)
    assert toks == g["tokens"].tolist()
