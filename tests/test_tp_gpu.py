"""Tensor-parallel decoder on 2 GPUs (one process per GPU, NCCL): greedy
tokens and prefill logits vs the reference decoder run at TP2 (fixture
decoder_tiny_tp2), through NCCL, through the in-kernel all-reduce of the
row-parallel projections, and through the step kernel (every layer of a decode
step in one launch per GPU).  Skipped when fewer than 2 GPUs are visible."""
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
        # same decode with o_proj/down all-reduced inside the kernel (peer memory)
        dec.enable_peer_allreduce()
        toks_peer = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
        # same decode through the step kernel: every layer of a step in one
        # launch per GPU, the all-reduce inside it (q3_decode_tp)
        dec.use_tp_kernel = True
        dec._graphs.clear()
        dec.enable_peer_allreduce()          # creates the step kernel's communicator
        toks_mk = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
        mk_ran = any(p_ is not None for p_ in dec._tp_plans.values())
        dec.use_tp_kernel = False
        dec._graphs.clear()
        # the fused kernel on its own: C = R + sum_r A_r W_r^T, identical on all ranks
        from q3vl import ops
        M, N, K = 8, 4096, 1024
        gen = [torch.Generator().manual_seed(100 + r) for r in range(world)]
        As = [torch.randn(M, K, generator=g_).to(torch.bfloat16) for g_ in gen]
        Ws = [(torch.randn(N, K, generator=g_) * 0.05).to(torch.bfloat16) for g_ in gen]
        R = torch.randn(M, N, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
        outs = []
        ss = torch.full((N // 64, 16), float("nan"), device=dev)
        for i in range(3):   # repeated calls exercise the flag/parity protocol
            outs.append(ops.gemm_ar(As[rank].to(dev), Ws[rank].to(dev), dec.comm,
                                    residual=R.to(dev), ss_out=ss if i == 2 else None).cpu())
        # per-64-column sums of squares of the stored output, for the next norm
        want_ss = (outs[-1].float() ** 2).view(M, N // 64, 64).sum(-1).t()
        ss_ok = bool(torch.allclose(ss[:, :M].cpu(), want_ss, rtol=1e-4) and
                     torch.all(ss[:, M:] == 0).item())
        want = R.float() + sum((As[r].float() @ Ws[r].float().t()) for r in range(world))
        gathered = [torch.zeros(M, N, dtype=torch.bfloat16, device=dev) for _ in range(world)]
        dist.all_gather(gathered, outs[-1].to(dev))
        same = all(torch.equal(gathered[0].cpu(), x.cpu()) for x in gathered)
        err = max((o.float() - want).abs().max().item() for o in outs)
        if rank == 0:
            q.put((logits.numpy(), toks, toks_peer, toks_mk, mk_ran, err, same, ss_ok))
        dist.barrier()
        dec.close()
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
    logits, toks, toks_peer, toks_mk, mk_ran, err, same, ss_ok = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    compare("tp2 logits", torch.from_numpy(logits), as_tensor(g["logits"]).float(),
            max_abs=5e-2, rel_scale=True, min_cos=0.999)
    want = g["tokens"].tolist()

    def first_diff(a):
        return next((i for i, (x, y) in enumerate(zip(a, want)) if x != y), None)

    assert toks == want, f"NCCL path: first mismatch at step {first_diff(toks)}"
    assert toks_peer == want, f"peer all-reduce: first mismatch at step {first_diff(toks_peer)}"
    assert mk_ran, "the step kernel did not run"
    assert toks_mk == want, f"step kernel: first mismatch at step {first_diff(toks_mk)}"
    assert same, "ranks disagree on the all-reduced projection"
    assert err < 0.25, f"gemm_ar max-abs {err} (bf16 output of magnitude ~10)"
    assert ss_ok, "gemm_ar sums of squares (ss_out) disagree with the stored output"
