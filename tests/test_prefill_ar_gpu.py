"""The prefill projection + two-shot all-reduce (q3_gemm_allreduce).

One GPU, world 1: the exchange degenerates to the GEMM's own push and the
reduce kernel, and must give the bits of the plain GEMM with the residual
epilogue, over consecutive calls (both buffer parities).  Two GPUs (one
process per GPU): every rank's output equals residual + sum of the ranks'
partials (max-abs <= 3e-2 of the output scale, cosine >= 0.9999, fp32
reference of bf16 partials), all ranks hold identical bits, including shapes
where one rank owns no rows; and the TP2 tiny decoder with the two-shot
prefill gives the reference's greedy tokens."""
import ctypes
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16


class _Comm:
    """A world-1 communicator made through the C ABI (no process group)."""

    def __init__(self, max_rows, max_cols):
        from q3vl import _lib
        self.lib = _lib.load()
        self.handle = ctypes.c_void_p()
        blob = ctypes.create_string_buffer(self.lib.q3_comm_handle_bytes())
        assert self.lib.q3_prefill_comm_create(0, 1, max_rows, max_cols,
                                               ctypes.byref(self.handle), blob) == _lib.Q3_OK
        assert self.lib.q3_prefill_comm_open(self.handle, blob) == _lib.Q3_OK

    def close(self):
        self.lib.q3_prefill_comm_destroy(self.handle)


@pytest.mark.parametrize("M,N,K", [(17, 4096, 1024), (300, 512, 4096), (1000, 4096, 512)])
def test_world1_is_the_residual_gemm(M, N, K):
    from q3vl import ops
    dev = "cuda:0"
    comm = _Comm(1024, 4096)
    try:
        for call in range(3):
            g = torch.Generator().manual_seed(10 * call + M)
            a = torch.randn(M, K, generator=g).to(BF16).to(dev)
            w = (torch.randn(N, K, generator=g) * 0.05).to(BF16).to(dev)
            r = torch.randn(M, N, generator=g).to(BF16).to(dev)
            got = ops.gemm_allreduce(a, w, comm, residual=r)
            assert torch.equal(got, ops.gemm(a, w, "residual", residual=r)), call
            got = ops.gemm_allreduce(a, w, comm)
            assert torch.equal(got, ops.gemm(a, w)), call
        assert ops.device_error(clear=True) == 0
    finally:
        comm.close()


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

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        import loader_fused
        from q3vl import ops
        from q3vl.comm import PrefillComm
        from tests.golden import cases
        from tests.helpers import compare, load_golden
        comm = PrefillComm(max_rows=1024, max_cols=4096, device=dev)
        results = []
        for M, N, K in ((40, 4096, 512), (300, 512, 1024), (1000, 4096, 512), (300, 512, 1024)):
            gen = [torch.Generator().manual_seed(1000 * M + r) for r in range(world)]
            As = [torch.randn(M, K, generator=g_).to(BF16) for g_ in gen]
            Ws = [(torch.randn(N, K, generator=g_) * 0.05).to(BF16) for g_ in gen]
            R = torch.randn(M, N, generator=torch.Generator().manual_seed(M)).to(BF16)
            out = ops.gemm_allreduce(As[rank].to(dev), Ws[rank].to(dev), comm,
                                     residual=R.to(dev))
            every = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(every, out)
            same = all(torch.equal(e, out) for e in every)
            parts = sum((a.float() @ w.float().t()).to(BF16).float() for a, w in zip(As, Ws))
            want = R.float() + parts.to(BF16).float()
            compare(f"two-shot M={M}", out.float().cpu(), want, max_abs=3e-2, rel_scale=True,
                    min_cos=0.9999)
            results.append(same)
        comm.close()
        # the tiny TP2 decoder with the two-shot prefill
        name = "decoder_tiny_tp2"
        c = cases.DECODER_CASES[name]
        s = c["spec"]
        w = cases.decoder_weights(name)
        spec = loader_fused.TextSpec(hidden=s.hidden, q_heads=s.q_heads, kv_heads=s.kv_heads,
                                     inter=s.inter, vocab=s.vocab, layers=s.layers,
                                     rope_theta=s.rope_theta, eps=s.eps)
        dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"],
                                         w["lm_head"], spec, rank, world, dev, c["max_seq"])
        dec.enable_prefill_allreduce(max_rows=1024)
        ids = cases.decoder_prompt(name).to(dev)
        toks = dec.generate(ids, max_new_tokens=c["new_tokens"], eos_token_id=-1)
        gold = load_golden(name)["tokens"].tolist()
        err = ops.device_error(clear=True)
        dec.close()
        q.put((rank, results, toks == gold, err))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), False, -1))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_two_shot_allreduce():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, results, tokens_ok, err in got:
        assert isinstance(results, list), (rank, results)
        assert all(results), (rank, results)
        assert tokens_ok, rank
        assert err == 0, (rank, hex(err))
