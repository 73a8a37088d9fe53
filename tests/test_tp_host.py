"""Host-side tensor-parallel logic on CPU with 2 gloo ranks: the loader's
column/row sharding (including the interleaved gate/up layout) must make the
all-reduced sum of the ranks' partial projections equal the unsharded
projection, and every rank must see the same collective sequence."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "qwen3-vl_b200"), repo):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist

    import loader_fused
    from oracle import decoder as odec
    from q3vl import layout

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        spec = odec.Spec(hidden=256, q_heads=8, kv_heads=4, inter=512, vocab=64, layers=1,
                         max_seq=32)
        w = odec.make_weights(spec, seed=21, random_norms=True)
        lw = w["layers"][0]
        ts = loader_fused.TextSpec(hidden=256, q_heads=8, kv_heads=4, inter=512, vocab=64,
                                   layers=1)
        dec = loader_fused.build_decoder(w["layers"], w["embed"], w["final_norm"],
                                         w["lm_head"], ts, rank, world, "cpu", 32)
        L = dec.layers[0]
        g = torch.Generator().manual_seed(5)
        x = torch.randn(3, 256, generator=g)
        # column-parallel gate/up: each rank's interleaved rows hold its slice
        gate, up = layout.deinterleave_gate_up(L.mlp_block.gate_up_weight_il.float())
        n = 512 // world
        assert torch.equal(gate, lw["gate"][rank * n:(rank + 1) * n].float())
        assert torch.equal(up, lw["up"][rank * n:(rank + 1) * n].float())
        # row-parallel o_proj / down: partial sums all-reduce to the full product
        a = torch.randn(3, 8 * 128, generator=g)
        part = a[:, rank * 512:(rank + 1) * 512] @ L.o_proj.weight_km.float().t()
        dist.all_reduce(part)
        full = a @ lw["o"].float().t()
        assert torch.allclose(part, full, atol=1e-3, rtol=1e-3)
        h = torch.randn(3, 512, generator=g)
        part = h[:, rank * 256:(rank + 1) * 256] @ L.mlp_block.down_weight_km.float().t()
        dist.all_reduce(part)
        assert torch.allclose(part, h @ lw["down"].float().t(), atol=1e-3, rtol=1e-3)
        # qkv: [q | k | v] of this rank's heads
        qkv = x @ L.attn_block.qkv_weight_km.float().t()
        ref = torch.cat([x @ lw["q"][rank * 512:(rank + 1) * 512].float().t(),
                         x @ lw["k"][rank * 256:(rank + 1) * 256].float().t(),
                         x @ lw["v"][rank * 256:(rank + 1) * 256].float().t()], dim=1)
        assert torch.allclose(qkv, ref, atol=1e-3, rtol=1e-3)
        # lm_head vocab shards gather to the full logits
        lg = x @ dec.lm_head.weight_km.float().t()
        out = [torch.zeros_like(lg) for _ in range(world)]
        dist.all_gather(out, lg)
        assert torch.allclose(torch.cat(out, -1), x @ w["lm_head"].float().t(), atol=1e-3,
                              rtol=1e-3)
        q.put((rank, "ok"))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_sharding_all_reduce_reconstructs_full_projection():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
