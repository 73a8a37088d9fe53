"""Per-kernel timing on chosen shapes (CUDA events, warm-up, L2 flush between
iterations), printing achieved GB/s or TFLOP/s.  Also the small-case driver
for ncu captures of a single kernel.

    python qwen3-vl_b200/q3vl/microbench.py gemv   --M 8 --N 24576 --K 4096 --epi swiglu
    python qwen3-vl_b200/q3vl/microbench.py gemm   --M 8192 --N 6144 --K 4096
    python qwen3-vl_b200/q3vl/microbench.py decode --B 8 --Hq 32 --Hkv 8 --L 1152
    python qwen3-vl_b200/q3vl/microbench.py prefill --B 1 --Hq 32 --Hkv 8 --S 2048 [--tc]
    python qwen3-vl_b200/q3vl/microbench.py rmsnorm --rows 8192 --hidden 4096
    python qwen3-vl_b200/q3vl/microbench.py layer  --B 8 --L 1152 --bucket 2048
    python qwen3-vl_b200/q3vl/microbench.py step   --B 8 --L 1152 --bucket 2048 --layers 36
    python qwen3-vl_b200/q3vl/microbench.py rope_index --B 8 --S 16384 [--hf]
    python qwen3-vl_b200/q3vl/microbench.py vision --B 16 --side 448 [--depth 27]
    python qwen3-vl_b200/q3vl/microbench.py paged  --B 8 --L 1152 --page 256
    python qwen3-vl_b200/q3vl/microbench.py e2e_vision --B 16 --side 448

`step` times q3_decode_step (every layer of a decode step in one persistent
kernel) as CUDA-graph replays and reports the step's HBM rate (weights + KV).
`rope_index` times q3_rope_index (3-axis position ids of a multimodal prompt:
text runs of 16 tokens between 32x32-patch images, merge 2) and, with --hf,
transformers' Qwen3VLModel.get_rope_index on the host cores for the same
layout.
`vision` times the vision tower (random weights of the 8B model's tower:
1152 hidden, 16 heads, MLP 4304, merger to 4096) on B images of side x side
pixels (patch 16, merge 2) and reports TFLOP/s over its GEMM and attention
FLOPs.  `paged` times decode attention through a block table against the
contiguous cache on the same K/V.
`layer` times every kernel of one TP1 decode layer of the 8B shape, and the
whole layer, as CUDA-graph replays cycling over 4 layers' weights (1.5 GB, so
every launch streams its weights from HBM), with the decode graph's arguments
(length read on the device, grid planned for the bucket).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

import torch  # noqa: E402

from q3vl import ops  # noqa: E402


def _time(fn, iters, warmup, flush):
    for _ in range(warmup):
        fn()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(iters)]
    for a, b in evs:
        if flush is not None:
            flush.zero_()
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    ts = sorted(a.elapsed_time(b) for a, b in evs)
    return ts[len(ts) // 2]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemv", "gemm", "decode", "prefill", "rmsnorm", "gemm_ar",
                                       "gemm_allreduce", "layer", "step", "tpstep", "rope_index",
                                       "vision", "paged", "e2e_vision"])
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--tp", type=int, default=1,
                    help="layer: time one rank's shard at this tensor-parallel degree")
    ap.add_argument("--bucket", type=int, default=2048)
    ap.add_argument("--M", type=int, default=8)
    ap.add_argument("--N", type=int, default=24576)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--epi", default="none", choices=["none", "residual", "swiglu", "allreduce"],
                    help="allreduce (gemv): q3_gemm_ar on a single-rank communicator")
    ap.add_argument("--norm", action="store_true",
                    help="gemv: RMSNorm fused in, sums of squares from a prior projection")
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--Hq", type=int, default=32)
    ap.add_argument("--Hkv", type=int, default=8)
    ap.add_argument("--L", type=int, default=1152)
    ap.add_argument("--S", type=int, default=2048)
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f32"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-flush", action="store_true", help="keep L2 warm between iterations")
    ap.add_argument("--side", type=int, default=448, help="vision: image side in pixels")
    ap.add_argument("--depth", type=int, default=27, help="vision: transformer blocks")
    ap.add_argument("--page", type=int, default=256, help="paged: tokens per page")
    ap.add_argument("--tc", action="store_true", help="prefill: the tcgen05 kernel")
    ap.add_argument("--variant", type=int, default=0,
                    help="prefill --tc: 0 V transposed in shared memory, 1 V MN-major, O in TMEM")
    ap.add_argument("--hf", action="store_true",
                    help="rope_index: also time transformers' get_rope_index on the host")
    a = ap.parse_args(argv)
    if a.kernel == "rope_index":
        return _rope_index(a)
    if a.kernel == "vision":
        return _vision(a)
    if a.kernel == "paged":
        return _paged(a)
    if a.kernel == "e2e_vision":
        return _e2e_vision(a)
    if a.kernel == "gemm_ar":
        return _gemm_ar(a)
    if a.kernel == "tpstep":
        return _tpstep(a)
    if a.kernel == "gemm_allreduce":
        return _gemm_allreduce(a)
    if a.kernel == "layer":
        return _layer(a)
    if a.kernel == "step":
        return _step(a)
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    flush = None if a.no_flush else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    bf = torch.bfloat16
    res = {"kernel": a.kernel}
    if a.kernel in ("gemv", "gemm"):
        x = torch.randn(a.M, a.K, device=dev).to(bf)
        w = (torch.randn(a.N, a.K, device=dev) * 0.02).to(bf)
        r = torch.randn(a.M, a.N, device=dev).to(bf) if a.epi in ("residual", "allreduce") \
            else None
        out_n = a.N // 2 if a.epi == "swiglu" else a.N
        out = torch.empty(a.M, out_n, dtype=bf, device=dev)
        if a.norm:
            if a.M > 16 or a.K % 64:
                raise SystemExit("--norm: decode shapes (M <= 16, K % 64 == 0) only")
            nw = torch.ones(a.K, dtype=bf, device=dev)
            ss = torch.zeros(a.K // 64, 16, device=dev)
            ss[:, :a.M] = (x.float() ** 2).view(a.M, a.K // 64, 64).sum(-1).t()
            fn = lambda: ops.gemm_decode(x, w, a.epi, residual=r, norm_w=nw, ss_in=ss,  # noqa
                                         ss_tiles=a.K // 64, out=out)
        elif a.epi == "allreduce":
            # q3_gemm_ar on a single-rank communicator: the all-reduce
            # projection's kernel and epilogue with no peer to exchange with
            import ctypes

            from q3vl import _lib

            class _Solo:
                handle = ctypes.c_void_p()
            solo = _Solo()
            nb = int(_lib.load().q3_comm_handle_bytes())
            _lib.call("q3_comm_create", 0, 1, a.N, ctypes.byref(solo.handle),
                      (ctypes.c_char * nb)())
            ss_out = torch.empty(a.N // 64, 16, device=dev)
            fn = lambda: ops.gemm_ar(x, w, solo, residual=r, out=out, ss_out=ss_out)  # noqa
        else:
            fn = lambda: ops.gemm(x, w, a.epi, residual=r, out=out)  # noqa: E731
        ms = _time(fn, a.iters, a.warmup, flush)
        nbytes = (w.numel() + x.numel() + out.numel() + (r.numel() if r is not None else 0)) * 2
        flops = 2.0 * a.M * a.N * a.K
        res.update(M=a.M, N=a.N, K=a.K, epi=a.epi, norm=a.norm, ms=ms, gbs=nbytes / ms / 1e6,
                   tflops=flops / ms / 1e9)
    elif a.kernel == "decode":
        dt = torch.float32 if a.dtype == "f32" else bf
        q = torch.randn(a.B, a.Hq, 128, device=dev).to(dt)
        kc = torch.randn(a.B, a.Hkv, a.L, 128, device=dev).to(dt)
        vc = torch.randn_like(kc)
        out = torch.empty_like(q)
        ms = _time(lambda: ops.attn_decode(q, kc, vc, kv_len=a.L, out=out), a.iters, a.warmup,
                   flush)
        nbytes = 2 * kc.numel() * kc.element_size() + 2 * q.numel() * q.element_size()
        res.update(B=a.B, Hq=a.Hq, Hkv=a.Hkv, L=a.L, dtype=a.dtype, ms=ms,
                   gbs=nbytes / ms / 1e6)
    elif a.kernel == "prefill":
        q = torch.randn(a.B, a.Hq, a.S, 128, device=dev).to(bf)
        k = torch.randn(a.B, a.Hkv, a.S, 128, device=dev).to(bf)
        v = torch.randn_like(k)
        out = torch.empty_like(q)
        if a.tc:
            fn = lambda q_, k_, v_, out: ops.attn_prefill_tc(q_, k_, v_, out=out,  # noqa: E731
                                                             variant=a.variant)
        else:
            fn = ops.attn_prefill
        ms = _time(lambda: fn(q, k, v, out=out), a.iters, a.warmup, flush)
        flops = 4.0 * a.B * a.Hq * a.S * a.S * 128 / 2
        res.update(B=a.B, Hq=a.Hq, Hkv=a.Hkv, S=a.S, tc=a.tc, variant=a.variant if a.tc else None,
                   ms=ms, tflops=flops / ms / 1e9)
    else:
        x = torch.randn(a.rows, a.hidden, device=dev).to(bf)
        w = torch.ones(a.hidden, dtype=bf, device=dev)
        y = torch.empty_like(x)
        ms = _time(lambda: ops.rmsnorm(x, w, out=y), a.iters, a.warmup, flush)
        res.update(rows=a.rows, hidden=a.hidden, ms=ms, gbs=2 * x.numel() * 2 / ms / 1e6)
    print(json.dumps(res), flush=True)


def _graph_ms(fns, rounds=5):
    """Device time per call: `rounds` passes over `fns` captured in one graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(rounds):
            for f in fns:
                f()
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(5):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (5 * rounds * len(fns))


def _layer(a):
    import dataclasses

    import loader_fused
    dev = torch.device("cuda:0")
    # with --tp N: one rank's shard of each layer (4N layers cycled, so the
    # weights still exceed L2); the all-reduce projections run as q3_gemm_ar
    # on a single-rank communicator (the kernel and its epilogue, no peers)
    NL = 4 * a.tp
    spec = dataclasses.replace(loader_fused.QWEN3_VL_8B, layers=NL)
    dec = loader_fused.random_decoder(spec, 0, a.tp, dev, seed=0, max_seq=a.bucket)
    comm = None
    if a.tp > 1:
        import ctypes

        from q3vl import _lib

        class _Solo:
            handle = ctypes.c_void_p()
        comm = _Solo()
        nb = int(_lib.load().q3_comm_handle_bytes())
        _lib.call("q3_comm_create", 0, 1, spec.hidden, ctypes.byref(comm.handle),
                  (ctypes.c_char * nb)())
    B, L, H = a.B, a.L, spec.hidden
    kv = dec._kv_for(B, a.bucket)
    for k, v in kv:
        k.normal_()
        v.normal_()
    pos = torch.tensor([L - 1], dtype=torch.int32, device=dev)
    kv_len = torch.tensor([L], dtype=torch.int32, device=dev)
    bf = torch.bfloat16
    x = torch.randn(B, H, device=dev).to(bf)
    ss0, ss1 = dec._ss_buf(0), dec._ss_buf(1)
    ss1.view(-1, 16)[:H // 64, :B] = (x.float() ** 2).view(B, H // 64, 64).sum(-1).t()
    ss0.copy_(ss1)
    cos, sin, _ = dec.rotary.tables(dev)
    L0 = dec.layers[0]
    ab0, mlp0 = L0.attn_block, L0.mlp_block
    qkv = torch.empty(B, ab0.qkv_weight_km.shape[0], dtype=bf, device=dev)
    q = torch.empty(B, ab0.num_q_heads, 1, 128, dtype=bf, device=dev)
    attn = torch.empty(B, ab0.num_q_heads, 128, dtype=bf, device=dev)
    x2 = torch.empty_like(x)
    act = torch.empty(B, mlp0.gate_up_weight_il.shape[0] // 2, dtype=bf, device=dev)
    y = torch.empty_like(x)
    ws = ops.decode_workspace(B, ab0.num_q_heads, ab0.num_kv_heads, dev)

    def k_qkv(i):
        ab = dec.layers[i].attn_block
        return lambda: ops.gemm_decode(x, ab.qkv_weight_km, norm_w=ab.input_norm_weight,
                                       eps=ab.eps, ss_in=ss1, ss_tiles=H // 64, out=qkv)

    def k_rope(i):
        ab = dec.layers[i].attn_block
        kc, vc = kv[i]

        def f():
            qq, _, _ = ops.qkv_norm_rope(qkv, ab.q_norm_weight, ab.k_norm_weight, cos, sin, B=B,
                                         S=1, Hq=ab.num_q_heads, Hkv=ab.num_kv_heads,
                                         pos_dev=pos, k_cache=kc, v_cache=vc, eps=ab.eps)
            return qq
        return f

    def k_attn(i):
        kc, vc = kv[i]
        return lambda: ops.attn_decode(q.view(B, -1, 128), kc, vc, kv_len=a.bucket,
                                       kv_len_dev=kv_len, out=attn, workspace=ws)

    def k_o(i):
        if comm is not None:
            return lambda: ops.gemm_ar(attn.view(B, -1), dec.layers[i].o_proj.weight_km, comm,
                                       residual=x, ss_out=ss0, out=x2)
        return lambda: ops.gemm_decode(attn.view(B, -1), dec.layers[i].o_proj.weight_km,
                                       "residual", residual=x, ss_out=ss0, out=x2)

    def k_gu(i):
        m = dec.layers[i].mlp_block
        return lambda: ops.gemm_decode(x2, m.gate_up_weight_il, "swiglu", norm_w=m.post_norm_weight,
                                       eps=m.eps, ss_in=ss0, ss_tiles=H // 64, out=act)

    def k_down(i):
        if comm is not None:
            return lambda: ops.gemm_ar(act, dec.layers[i].mlp_block.down_weight_km, comm,
                                       residual=x2, ss_out=ss1, out=y)
        return lambda: ops.gemm_decode(act, dec.layers[i].mlp_block.down_weight_km, "residual",
                                       residual=x2, ss_out=ss1, out=y)

    def k_layer(i):
        if comm is not None:
            # the rank's six launches back to back (no exchange with peers)
            fs = [k(i) for k in (k_qkv, k_rope, k_attn, k_o, k_gu, k_down)]
            return lambda: [f() for f in fs]
        return lambda: dec._layer(x, None, i, kv, 0, 1, B, pos_dev=pos, kv_len_dev=kv_len,
                                  kv_bound=a.bucket, ss_valid=True)

    W = dict(qkv=ab0.qkv_weight_km.numel() * 2, o_proj=L0.o_proj.weight_km.numel() * 2,
             gate_up=mlp0.gate_up_weight_il.numel() * 2,
             down=mlp0.down_weight_km.numel() * 2,
             attention=2 * B * ab0.num_kv_heads * L * 128 * 2)
    res = {"kernel": "layer", "tp": a.tp, "B": B, "L": L, "bucket": a.bucket, "us": {},
           "gbs": {}}
    tot = 0.0
    for name, mk in (("qkv", k_qkv), ("qkv_norm_rope", k_rope), ("attention", k_attn),
                     ("o_proj", k_o), ("gate_up", k_gu), ("down", k_down)):
        ms = _graph_ms([mk(i) for i in range(NL)])
        tot += ms
        res["us"][name] = round(ms * 1e3, 2)
        if name in W:
            res["gbs"][name] = round(W[name] / ms / 1e6, 1)
    res["us"]["sum_of_kernels"] = round(tot * 1e3, 2)
    ms = _graph_ms([k_layer(i) for i in range(NL)])
    res["us"]["layer"] = round(ms * 1e3, 2)
    res["layer_hbm_gbs"] = round(sum(W.values()) / ms / 1e6, 1)
    print(json.dumps(res), flush=True)


def _step(a):
    import dataclasses

    import loader_fused
    dev = torch.device("cuda:0")
    spec = dataclasses.replace(loader_fused.QWEN3_VL_8B, layers=a.layers, vocab=4096)
    dec = loader_fused.random_decoder(spec, 0, 1, dev, seed=0, max_seq=a.bucket)
    B, L, H = a.B, a.L, spec.hidden
    kv = dec._kv_for(B, a.bucket)
    for k, v in kv:
        k.normal_()
        v.normal_()
    plan = dec._step_plan(B, kv)
    x0 = torch.randn(B, H, device=dev).to(torch.bfloat16)
    x = x0.clone()
    ss = torch.zeros(H // 128, 16, device=dev)
    kv_len = torch.tensor([L], dtype=torch.int32, device=dev)

    def f():
        x.copy_(x0)
        plan.run(x, ss, kv_len)
    ms = _graph_ms([f], rounds=4)
    torch.cuda.synchronize()
    err = ops.device_error(clear=True)
    L0 = dec.layers[0]
    wbytes = sum(t.numel() * 2 for t in (L0.attn_block.qkv_weight_km, L0.o_proj.weight_km,
                                         L0.mlp_block.gate_up_weight_il,
                                         L0.mlp_block.down_weight_km))
    kvbytes = 2 * B * L0.attn_block.num_kv_heads * L * 128 * 2
    tot = a.layers * (wbytes + kvbytes)
    print(json.dumps({"kernel": "step", "B": B, "L": L, "layers": a.layers,
                      "ms": round(ms, 4), "us_per_layer": round(ms * 1e3 / a.layers, 2),
                      "gbs": round(tot / ms / 1e6, 1), "bytes": tot, "device_error": err}),
          flush=True)
    plan.close()


def _tpstep(a):
    """The tensor-parallel decode step kernel (q3_decode_tp) on one GPU at the
    shard shapes of one rank at TP = --tp (8B model, --layers layers), on a
    single-rank communicator (no peer exchange), as CUDA-graph replays;
    against the same rank's per-kernel layer (the layer microbench's kernels)
    it shows what one launch per step saves."""
    import dataclasses

    import loader_fused
    from q3vl.comm import SoloComm
    dev = torch.device("cuda:0")
    base = loader_fused.QWEN3_VL_8B
    spec = dataclasses.replace(base, layers=a.layers, vocab=4096, q_heads=base.q_heads // a.tp,
                               kv_heads=base.kv_heads // a.tp, inter=base.inter // a.tp)
    dec = loader_fused.random_decoder(spec, 0, 1, dev, seed=0, max_seq=a.bucket)
    B, L, H = a.B, a.L, spec.hidden
    kv = dec._kv_for(B, a.bucket)
    for k, v in kv:
        k.normal_()
        v.normal_()
    comm = SoloComm(max_cols=H, device=dev)
    layers = []
    for Ly, (kc, vc) in zip(dec.layers, kv):
        ab, mlp = Ly.attn_block, Ly.mlp_block
        layers.append(dict(w_qkv=ab.qkv_weight_km, w_o=Ly.o_proj.weight_km,
                           w_gate_up=mlp.gate_up_weight_il, w_down=mlp.down_weight_km,
                           input_norm=ab.input_norm_weight, post_norm=mlp.post_norm_weight,
                           q_norm=ab.q_norm_weight, k_norm=ab.k_norm_weight, k_cache=kc,
                           v_cache=vc))
    cos, sin, _ = dec.rotary.tables(dev)
    plan = ops.DecodeTPPlan(layers, batch=B, hidden=H, q_heads=spec.q_heads,
                            kv_heads=spec.kv_heads, inter=spec.inter, max_seq=a.bucket,
                            eps=spec.eps, cos=cos, sin=sin, comm=comm)
    x0 = (torch.randn(B, H, device=dev) * 0.02).to(torch.bfloat16)
    x = x0.clone()
    kv_len = torch.tensor([L], dtype=torch.int32, device=dev)

    def f():
        x.copy_(x0)
        plan.run(x, kv_len)
    ms = _graph_ms([f], rounds=4)
    torch.cuda.synchronize()
    err = ops.device_error(clear=True)
    L0 = dec.layers[0]
    wbytes = sum(t.numel() * 2 for t in (L0.attn_block.qkv_weight_km, L0.o_proj.weight_km,
                                         L0.mlp_block.gate_up_weight_il,
                                         L0.mlp_block.down_weight_km))
    kvbytes = 2 * B * L0.attn_block.num_kv_heads * L * 128 * 2
    tot = a.layers * (wbytes + kvbytes)
    print(json.dumps({"kernel": "tpstep", "tp": a.tp, "B": B, "L": L, "layers": a.layers,
                      "ms": round(ms, 4), "us_per_layer": round(ms * 1e3 / a.layers, 2),
                      "gbs": round(tot / ms / 1e6, 1), "bytes": tot, "device_error": err}),
          flush=True)
    plan.close()
    comm.close()


def _gemm_ar(a):
    """Row-parallel decode projection at TP=WORLD_SIZE (run under torchrun):
    GEMV alone, GEMV + NCCL all-reduce, and the fused in-kernel all-reduce.
    Back-to-back launches on one stream (no flush), median of 5 runs of
    `iters` launches, max over ranks."""
    import torch.distributed as dist

    from q3vl.comm import PeerComm
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    comm = PeerComm(max_cols=a.N, device=dev)
    bf = torch.bfloat16
    x = torch.randn(a.M, a.K, device=dev).to(bf)
    w = (torch.randn(a.N, a.K, device=dev) * 0.02).to(bf)
    r = torch.randn(a.M, a.N, device=dev).to(bf)
    out = torch.empty(a.M, a.N, dtype=bf, device=dev)

    def plain():
        ops.gemm(x, w, out=out)

    def nccl():
        ops.gemm(x, w, out=out)
        dist.all_reduce(out)

    def fused():
        ops.gemm_ar(x, w, comm, residual=r, out=out)

    res = {"kernel": "gemm_ar", "M": a.M, "N": a.N, "K": a.K, "world": world}
    for name, fn in (("gemv_us", plain), ("gemv_nccl_us", nccl), ("gemm_ar_us", fused)):
        for _ in range(a.warmup):
            fn()
        ts = []
        for _ in range(5):
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / a.iters)
        t = torch.tensor([sorted(ts)[2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(float(t), 2)
    if rank == 0:
        print(json.dumps(res), flush=True)
    comm.close()
    dist.destroy_process_group()


def _gemm_allreduce(a):
    """Row-parallel prefill projection at TP=WORLD_SIZE (run under torchrun):
    the tcgen05 GEMM alone, GEMM + NCCL all-reduce + residual add, and the
    two-shot exchange started from the GEMM epilogue (q3_gemm_allreduce).
    Median of 5 runs of `iters` calls, max over ranks.  The roofline of the
    fused call is the slower of its FLOPs at the tensor peak and the bytes
    each rank must send over NVLink, 2 * (world - 1) / world * M * N * 2 B
    (reduce-scatter plus all-gather), at the link's bandwidth."""
    import torch.distributed as dist

    from q3vl.comm import PrefillComm
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    comm = PrefillComm(max_rows=a.M, max_cols=a.N, device=dev)
    bf = torch.bfloat16
    x = torch.randn(a.M, a.K, device=dev).to(bf)
    w = (torch.randn(a.N, a.K, device=dev) * 0.02).to(bf)
    r = torch.randn(a.M, a.N, device=dev).to(bf)
    part = torch.empty(a.M, a.N, dtype=bf, device=dev)
    out = torch.empty(a.M, a.N, dtype=bf, device=dev)

    def plain():
        ops.gemm(x, w, out=part)

    def nccl():
        ops.gemm(x, w, out=part)
        dist.all_reduce(part)
        ops.add(part, r, out=out)

    def fused():
        ops.gemm_allreduce(x, w, comm, residual=r, out=out)

    res = {"kernel": "gemm_allreduce", "M": a.M, "N": a.N, "K": a.K, "world": world,
           "nvlink_bytes_per_rank": 2 * (world - 1) * a.M * a.N * 2 // world}
    for name, fn in (("gemm_us", plain), ("gemm_nccl_us", nccl), ("gemm_allreduce_us", fused)):
        for _ in range(a.warmup):
            fn()
        ts = []
        for _ in range(5):
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / a.iters)
        t = torch.tensor([sorted(ts)[2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(float(t), 2)
    res["device_error"] = ops.device_error(clear=True)
    if rank == 0:
        print(json.dumps(res), flush=True)
    comm.close()
    dist.destroy_process_group()


def _rope_layout(B, S, side=32, text=16, merge=2):
    """Token types [B, S] int32: text runs of `text` tokens between
    (1, side, side) images, the tail text; image grids in batch order."""
    n_img = (side // merge) ** 2
    types = torch.zeros(B, S, dtype=torch.int32)
    grids = []
    for b in range(B):
        s = text
        while s + n_img + text <= S:
            types[b, s:s + n_img] = 1
            grids.append((1, side, side))
            s += n_img + text
    return types, torch.tensor(grids, dtype=torch.int64).reshape(-1, 3)


def _rope_index(a):
    import ctypes
    from q3vl import _lib
    dev = torch.device("cuda:0")
    types_h, grids_h = _rope_layout(a.B, a.S)
    types, grids = types_h.to(dev), grids_h.to(dev)
    B, S = types.shape
    pos = torch.empty(3, B, S, dtype=torch.int64, device=dev)
    delta = torch.empty(B, dtype=torch.int64, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    nbytes = _lib.raw("q3_rope_index_workspace_bytes")(B)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    fn = lambda: _lib.call("q3_rope_index", p(types), None, B, S, p(grids), grids.shape[0],  # noqa
                           None, 0, 2, p(pos), p(delta), p(status), p(ws), nbytes, st)
    flush = None if a.no_flush else torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ms = _time(fn, a.iters, a.warmup, flush)
    if int(status.abs().sum()) != 0:
        raise SystemExit("rope_index: nonzero status on a valid layout")
    nbytes_io = B * S * (4 + 24) + B * 8
    res = {"kernel": "rope_index", "B": B, "S": S, "images": int(grids.shape[0]), "ms": ms,
           "mtok_s": B * S / ms / 1e3, "gbs": nbytes_io / ms / 1e6}
    if a.hf:
        import time
        import types as pytypes
        import functools
        from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLModel
        host = pytypes.SimpleNamespace(config=pytypes.SimpleNamespace(
            vision_config=pytypes.SimpleNamespace(spatial_merge_size=2)))
        host.get_vision_position_ids = functools.partial(Qwen3VLModel.get_vision_position_ids,
                                                         host)
        ids = torch.zeros(B, S, dtype=torch.int64)
        t0 = time.perf_counter()
        hp, hd = Qwen3VLModel.get_rope_index(host, ids, types_h.long(), grids_h, None, None)
        hf_ms = (time.perf_counter() - t0) * 1e3
        same = torch.equal(hp, pos.cpu()) and torch.equal(hd.view(-1), delta.cpu())
        res.update(hf_ms=hf_ms, hf_threads=torch.get_num_threads(), hf_equal=same)
    print(json.dumps(res), flush=True)



def _random_tower(depth, dev):
    """The 8B model's vision tower shape with random weights (1152 hidden, 16
    heads, MLP 4304, merger to 4096, deepstack after blocks 8/16/24)."""
    from q3vl.vision_tower import VisionTower
    H, I, O, M = 1152, 4304, 4096, 1152 * 4
    c = dict(depth=depth, hidden_size=H, num_heads=16, intermediate_size=I, out_hidden_size=O,
             num_position_embeddings=2304, spatial_merge_size=2,
             deepstack_visual_indexes=[i for i in (8, 16, 24) if i < depth])
    bf = torch.bfloat16

    def mat(o, i):
        return (torch.randn(o, i, device=dev) * (i ** -0.5)).to(bf)

    def vec(n, base=0.0):
        return (base + torch.randn(n, device=dev) * 0.02).to(bf)

    w = {"patch_embed.proj.weight": mat(H, 1536).view(H, 3, 2, 16, 16),
         "patch_embed.proj.bias": vec(H), "pos_embed.weight": mat(2304, H)}
    for i in range(depth):
        b = f"blocks.{i}."
        w.update({b + "norm1.weight": vec(H, 1.0), b + "norm1.bias": vec(H),
                  b + "norm2.weight": vec(H, 1.0), b + "norm2.bias": vec(H),
                  b + "attn.qkv.weight": mat(3 * H, H), b + "attn.qkv.bias": vec(3 * H),
                  b + "attn.proj.weight": mat(H, H), b + "attn.proj.bias": vec(H),
                  b + "mlp.linear_fc1.weight": mat(I, H), b + "mlp.linear_fc1.bias": vec(I),
                  b + "mlp.linear_fc2.weight": mat(H, I), b + "mlp.linear_fc2.bias": vec(H)})
    for j, m in enumerate(["merger."] + [f"deepstack_merger_list.{k}."
                                         for k in range(len(c["deepstack_visual_indexes"]))]):
        n = H if j == 0 else M
        w.update({m + "norm.weight": vec(n, 1.0), m + "norm.bias": vec(n),
                  m + "linear_fc1.weight": mat(M, M), m + "linear_fc1.bias": vec(M),
                  m + "linear_fc2.weight": mat(O, M), m + "linear_fc2.bias": vec(O)})
    return VisionTower(w, c, dev), c


def _vision(a):
    """The vision tower on B images of side x side pixels (config 5 at B=16, 448)."""
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    depth = a.depth
    H, I, O, M = 1152, 4304, 4096, 1152 * 4
    bf = torch.bfloat16
    tower, c = _random_tower(depth, dev)
    g = a.side // 16
    grid = torch.tensor([[1, g, g]] * a.B)
    n = a.B * g * g
    x = torch.rand(n, 1536, device=dev).to(bf)
    ms = _time(lambda: tower(x, grid), a.iters, a.warmup, None)
    per_img = g * g
    blk = 2 * per_img * H * (3 * H + H + 2 * I) + 4 * per_img * per_img * H
    flops = a.B * (depth * blk + 2 * per_img * 1536 * H
                   + (1 + len(c["deepstack_visual_indexes"])) * 2 * (per_img // 4) * M * (M + O))
    print(json.dumps({"kernel": "vision", "images": a.B, "side": a.side, "patches": n,
                      "layers": depth, "ms": ms, "tflops": flops / ms / 1e9}), flush=True)


def _paged(a):
    """Decode attention through a block table vs the contiguous cache."""
    from q3vl.kv_pages import KVPagePool
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    bf = torch.bfloat16
    B, Hq, Hkv, L, page = a.B, a.Hq, a.Hkv, a.L, a.page
    width = (L + page - 1) // page
    pool = KVPagePool(B * width + 8, page, max_seqs=B, buckets=(), max_pages_per_seq=width,
                      layers=1, kv_heads=Hkv, device=dev)
    for b in reversed(range(B)):
        pool.reserve(b, L)
    table = pool.device_table(range(B))
    k = torch.randn(B, Hkv, L, 128, device=dev).to(bf)
    v = torch.randn_like(k)
    ops.kv_pages_write(k, v, pool.k[0], pool.v[0], table)
    q = torch.randn(B, Hq, 128, device=dev).to(bf)
    out = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    t_c = _time(lambda: ops.attn_decode(q, k, v, kv_len=L, out=out), a.iters, a.warmup, flush)
    t_p = _time(lambda: ops.attn_decode_paged(q, pool.k[0], pool.v[0], table, kv_len=L, out=out),
                a.iters, a.warmup, flush)
    nbytes = 2 * k.numel() * 2
    print(json.dumps({"kernel": "paged", "B": B, "L": L, "page": page, "contiguous_ms": t_c,
                      "paged_ms": t_p, "contiguous_gbs": nbytes / t_c / 1e6,
                      "paged_gbs": nbytes / t_p / 1e6}), flush=True)



def _e2e_vision(a):
    """Vision + text end to end at one GPU (the multimodal workload at B=16):
    B images of side x side pixels through the tower, the merged image tokens
    in front of a 256-token random text prompt, device position ids, then the
    36-layer decoder generating 128 tokens with M-RoPE rows and deepstack."""
    import loader_fused
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    B, g = a.B, a.side // 16
    n_img = (g // 2) ** 2
    text_len, new_tokens = 256, 128
    S = n_img + text_len
    tower, _ = _random_tower(a.depth, dev)
    dec = loader_fused.random_decoder(loader_fused.QWEN3_VL_8B, 0, 1, dev, seed=0, max_seq=2048)
    grid = torch.tensor([[1, g, g]] * B)
    x = torch.rand(B * g * g, 1536, device=dev).to(torch.bfloat16)
    ids = torch.randint(0, 151936, (B, S), device=dev)
    types = torch.zeros(B, S, dtype=torch.int32, device=dev)
    types[:, :n_img] = 1
    mask = types == 1

    def step():
        pooler, deep, _ = tower(x, grid)
        emb = dec._embed(ids).view(B, S, -1)
        emb[mask] = pooler
        pos, delta = dec.get_rope_index(ids, types, grid)
        return dec.generate_tokens(None, new_tokens, eos_token_id=None, inputs_embeds=emb,
                                   position_ids=pos, deepstack_embeds=deep, visual_mask=mask,
                                   rope_delta=int(delta[0, 0]))

    for _ in range(max(1, a.warmup)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_v0, t_v1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_v0.record()
    tower(x, grid)
    t_v1.record()
    e0.record()
    toks = step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    print(json.dumps({"kernel": "e2e_vision", "B": B, "side": a.side, "prompt": S,
                      "new_tokens": new_tokens, "vision_ms": t_v0.elapsed_time(t_v1),
                      "step_ms": ms, "gen_tok_s": B * toks.shape[1] / ms * 1e3}), flush=True)


if __name__ == "__main__":
    main()
