"""Benchmark: Qwen3-VL-8B-shape text decoder, greedy generation at TP = N.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1 under: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N)

Workload (the full 36-layer decoder of the 8B shape, random-init bf16 weights
N(0, 0.02)): batch 8, prompts of 1024 uniformly random token ids, greedy
generation of 256 new tokens, KV bucket 2048.  One step = one generate():
prefill of 8x1024 tokens + 255 CUDA-graph decode steps.  Tensor parallelism
splits every layer over the N GPUs (strong scaling: total work is fixed).

value  = generated tokens per second over the whole step (8 x 256 / step time);
         prefill and decode rates are reported beside it.
e2e    = the same metric through the public API (decoder.generate_tokens) with
         the prompt copied from pinned host memory and the tokens read back
         every step.
The reference arm (--impl reference) times the CPU oracle -- a restatement of
the reference's own PyTorch decoder -- on the host cores, all 36 layers deep,
on a bounded sample of the same workload (one prompt's prefill and a few
decode steps of the whole batch) scaled by batch rows and decode steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "qwen3-vl_b200")
for _p in (PKG, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the gate/up
# decode projection (fused-norm variant, 8 tokens, TP1), from an ncu capture
# of `microbench.py gemv --M 8 --N 24576 --K 4096 --epi swiglu --norm`
# (201.44 MB read + 4.06 MB written)
GEMV_TRAFFIC_BYTES = 205502720

METRIC = "decode & prefill tok/s at TP1/2/4/8 (8B shape); attention HBM GB/s vs peak"
BATCH, PROMPT, NEW_TOKENS, BUCKET = 8, 1024, 256, 2048
WORKLOAD = (f"Qwen3-VL-8B-shape text decoder (36 layers, hidden 4096, 32/8 heads, inter "
            f"12288, vocab 151936), batch {BATCH}, prompt {PROMPT} random ids, "
            f"{NEW_TOKENS} greedy tokens, KV bucket {BUCKET}")


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    import loader_fused
    from q3vl import _lib, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=300), device_id=dev)
    torch.manual_seed(0)
    dec = loader_fused.random_decoder(loader_fused.QWEN3_VL_8B, rank, world, dev, seed=0,
                                      max_seq=BUCKET)
    # Decode o_proj/down all-reduce inside the projection kernel over NVLink
    # peer memory (Q3VL_PEER_AR=0 times the NCCL path instead).
    peer_ar = world > 1 and os.environ.get("Q3VL_PEER_AR", "1") == "1"
    if peer_ar:
        dec.enable_peer_allreduce()     # decode o_proj/down: in-kernel NVLink all-reduce
    # Q3VL_BENCH_KV=paged: the KV cache of every generate step lives in a page
    # pool (256-token pages, one slot per batch row) instead of contiguous
    # per-batch caches
    kv_mode = os.environ.get("Q3VL_BENCH_KV", "paged")
    gen_kw = {}
    if kv_mode == "paged":
        from q3vl.kv_pages import KVPagePool
        page = 256
        pool = KVPagePool(BATCH * (BUCKET // page), page, max_seqs=BATCH, buckets=(BUCKET,),
                          layers=dec.num_layers, kv_heads=dec.num_kv_heads, device=dev)
        gen_kw = {"kv_pages": pool}
    elif kv_mode != "contiguous":
        raise SystemExit(f"Q3VL_BENCH_KV={kv_mode!r}: expected contiguous or paged")
    g = torch.Generator().manual_seed(1234)
    prompt_host = torch.randint(0, 151936, (BATCH, PROMPT), generator=g).pin_memory()
    prompt = prompt_host.to(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    if args.profile:
        # profiling mode (for ncu launch lists): the same generate step with
        # --new-tokens decode tokens, no side measurements
        for _ in range(args.warmup + args.steps):
            dec.generate_tokens(prompt, args.new_tokens, eos_token_id=None, **gen_kw)
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"profile": True, "new_tokens": args.new_tokens,
                              "steps": args.warmup + args.steps}), flush=True)
        if world > 1:
            dec.close()
            dist.destroy_process_group()
        return

    # warm-up (includes CUDA-graph capture of the decode step)
    for _ in range(args.warmup):
        dec.generate_tokens(prompt, NEW_TOKENS, eos_token_id=None, **gen_kw)

    # launch accounting: one step run eagerly (graphs replay exactly these
    # kernels), counted by the library itself (q3_launch_count: every kernel
    # launch of every entry point, the split-K merge of decode attention
    # included when it runs as its own kernel)
    launch_count = _lib.raw("q3_launch_count")
    n0 = int(launch_count())
    dec.use_graphs = False
    dec.generate_tokens(prompt, NEW_TOKENS, eos_token_id=None, **gen_kw)
    dec.use_graphs = True
    launches_per_step = int(launch_count()) - n0
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            ev[i][0].record(stream)
            dec.generate_tokens(prompt, NEW_TOKENS, eos_token_id=None, prefill_done=ev[i][1],
                                **gen_kw)
            ev[i][2].record(stream)
        barrier()
    tot = sum(e[0].elapsed_time(e[2]) for e in ev)
    pre = sum(e[0].elapsed_time(e[1]) for e in ev)
    t = torch.tensor([tot, pre], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tot_ms, pre_ms = float(t[0]), float(t[1])
    dec_ms = tot_ms - pre_ms
    K = args.steps
    gen_tok = BATCH * NEW_TOKENS * K
    value = gen_tok / (tot_ms / 1e3)
    prefill_tps = BATCH * PROMPT * K / (pre_ms / 1e3)
    decode_tps = BATCH * (NEW_TOKENS - 1) * K / (dec_ms / 1e3)

    # ---- e2e through the public API: H2D prompt, D2H tokens each step ----
    e2e_ms = []
    for _ in range(max(2, min(3, K))):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        p = prompt_host.to(dev, non_blocking=True)
        toks = dec.generate_tokens(p, NEW_TOKENS, eos_token_id=None, **gen_kw).cpu()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms.append(e0.elapsed_time(e1))
    te = torch.tensor([sum(e2e_ms) / len(e2e_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = BATCH * NEW_TOKENS / (float(te[0]) / 1e3)

    # ---- per-kernel launch durations, as CUDA-graph replays (no host gaps) ----
    hbm, tflops, peak_kind = peaks()

    def graph_launch_ms(fns, reps=20):
        """Average device time of one call, over `reps` rounds of the calls in
        `fns` captured in one CUDA graph (inputs cycled so they exceed L2)."""
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for f in fns:
                f()
        torch.cuda.current_stream(dev).wait_stream(s)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            for _ in range(reps):
                for f in fns:
                    f()
        for _ in range(3):
            gr.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(3):
            gr.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (3 * reps * len(fns))
        del gr
        return ms

    # dominant kernel: the layer's gate/up projection exactly as the decode step
    # runs it (post-attention RMSNorm fused in from the o_proj's sums of
    # squares, SwiGLU epilogue); its 201 MB of weights exceed L2 on every call
    mlp = dec.layers[0].mlp_block
    H = 4096
    x = torch.randn(BATCH, H, device=dev).to(torch.bfloat16)
    w = mlp.gate_up_weight_il
    ss = (x.float() ** 2).view(BATCH, H // 64, 64).sum(-1).t().contiguous()
    ss = torch.nn.functional.pad(ss, (0, 16 - BATCH)).contiguous()      # [H/64, 16]
    act = torch.empty(BATCH, w.shape[0] // 2, dtype=torch.bfloat16, device=dev)
    fused_norm = dec.fuse_norm
    if fused_norm:
        gemv_fn = [lambda: ops.gemm_decode(x, w, "swiglu", norm_w=mlp.post_norm_weight,
                                           eps=mlp.eps, ss_in=ss, ss_tiles=H // 64, out=act)]
    else:
        gemv_fn = [lambda: ops.gemm(x, w, "swiglu", out=act)]
    gemv_ms = graph_launch_ms(gemv_fn)
    gemv_bytes = w.numel() * 2 + x.numel() * 2 + act.numel() * 2 + ss.numel() * 4
    gemv_gbs = gemv_bytes / (gemv_ms / 1e3) / 1e9

    # decode attention at the workload's mid-generation length; four KV sets
    # (151 MB) cycled so every launch reads its K/V from HBM
    L = PROMPT + NEW_TOKENS // 2
    ab = dec.layers[0].attn_block
    sets = []
    for _ in range(4):
        kc = torch.randn(BATCH, ab.num_kv_heads, BUCKET, 128, device=dev).to(torch.bfloat16)
        sets.append((kc, torch.randn_like(kc)))
    q = torch.randn(BATCH, ab.num_q_heads, 128, device=dev).to(torch.bfloat16)
    ao = torch.empty_like(q)
    attn_ms = graph_launch_ms([lambda kc=kc, vc=vc: ops.attn_decode(q, kc, vc, kv_len=L, out=ao)
                               for kc, vc in sets])
    attn_bytes = BATCH * ab.num_kv_heads * L * 128 * 2 * 2 + 2 * q.numel() * 2
    attn_gbs = attn_bytes / (attn_ms / 1e3) / 1e9
    del sets

    # decode-step bytes (weights + KV) for the whole-step HBM fraction
    n_params = sum(p.numel() for lyr in dec.layers for p in
                   (lyr.attn_block.qkv_weight_km, lyr.o_proj.weight_km,
                    lyr.mlp_block.gate_up_weight_il, lyr.mlp_block.down_weight_km))
    n_params += dec.lm_head.weight_km.numel()
    kv_step = 36 * BATCH * ab.num_kv_heads * (PROMPT + NEW_TOKENS // 2) * 128 * 2 * 2
    step_bytes = n_params * 2 + kv_step
    dec_step_ms = dec_ms / K / (NEW_TOKENS - 1)
    step_gbs = step_bytes / (dec_step_ms / 1e3) / 1e9

    clocks = clk.summary()
    if rank == 0:
        # the CPU baseline is measured on rank 0 of single-GPU runs only
        cpu = cpu_baseline() if (args.cpu_budget > 0 and world == 1) else None
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s",
            "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": round(tot_ms / K, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init N(0,0.02) bf16 weights, uniform random prompt ids)",
            "config": {"workload": WORKLOAD, "model": "Qwen3-VL-8B text decoder shape",
                       "global_batch": BATCH, "seq_len": PROMPT, "new_tokens": NEW_TOKENS,
                       "parallelism": f"tp{world}", "l2": "weights > L2 (126 MB) every step",
                       "tp_allreduce": ("decode: in-kernel NVLink peer push; prefill: NCCL"
                                        if peer_ar else ("NCCL" if world > 1 else "none")),
                       "kv_cache": ("paged (256-token pages)" if kv_mode == "paged"
                                    else f"contiguous per batch, bucket {BUCKET}"),
                       "prefill_attention": "tcgen05" if dec.prefill_tc else "mma.sync",
                       "prefill_allreduce": "two-shot over peer memory (q3_gemm_allreduce)"
                       if getattr(dec, "pcomm", None) is not None else
                       ("nccl" if args.gpus > 1 else "none"),
                       "l2_prefetch": "+".join(
                           n for n, on in (("o_proj", dec.l2_prefetch_oproj),
                                           ("next QKV", dec.l2_prefetch_qkv)) if on) or "none"},
            "prefill_tok_s": round(prefill_tps, 1), "decode_tok_s": round(decode_tps, 1),
            "decode_step_ms": round(dec_step_ms, 4),
            "decode_step_hbm": {"bytes": step_bytes, "achieved_gbs": round(step_gbs, 1),
                                "frac": round(step_gbs / hbm, 4)},
            "attention_hbm_gbs": round(attn_gbs, 1),
            "attention_hbm_frac": round(attn_gbs / hbm, 4),
            "attention_launch_ms": round(attn_ms, 5),
            "roofline": {"bound": "hbm",
                         "kernel": ("gemv_tma_kernel<1, SWIGLU, NORM> (gate_up, 8 tokens, "
                                    "post-attention RMSNorm fused)" if fused_norm else
                                    "gemv_tma_kernel<1, SWIGLU, 0> (gate_up, 8 tokens)"),
                         "achieved": round(gemv_gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gemv_gbs / hbm, 4),
                         "traffic": GEMV_TRAFFIC_BYTES if fused_norm else None,
                         "peak_source": f"{peak_kind} (burst copy)",
                         "bytes_per_launch": gemv_bytes, "launch_ms": round(gemv_ms, 5),
                         "timing": "CUDA-graph replay of 20 launches, events on the stream"},
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": BATCH * PROMPT * 8,
                    "d2h_bytes_per_step": BATCH * NEW_TOKENS * 8},
            "gpu_launches": launches_per_step * K,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dec.close()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle (restated reference decoder)
# ---------------------------------------------------------------------------
_CPU_MODEL = {}


def _cpu_oracle():
    """The CPU oracle (the reference decoder restated, model_fused.py:234-328)
    with the workload's 36 layers, built once per process.  All 36 layers use
    one layer's N(0, 0.02) weight tensors: the CPU time does not depend on the
    values, and a layer's 436 MB of weights exceeds the host caches, so every
    layer still streams its weights from memory."""
    if "o" not in _CPU_MODEL:
        import torch

        from oracle import decoder as odec
        spec = odec.Spec(max_seq=PROMPT + NEW_TOKENS)
        one = odec.make_weights(odec.Spec(layers=1, vocab=16), seed=0)
        g = torch.Generator().manual_seed(1)

        def rn(*shape):
            out = torch.empty(*shape, dtype=torch.bfloat16)
            for i in range(0, shape[0], 8192):     # fp32 draws in chunks
                n = min(8192, shape[0] - i)
                out[i:i + n] = (torch.randn(n, *shape[1:], generator=g) * 0.02).to(torch.bfloat16)
            return out
        w = dict(layers=one["layers"], embed=rn(spec.vocab, spec.hidden),
                 final_norm=one["final_norm"], lm_head=rn(spec.vocab, spec.hidden))
        o = odec.OracleDecoder(spec, w, tp=1)
        o.shards = o.shards * spec.layers      # the same tensors for every layer
        o.n_layers = spec.layers
        _CPU_MODEL["o"] = o
    return _CPU_MODEL["o"]


def host_cores():
    import torch
    aff = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"cpu_count": os.cpu_count(), "affinity": aff, "torch_threads": torch.get_num_threads()}


def cpu_baseline(decode_steps: int = 8):
    """Time the CPU oracle on a bounded sample of the workload, all 36 layers
    deep: the prefill of one of the 8 prompts (1024 tokens) with its lm_head,
    then `decode_steps` greedy decode steps of the whole batch of 8 at context
    1024 + i (the other rows' caches filled with noise).  Whole-workload time
    = 8 x the one-row prefill + (255 / decode_steps) x the sampled decode
    steps; returns the cpu_baseline object."""
    import torch

    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(threads)
    o = _cpu_oracle()
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 151936, (BATCH, PROMPT), generator=g)
    with torch.no_grad():
        caches = o.init_kv_cache(BATCH, PROMPT + NEW_TOKENS)
        for lyr in caches:
            for kc, vc in lyr:
                kc.normal_(generator=g)
                vc.normal_(generator=g)
        one = [[(kc[:1], vc[:1]) for kc, vc in lyr] for lyr in caches]
        t0 = time.perf_counter()
        nxt = o.forward(ids[:1], 0, one)[:, -1, :].argmax(-1)
        t_pf = time.perf_counter() - t0
        nxt = nxt.expand(BATCH).contiguous()
        t0 = time.perf_counter()
        for i in range(decode_steps):
            nxt = o.forward(nxt.view(BATCH, 1), PROMPT + i, caches)[:, -1, :].argmax(-1)
        t_dec = time.perf_counter() - t0
    total = BATCH * t_pf + (NEW_TOKENS - 1) / decode_steps * t_dec
    value = BATCH * NEW_TOKENS / total
    cores = host_cores()
    return {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"oracle (restated model_fused.py decoder, bf16), all 36 layers: prefill "
                       f"of 1 of the {BATCH} prompts ({PROMPT} tokens, {t_pf:.2f}s) and "
                       f"{decode_steps} decode steps of the batch of {BATCH} at context "
                       f"{PROMPT}+ ({t_dec / decode_steps:.3f}s/step); whole workload = "
                       f"{BATCH} x prefill + {NEW_TOKENS - 1}/{decode_steps} x the decode "
                       f"sample"),
            "host": cores,
            "prefill_tok_s": round(PROMPT / t_pf, 3),
            "decode_tok_s": round(BATCH * decode_steps / t_dec, 4)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import torch
    torch.set_num_threads(host_cores()["affinity"])
    vals = []
    o = _cpu_oracle()
    for _ in range(args.warmup):
        # warm-up: one decode step of the first layers (untimed)
        with torch.no_grad():
            kv = o.init_kv_cache(BATCH, 64)
            o.forward(torch.zeros(BATCH, 1, dtype=torch.long), 0, kv, n_layers=2)
    info = None
    for _ in range(args.steps):
        info = cpu_baseline(decode_steps=2)
        vals.append(info["value"])
    value = statistics.mean(vals)
    line = {"metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "model": "Qwen3-VL-8B text decoder shape",
                       "global_batch": BATCH, "seq_len": PROMPT, "new_tokens": NEW_TOKENS,
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": info["cores"],
                             "kind": "port", "sample": info["sample"], "host": info["host"]},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=1.0,
                    help="0 skips the cpu_baseline (the CPU oracle's bounded sample)")
    ap.add_argument("--profile", action="store_true",
                    help="run warmup+steps generate steps only (for ncu); prints no bench line")
    ap.add_argument("--new-tokens", type=int, default=NEW_TOKENS,
                    help="decode tokens per step in --profile mode")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
