"""CPU oracle for the Qwen3-VL tensor-parallel decoder path -- TEST INFRASTRUCTURE.

This package restates, in plain PyTorch on the CPU, the reference algorithm of
yahavb/qwen3-vl for the decoder hot path (model_fused.py / model.py,
kernels/*.py and the test oracles of test_kernels.py) and, for interleaved
M-RoPE, the published algorithm of transformers==5.5.0
(models/qwen3_vl/modeling_qwen3_vl.py), which the reference reaches only
through AutoModelForImageTextToText.  Every function cites the reference
file:line it follows.

It is the checker, never the product: only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline / reference arm may import it.  Parity is pinned
by tests/golden/, fixtures produced by running the reference's own Python code
(and HF's M-RoPE) in a container that holds the reference, with the generating
script tests/golden/make_golden.py committed beside them.
"""
