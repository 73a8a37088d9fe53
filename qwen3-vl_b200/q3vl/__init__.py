"""q3vl: B200 (sm_100a) kernels for the Qwen3-VL tensor-parallel decoder path.

`q3vl.ops` holds the torch-facing wrappers of the C ABI in include/q3vl.h,
`q3vl.layout` the weight re-layouts the kernels expect, `q3vl.engine` the
decoder runtime (KV buffers, CUDA-graph decode loop, tensor-parallel comm).
"""
from . import _lib, layout, ops  # noqa: F401

__all__ = ["ops", "layout"]
