"""ctypes binding of libq3vl.so (the C ABI declared in include/q3vl.h).

The library is loaded once per process.  There is no fallback: if the shared
object is missing or fails to load, every op raises.  Entry points return an
int status; non-zero statuses raise `Q3Error` with the library's message.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libq3vl.so")

(Q3_OK, Q3_ERR_INVALID, Q3_ERR_UNSUPPORTED, Q3_ERR_CUDA, Q3_ERR_TIMEOUT, Q3_ERR_COMM,
 Q3_ERR_NO_MEMORY) = range(7)
Q3_F32, Q3_BF16 = 0, 1
Q3_EPI_NONE, Q3_EPI_RESIDUAL, Q3_EPI_SWIGLU = 0, 1, 2
Q3_EPI_BIAS, Q3_EPI_BIAS_GELU_TANH, Q3_EPI_BIAS_GELU, Q3_EPI_BIAS_RESIDUAL = 3, 4, 5, 6

_STATUS_NAMES = {
    Q3_ERR_INVALID: "invalid argument",
    Q3_ERR_UNSUPPORTED: "unsupported",
    Q3_ERR_CUDA: "CUDA error",
    Q3_ERR_TIMEOUT: "in-kernel wait timed out",
    Q3_ERR_COMM: "communication error",
    Q3_ERR_NO_MEMORY: "pool exhausted",
}


class Q3Error(RuntimeError):
    def __init__(self, status: int, fn: str, msg: str):
        super().__init__(f"{fn}: {_STATUS_NAMES.get(status, 'error')} ({status}): {msg}")
        self.status = status


P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
F32 = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "q3_version": (I32, []),
    "q3_last_error": (ctypes.c_char_p, []),
    "q3_launch_count": (ctypes.c_uint64, []),
    "q3_device_error": (I32, [I32]),
    "q3_rmsnorm": (I32, [P, P, P, P, P, I64, I64, F32, P]),
    "q3_rope": (I32, [P, P, P, I64, I32, I32, P]),
    "q3_mrope_cos_sin": (I32, [P, P, I64, I32, I32, I32, P, P, P]),
    "q3_gemm_bias": (I32, [P, P, P, P, I64, I64, I64, I32, P, P]),
    "q3_layernorm": (I32, [P, P, P, P, I64, I64, F32, P]),
    "q3_vision_pos_embed": (I32, [P, I32, I32, P, P, I32, I32, I64, P, P]),
    "q3_vision_rope": (I32, [P, I32, I32, P, P, P, I32, I32, I64, P]),
    "q3_vision_attention": (I32, [P, P, I32, I32, P, P, I32, I64, P]),
    "q3_kv_pages_create": (I32, [I32, I32, I32, I32, P, I32, P]),
    "q3_kv_pages_destroy": (I32, [P]),
    "q3_kv_pages_reserve": (I32, [P, I32, I64, P]),
    "q3_kv_pages_release": (I32, [P, I32]),
    "q3_kv_pages_table": (I32, [P, P, I32, I32, P]),
    "q3_kv_pages_stats": (I32, [P, I32, P, P]),
    "q3_gemm_qkv_rope_paged": (I32, [P, P, I64, P, P, P, P, I32, I32, I64, I64, P, P, P, I32,
                                     I32, I32, I32, I32, I64, P, I64, I32, I32, F32, P]),
    "q3_qkv_norm_rope_paged": (I32, [P, P, P, P, P, I32, I32, I64, I64, P, P, P, I32, I32, I32,
                                     I32, I32, I64, P, P, I64, I32, I32, F32, P]),
    "q3_attn_prefill_tc": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I64, I32, F32, I64, P, I32, P]),
    "q3_attn_prefill_tc_paged": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I64, I32, F32, P, P,
                                       I64, I32, I32, P]),
    "q3_attn_prefill_paged": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I64, I32, F32, P, P, P,
                                    I64, I32, I32, P]),
    "q3_kv_pages_write": (I32, [P, P, P, P, I32, I32, I32, I32, P, I64, I32, I32, I64, P, P]),
    "q3_attn_decode_paged": (I32, [P, P, P, P, I32, I32, I32, I32, I64, P, P, I64, I32, I32, F32,
                                   P, SZ, P]),
    "q3_rope_index_workspace_bytes": (SZ, [I32]),
    "q3_rope_index": (I32, [P, P, I32, I64, P, I32, P, I32, I32, P, P, P, P, SZ, P]),
    "q3_qkv_norm_rope": (I32, [P, P, P, P, P, I32, I32, I64, I64, P, P, P, P, P, I32, I32, I32,
                               I32, I32, I64, P, I64, F32, P]),
    "q3_attn_decode_workspace_bytes": (SZ, [I32, I32, I32, I32, I64]),
    "q3_attn_decode": (I32, [P, P, P, P, I32, I32, I32, I32, I64, P, I64, F32, I32, P, SZ, P]),
    "q3_attn_decode_qkv": (I32, [P, P, P, P, P, I64, P, P, P, I32, I32, I32, I32, I64, P, I64,
                                 F32, F32, P, SZ, P]),
    "q3_attn_decode_qkv_paged": (I32, [P, P, P, P, P, I64, P, P, P, I32, I32, I32, I32, I64, P,
                                       P, I64, I32, I32, F32, F32, P, SZ, P]),
    "q3_attn_decode_noalloc": (I32, [P, P, P, P, I32, I32, I32, I32, I64, P, I64, F32, I32, P]),
    "q3_attn_prefill": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I64, I32, F32, P, P, P, P]),
    "q3_gemm": (I32, [P, P, P, I64, I64, I64, I32, P, P]),
    "q3_gemm_norm": (I32, [P, P, F32, P, P, I64, I64, I64, I32, P, P]),
    "q3_gate_up_swiglu": (I32, [P, P, P, I64, I64, I64, P, F32, P]),
    "q3_gemm_qkv_rope": (I32, [P, P, I64, P, P, P, P, I32, I32, I64, I64, P, P, P, I32, I32,
                               I32, I32, I32, I64, I64, F32, P]),
    "q3_gemm_decode": (I32, [P, P, P, I64, I64, I64, I32, P, P, F32, P, I32, P, P]),
    "q3_comm_handle_bytes": (I32, []),
    "q3_comm_create": (I32, [I32, I32, I64, ctypes.POINTER(P), P]),
    "q3_comm_open_peers": (I32, [P, P]),
    "q3_prefill_comm_create": (I32, [I32, I32, I64, I64, P, P]),
    "q3_prefill_comm_open": (I32, [P, P]),
    "q3_prefill_comm_destroy": (I32, [P]),
    "q3_gemm_allreduce": (I32, [P, P, P, I64, I64, I64, P, P, P]),
    "q3_init_comm": (I32, [P, I32, I32, P]),
    "q3_comm_destroy": (I32, [P]),
    "q3_gemm_ar": (I32, [P, P, P, I64, I64, I64, P, P, P, P]),
    "q3_comm_buffer": (I32, [P, ctypes.POINTER(P), ctypes.POINTER(SZ)]),
    "q3_comm_attach_peer": (I32, [P, I32, P]),
    "q3_comm_set_wait_limit": (I32, [P, ctypes.c_uint64]),
    "q3_prefill_comm_buffer": (I32, [P, ctypes.POINTER(P), ctypes.POINTER(SZ)]),
    "q3_prefill_comm_attach_peer": (I32, [P, I32, P]),
    "q3_prefill_comm_set_wait_limit": (I32, [P, ctypes.c_uint64]),
    "q3_decode_step_create": (I32, [P, I32, I32, I32, I32, I32, I32, I64, F32, P, P, I64,
                                    ctypes.POINTER(P)]),
    "q3_decode_step": (I32, [P, P, P, P, I64, P]),
    "q3_decode_step_destroy": (I32, [P]),
    "q3_decode_tp_create": (I32, [P, I32, I32, I32, I32, I32, I32, I64, F32, P, P, I64, P,
                                  ctypes.POINTER(P)]),
    "q3_decode_tp_create_paged": (I32, [P, I32, I32, I32, I32, I32, I32, I64, F32, P, P, I64, P,
                                        P, I32, I32, I64, ctypes.POINTER(P)]),
    "q3_decode_tp": (I32, [P, P, P, I64, P]),
    "q3_decode_tp_destroy": (I32, [P]),
    "q3_embed": (I32, [P, P, P, I64, I64, I64, P]),
    "q3_add": (I32, [P, P, P, I64, P]),
    "q3_argmax": (I32, [P, I64, I64, P, P]),
    "q3_argmax_key": (I32, [P, I64, I64, I64, P, P]),
    "q3_argmax_key_index": (I32, [P, I64, P, P]),
    "q3_lm_head_argmax": (I32, [P, P, F32, P, I64, I64, I64, I64, P, I32, P, P]),
    "q3_l2_prefetch": (I32, [P, I64, P]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libq3vl.so (raises if it is absent: there is no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} not found: build it with `python qwen3-vl_b200/build.py` "
                "(the q3vl ops have no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class StepLayer(ctypes.Structure):
    """q3_step_layer of include/q3vl.h (device pointers of one decoder layer)."""
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("w_qkv", "w_o", "w_gate_up", "w_down", "input_norm", "post_norm", "q_norm",
                 "k_norm", "k_cache", "v_cache")]


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != Q3_OK:
        msg = lib.q3_last_error().decode(errors="replace")
        raise Q3Error(rc, name, msg)


def raw(name: str):
    return getattr(load(), name)
