"""Host-side checks of the C-ABI library (no GPU needed, no kernel launches):
it loads, exports every entry point include/q3vl.h declares, and rejects bad
arguments with a status and a message before touching the device."""
import ctypes
import os
import re

import pytest

from q3vl import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(REPO, "include", f) for f in os.listdir(os.path.join(REPO, "include"))
           if f.endswith(".h")]


def declared_symbols():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        names.update(re.findall(r"^Q3_API\s+[\w\s\*]+?\b(q3_\w+)\s*\(", src, flags=re.M))
    return names


def test_library_loads_and_reports_version():
    lib = _lib.load()
    assert lib.q3_version() >= 100


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.load()
    decl = declared_symbols()
    assert decl, "no declarations found in include/*.h"
    for name in sorted(decl):
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert decl == set(_lib.SIGNATURES) - set(), (
        f"ctypes table and header differ: {sorted(decl ^ set(_lib.SIGNATURES))}")


def test_invalid_arguments_are_rejected_on_the_host():
    lib = _lib.load()
    rc = lib.q3_gemm(None, None, None, 4, 16, 32, 0, None, None)
    assert rc == _lib.Q3_ERR_INVALID
    assert b"null" in lib.q3_last_error()
    one = ctypes.c_void_p(16)
    rc = lib.q3_gemm(one, one, one, 4, 10, 32, 0, None, None)          # N % 16 != 0
    assert rc == _lib.Q3_ERR_INVALID
    rc = lib.q3_attn_decode(one, one, one, one, 1, 6, 4, 128, 8, None, 16, 0.1, 1, None, 0,
                            None)                                       # Hq % Hkv != 0
    assert rc == _lib.Q3_ERR_INVALID
    rc = lib.q3_rope(one, one, one, 4, 2, 64, None)                      # head_dim != 128
    assert rc == _lib.Q3_ERR_INVALID
    rc = lib.q3_qkv_norm_rope(one, one, one, one, one, 1, 1, 0, 0, None, None, None, one, one,
                              1, 8, 4, 1, 128, 60, None, 64, 1e-6, None)  # cache overflow
    assert rc == _lib.Q3_ERR_INVALID
    assert b"max_seq" in lib.q3_last_error()
    # communicator set-up calls check their arguments before touching a device
    for fn in ("q3_comm_set_wait_limit", "q3_prefill_comm_set_wait_limit"):
        assert getattr(lib, fn)(None, 50_000_000) == _lib.Q3_ERR_INVALID
    for fn in ("q3_comm_attach_peer", "q3_prefill_comm_attach_peer"):
        assert getattr(lib, fn)(None, 1, one) == _lib.Q3_ERR_INVALID
    for fn in ("q3_comm_buffer", "q3_prefill_comm_buffer"):
        assert getattr(lib, fn)(None, None, None) == _lib.Q3_ERR_INVALID


def test_fused_entry_points_reject_bad_arguments_on_the_host():
    lib = _lib.load()
    one = ctypes.c_void_p(16)
    # fused prefill QKV: decode-sized token count (B*S <= 16) belongs to the GEMV path
    rc = lib.q3_gemm_qkv_rope(one, one, 4096, one, one, one, one, 1, 1, 0, 0, one, one, one,
                              1, 16, 32, 8, 128, 0, 2048, 1e-6, None)
    assert rc == _lib.Q3_ERR_INVALID and b"B*S > 16" in lib.q3_last_error()
    # ... and positions past the cache
    rc = lib.q3_gemm_qkv_rope(one, one, 4096, one, one, one, one, 1, 1, 0, 0, one, one, one,
                              2, 100, 32, 8, 128, 2000, 2048, 1e-6, None)
    assert rc == _lib.Q3_ERR_INVALID and b"outside the cache" in lib.q3_last_error()
    # decode attention from qkv: Hq must be a multiple of Hkv
    rc = lib.q3_attn_decode_qkv(one, one, one, one, one, 0, one, one, one, 1, 6, 4, 128, 8,
                                None, 16, 0.1, 1e-6, None, 0, None)
    assert rc == _lib.Q3_ERR_INVALID
    # tcgen05 prefill attention: the cache must hold the prompt's positions
    strides = (ctypes.c_int64 * 3)(8 * 128 * 100, 128, 8 * 128)
    rc = lib.q3_attn_prefill_tc(one, one, one, one, 1, 8, 2, 100, 128, 50, 1, 0.1, 120, strides,
                                0, None)
    assert rc == _lib.Q3_ERR_INVALID and b"rows per head" in lib.q3_last_error()
    rc = lib.q3_attn_prefill_tc(one, one, one, one, 1, 8, 2, 100, 64, 0, 1, 0.1, 128, strides,
                                0, None)
    assert rc == _lib.Q3_ERR_INVALID and b"head_dim" in lib.q3_last_error()
    rc = lib.q3_attn_prefill_tc(one, one, one, one, 1, 8, 2, 100, 128, 0, 1, 0.1, 128, strides,
                                3, None)
    assert rc == _lib.Q3_ERR_INVALID and b"variant" in lib.q3_last_error()
    rc = lib.q3_attn_prefill_tc(one, one, one, one, 1, 6, 2, 100, 128, 0, 1, 0.1, 128, strides,
                                2, None)                               # Hq/Hkv odd
    assert rc == _lib.Q3_ERR_INVALID and b"variant 2" in lib.q3_last_error()
    rc = lib.q3_attn_prefill_tc(one, one, one, one, 1, 8, 2, 100, 64, 0, 1, 0.1, 128, strides,
                                1, None)
    assert rc == _lib.Q3_ERR_INVALID and b"head_dim" in lib.q3_last_error()
    # paged attention: positions must stay inside the block table
    rc = lib.q3_attn_prefill_paged(one, one, one, one, 1, 8, 2, 100, 128, 200, 1, 0.1, strides,
                                   strides, one, 4, 64, 16, None)
    assert rc == _lib.Q3_ERR_INVALID and b"table width" in lib.q3_last_error()
    rc = lib.q3_attn_decode_paged(one, one, one, one, 1, 8, 2, 128, 300, None, one, 4, 64, 16,
                                  0.1, None, 0, None)
    assert rc == _lib.Q3_ERR_INVALID and b"table width" in lib.q3_last_error()
    # distributed argmax keys hold 32-bit vocabulary indices
    rc = lib.q3_argmax_key(one, 8, 1 << 16, (1 << 32) - 8, one, None)
    assert rc == _lib.Q3_ERR_INVALID and b"32 bits" in lib.q3_last_error()
    # position ids: merge size must be positive
    rc = lib.q3_rope_index(one, None, 1, 16, None, 0, None, 0, 0, one, one, one, one, 64, None)
    assert rc == _lib.Q3_ERR_INVALID and b"merge" in lib.q3_last_error()
    # in-kernel all-reduce needs a communicator
    rc = lib.q3_gemm_ar(one, one, one, 8, 4096, 512, None, None, None, None)
    assert rc == _lib.Q3_ERR_INVALID and b"null" in lib.q3_last_error()
    # decode projection: sums of squares come out of the residual epilogue only
    rc = lib.q3_gemm_decode(one, one, one, 8, 4096, 4096, 0, None, None, 1e-6, None, 0, one,
                            None)
    assert rc == _lib.Q3_ERR_INVALID and b"residual" in lib.q3_last_error()
    # gate/up + SwiGLU: the fused norm is for decode shapes; inter must be a multiple of 8
    rc = lib.q3_gate_up_swiglu(one, one, one, 64, 12288, 4096, one, 1e-6, None)
    assert rc == _lib.Q3_ERR_INVALID and b"M <= 16" in lib.q3_last_error()
    rc = lib.q3_gate_up_swiglu(one, one, one, 8, 100, 4096, None, 1e-6, None)
    assert rc == _lib.Q3_ERR_INVALID and b"inter" in lib.q3_last_error()
    # lm_head + argmax: indices over a slice need keys; the fused norm needs <= 16 rows
    rc = lib.q3_lm_head_argmax(one, None, 1e-6, one, 8, 18992, 4096, 18992, one, 0, one, None)
    assert rc == _lib.Q3_ERR_INVALID and b"need keys" in lib.q3_last_error()
    rc = lib.q3_lm_head_argmax(one, one, 1e-6, one, 32, 18992, 4096, 0, one, 0, one, None)
    assert rc == _lib.Q3_ERR_INVALID and b"rows <= 16" in lib.q3_last_error()
    # ... and the projection's own checks still apply (V % 16)
    rc = lib.q3_lm_head_argmax(one, None, 1e-6, one, 4, 1000, 4096, 0, one, 0, one, None)
    assert rc == _lib.Q3_ERR_INVALID and b"multiple of 16" in lib.q3_last_error()
    # L2 prefetch: 16-byte aligned start, whole 16-byte units
    rc = lib.q3_l2_prefetch(one, 100, None)
    assert rc == _lib.Q3_ERR_INVALID and b"multiple of 16" in lib.q3_last_error()
    rc = lib.q3_l2_prefetch(ctypes.c_void_p(24), 160, None)
    assert rc == _lib.Q3_ERR_INVALID and b"aligned" in lib.q3_last_error()
    # prefill all-reduce: a communicator, and column counts in whole 32-column chunks
    rc = lib.q3_gemm_allreduce(one, one, one, 64, 4096, 4096, None, None, None)
    assert rc == _lib.Q3_ERR_INVALID and b"null" in lib.q3_last_error()
    comm = ctypes.c_void_p()
    blob = ctypes.create_string_buffer(64)
    rc = lib.q3_prefill_comm_create(0, 2, 8192, 4100, ctypes.byref(comm), blob)
    assert rc == _lib.Q3_ERR_INVALID and b"multiple of 32" in lib.q3_last_error()
    rc = lib.q3_prefill_comm_create(2, 2, 8192, 4096, ctypes.byref(comm), blob)
    assert rc == _lib.Q3_ERR_INVALID and b"rank 2 / world 2" in lib.q3_last_error()
    assert not comm.value
    # communicator set-up needs a communicator
    rc = lib.q3_init_comm(None, 0, 2, one)
    assert rc == _lib.Q3_ERR_INVALID and b"null" in lib.q3_last_error()
    # whole-step kernel: 1..16 sequences
    plan = ctypes.c_void_p()
    layer = _lib.StepLayer()
    rc = lib.q3_decode_step_create(ctypes.byref(layer), 1, 17, 4096, 32, 8, 12288, 2048, 1e-6,
                                   one, one, 2048, ctypes.byref(plan))
    assert rc == _lib.Q3_ERR_INVALID and b"batch" in lib.q3_last_error()
    assert not plan.value


def test_error_raises_q3error():
    with pytest.raises(_lib.Q3Error) as e:
        _lib.call("q3_rmsnorm", None, None, None, None, None, 1, 8, 1e-6, None)
    assert e.value.status == _lib.Q3_ERR_INVALID


def test_decode_workspace_sizing_is_host_only():
    f = _lib.raw("q3_attn_decode_workspace_bytes")
    assert f(1, 32, 8, 128, 1024) > 0
    assert f(0, 32, 8, 128, 1024) == 0


def test_noalloc_bound_holds_for_supported_shapes():
    """q3_attn_decode_noalloc keeps split-K partials in a 4 MiB built-in array.
    Its need is the workspace q3_attn_decode asks for (same split plan).  With
    no GPU the plan assumes a 148-SM B200: every supported shape stays under
    the limit, so the entry point's refusal only matters on larger GPUs."""
    f = _lib.raw("q3_attn_decode_workspace_bytes")
    worst = 0
    for B in (1, 2, 3, 4, 7, 8, 16, 32, 37, 64, 128, 256, 512):
        for Hkv in (1, 2, 4, 8):
            for G in (1, 2, 4, 8):
                for L in (1, 63, 64, 1000, 1024, 2048, 8192, 32768, 262144):
                    worst = max(worst, f(B, Hkv * G, Hkv, 128, L))
    assert 0 < worst <= 4 << 20, worst
    assert worst <= 4 * 148 * 8 * 520


def test_ops_refuse_cpu_tensors():
    import torch
    from q3vl import ops
    x = torch.zeros(2, 4096, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rmsnorm(x, torch.ones(4096, dtype=torch.bfloat16))


def test_header_is_plain_c():
    """include/*.h is the boundary for foreign bindings: it must compile as C99."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    for h in HEADERS:
        r = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x",
                            "c", h], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
