"""Bounded peer waits on one GPU, without faulting or hanging anything.

A world-2 communicator is built for rank 0 whose rank-1 "peer" buffer is a
second communicator's buffer on the same GPU (q3_comm_attach_peer).  Nothing
ever runs rank 1, so rank 0's exchange pushes its partials into that buffer
and then waits for rank 1's words, which never come.  With the wait limit set
to 50 ms (q3_comm_set_wait_limit) the kernel must give up, record the peer
timeout code in the device error word (0x501 for the decode all-reduce,
0x701 / 0x702 for the prefill two-shot exchange), and complete; the host
turns that into Q3_ERR_TIMEOUT (ops.check_device_error).  The next call on a
fresh communicator must then succeed: the context stays usable.

Only one kernel waits at any time and nothing waits on another launch, so no
two launches on this GPU depend on each other."""
import ctypes
import time

import pytest
import torch

from q3vl import _lib, ops
from q3vl._lib import call
from tests.helpers import compare

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
LIMIT_NS = 50_000_000


class _Comm:
    """A communicator made straight through the C ABI (no process group)."""

    def __init__(self, rank, world, *, prefill=False, max_rows=512, max_cols=4096):
        self.prefill = prefill
        nb = int(_lib.load().q3_comm_handle_bytes())
        self._h = (ctypes.c_char * nb)()
        self.handle = ctypes.c_void_p()
        if prefill:
            call("q3_prefill_comm_create", rank, world, max_rows, max_cols,
                 ctypes.byref(self.handle), self._h)
        else:
            call("q3_comm_create", rank, world, max_cols, ctypes.byref(self.handle), self._h)

    def buffer(self):
        ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        fn = "q3_prefill_comm_buffer" if self.prefill else "q3_comm_buffer"
        call(fn, self.handle, ctypes.byref(ptr), ctypes.byref(nbytes))
        return ptr, nbytes.value

    def attach(self, rank, buf):
        call("q3_prefill_comm_attach_peer" if self.prefill else "q3_comm_attach_peer",
             self.handle, rank, buf)

    def set_wait_limit(self, ns):
        call("q3_prefill_comm_set_wait_limit" if self.prefill else "q3_comm_set_wait_limit",
             self.handle, ns)

    def close(self):
        call("q3_prefill_comm_destroy" if self.prefill else "q3_comm_destroy", self.handle)


def rnd(*shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(DEV)


def _timed(fn):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    return time.perf_counter() - t0


@pytest.mark.parametrize("prefill", [False, True], ids=["decode_gemm_ar", "prefill_allreduce"])
def test_a_peer_that_never_arrives_times_out_and_the_next_call_succeeds(prefill):
    M = 256 if prefill else 1
    N, K = 1024, 512
    x, w, r = rnd(M, K, seed=1), rnd(N, K, seed=2, scale=0.05), rnd(M, N, seed=3)
    run = ops.gemm_allreduce if prefill else ops.gemm_ar
    ops.device_error(clear=True)

    rank0 = _Comm(0, 2, prefill=prefill)
    idle_rank1 = _Comm(1, 2, prefill=prefill)   # its buffer stands in for rank 1's; never run
    try:
        buf, nbytes = idle_rank1.buffer()
        assert buf.value and nbytes > 0
        rank0.attach(1, buf)
        with pytest.raises(_lib.Q3Error, match="already has a buffer"):
            rank0.attach(1, buf)
        with pytest.raises(_lib.Q3Error, match="outside"):
            rank0.set_wait_limit(10)
        rank0.set_wait_limit(LIMIT_NS)
        out = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
        dt = _timed(lambda: run(x, w, rank0, residual=r, out=out))
        code = ops.device_error(clear=False)
        want = (0x701, 0x702) if prefill else (0x501,)
        assert code in want, f"device error word {code:#x}, expected one of {want}"
        with pytest.raises(_lib.Q3Error) as e:
            ops.check_device_error("gemm all-reduce")
        assert e.value.status == _lib.Q3_ERR_TIMEOUT
        assert ops.device_error() == 0
        # the 50 ms limit applied, not the 2 s default (each tile waits once;
        # the tiles wait side by side)
        assert dt < 1.0, f"the timed-out call took {dt:.3f} s"
    finally:
        rank0.close()
        idle_rank1.close()

    # the context is still usable: a fresh single-rank communicator reduces
    # over itself, so its result is residual + x @ w.T
    solo = _Comm(0, 1, prefill=prefill)
    try:
        out = run(x, w, solo, residual=r)
        torch.cuda.synchronize()
        ops.check_device_error("gemm all-reduce")
        ref = r.float() + (x.float() @ w.float().t()).to(torch.bfloat16).float()
        compare("after the timeout", out.float(), ref, max_abs=3e-2, rel_scale=True,
                min_cos=0.9999)
    finally:
        solo.close()
