"""Peer-memory communicator for the fused row-parallel projection + all-reduce.

Each rank allocates one device buffer through the C ABI (q3_comm_create); the
CUDA IPC handles are all-gathered over the existing torch.distributed process
group and opened by every rank (q3_comm_open_peers), so the q3_gemm_ar kernel
can push its partial tiles straight into the peers' memory over NVLink.
torch.distributed is used only for this one-time handle exchange.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call


class PeerComm:
    def __init__(self, group=None, max_cols: int = 16384, device=None):
        if not dist.is_initialized():
            raise RuntimeError("PeerComm needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nb = int(lib.q3_comm_handle_bytes())
        handle = (ctypes.c_char * nb)()
        self._ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("q3_comm_create", self.rank, self.world, int(max_cols), ctypes.byref(self._ptr),
                 handle)
        mine = torch.tensor(bytearray(handle.raw), dtype=torch.uint8)
        backend = dist.get_backend(group)
        mine = mine.to(self.device) if backend == "nccl" else mine
        every = torch.empty(self.world * nb, dtype=torch.uint8, device=mine.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        blob = bytes(every.cpu().numpy().tobytes())
        with torch.cuda.device(self.device):
            call("q3_comm_open_peers", self._ptr, ctypes.c_char_p(blob))
        dist.barrier(group=group)
        self.max_cols = max_cols

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._ptr

    def set_wait_limit(self, seconds: float) -> None:
        """Bound of each in-kernel wait on a peer (q3_comm_set_wait_limit;
        1 ms .. 60 s, default 2 s)."""
        call("q3_comm_set_wait_limit", self._ptr, int(seconds * 1e9))

    def close(self):
        if self._ptr is not None and self._ptr.value:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            call("q3_comm_destroy", self._ptr)
            self._ptr = ctypes.c_void_p()


class PrefillComm:
    """The exchange buffers of the prefill all-reduce (q3_gemm_allreduce): one
    IPC-shared device buffer per rank holding every source's receive stripe,
    the reduced stripe and the flags, sized for calls of up to max_rows x
    max_cols outputs.  Collective: every rank of `group` constructs it."""

    def __init__(self, group=None, max_rows: int = 8192, max_cols: int = 4096, device=None):
        if not dist.is_initialized():
            raise RuntimeError("PrefillComm needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nb = int(lib.q3_comm_handle_bytes())
        handle = (ctypes.c_char * nb)()
        self._ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("q3_prefill_comm_create", self.rank, self.world, int(max_rows), int(max_cols),
                 ctypes.byref(self._ptr), handle)
        mine = torch.tensor(bytearray(handle.raw), dtype=torch.uint8)
        mine = mine.to(self.device) if dist.get_backend(group) == "nccl" else mine
        every = torch.empty(self.world * nb, dtype=torch.uint8, device=mine.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        blob = bytes(every.cpu().numpy().tobytes())
        with torch.cuda.device(self.device):
            call("q3_prefill_comm_open", self._ptr, ctypes.c_char_p(blob))
        dist.barrier(group=group)
        self.max_rows, self.max_cols = max_rows, max_cols

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._ptr

    def set_wait_limit(self, seconds: float) -> None:
        """Bound of each in-kernel wait on a peer (q3_prefill_comm_set_wait_limit;
        1 ms .. 60 s, default 2 s)."""
        call("q3_prefill_comm_set_wait_limit", self._ptr, int(seconds * 1e9))

    def close(self):
        if self._ptr is not None and self._ptr.value:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            call("q3_prefill_comm_destroy", self._ptr)
            self._ptr = ctypes.c_void_p()


class SoloComm:
    """A single-rank communicator (q3_comm_create with world 1), for the
    decode step kernel on one GPU: its all-reduce is the identity, and no
    process group is needed."""

    def __init__(self, max_cols: int = 16384, device=None):
        self.device = torch.device(device) if device is not None else \
            torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        nb = int(lib.q3_comm_handle_bytes())
        self._ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("q3_comm_create", 0, 1, int(max_cols), ctypes.byref(self._ptr),
                 (ctypes.c_char * nb)())
        self.rank, self.world, self.max_cols = 0, 1, max_cols

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._ptr

    def close(self):
        if self._ptr is not None and self._ptr.value:
            call("q3_comm_destroy", self._ptr)
            self._ptr = ctypes.c_void_p()

