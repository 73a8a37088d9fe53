"""Paged KV cache: page storage shared by every sequence plus its allocator.

The reference allocates one contiguous [B, Hkv, max_seq_len, D] K and V
tensor per layer for every request (init_kv_cache, model_fused.py:224-232).
A server that interleaves requests of different lengths wastes most of that.
Here the K/V storage of each layer is a pool of pages, [num_pages, Hkv,
page_tokens, D], and a sequence slot owns pages in position order (position
p -> page table[p // page_tokens], offset p % page_tokens).  The allocator is
host C++ (q3_kv_pages_*): bucketed, all-or-nothing, deterministic across
tensor-parallel ranks that issue the same calls.

Sizing on a 180 GB B200: the 8B decoder holds 2 x 8 KV heads x 128 x 2 bytes =
4 KiB per token per layer (TP1), 144 KiB per token over 36 layers, so 100 GB
of pages is about 700 k tokens.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

DEFAULT_BUCKETS = (2048, 4096, 8192)


class PagedLayer(tuple):
    """One layer's page pools as a (k_pages, v_pages) pair, plus the batch's
    device block table [B, width] int32: a drop-in for the (k_cache, v_cache)
    pair of a contiguous cache wherever the decoder takes one."""

    def __new__(cls, k_pages: torch.Tensor, v_pages: torch.Tensor, table: torch.Tensor):
        obj = super().__new__(cls, (k_pages, v_pages))
        obj.table = table
        return obj


def pages_for_bytes(nbytes: int, layers: int, kv_heads: int, page_tokens: int,
                    head_dim: int = 128, elem_bytes: int = 2) -> int:
    """Pages that fit in `nbytes` of device memory (K and V of every layer)."""
    per_page = 2 * layers * kv_heads * page_tokens * head_dim * elem_bytes
    return int(nbytes // per_page)


class KVPagePool:
    """Pages for `layers` decoder layers and the allocator that hands them out.

    With `device` and `layers`, K and V storage [num_pages, kv_heads,
    page_tokens, head_dim] is allocated per layer (`self.k[i]`, `self.v[i]`);
    without, only the allocator exists (host-side planning, tests)."""

    def __init__(self, num_pages: int, page_tokens: int = 256, *, max_seqs: int = 64,
                 buckets=DEFAULT_BUCKETS, max_pages_per_seq: int | None = None,
                 layers: int = 0, kv_heads: int = 0, head_dim: int = 128, device=None,
                 dtype=torch.bfloat16):
        buckets = tuple(int(b) for b in (buckets or ()))
        if max_pages_per_seq is None:
            max_pages_per_seq = (max(buckets) // page_tokens) if buckets else num_pages
        self.num_pages, self.page_tokens = int(num_pages), int(page_tokens)
        self.max_seqs, self.max_pages_per_seq = int(max_seqs), int(max_pages_per_seq)
        self.buckets = buckets
        arr = (ctypes.c_int64 * max(1, len(buckets)))(*buckets)
        handle = ctypes.c_void_p()
        _lib.call("q3_kv_pages_create", self.num_pages, self.page_tokens, self.max_seqs,
                  self.max_pages_per_seq, arr if buckets else None, len(buckets),
                  ctypes.byref(handle))
        self._h = handle
        self.k, self.v = [], []
        if device is not None and layers > 0:
            shape = (self.num_pages, kv_heads, self.page_tokens, head_dim)
            for _ in range(layers):
                self.k.append(torch.zeros(shape, dtype=dtype, device=device))
                self.v.append(torch.zeros(shape, dtype=dtype, device=device))

    # ------------------------------------------------------------- allocator
    def reserve(self, slot: int, tokens: int) -> int:
        """Grow `slot` to cover `tokens` positions; returns its capacity in
        tokens.  Raises Q3Error (status Q3_ERR_NO_MEMORY) when the pool is
        short, leaving every slot as it was."""
        cap = ctypes.c_int64()
        _lib.call("q3_kv_pages_reserve", self._h, int(slot), int(tokens), ctypes.byref(cap))
        return int(cap.value)

    def release(self, slot: int) -> None:
        _lib.call("q3_kv_pages_release", self._h, int(slot))

    def table(self, slots, width: int | None = None) -> torch.Tensor:
        """Block-table rows int32 [len(slots), width] (host); -1 past a slot's
        pages.  width defaults to max_pages_per_seq."""
        slots = [int(s) for s in slots]
        width = self.max_pages_per_seq if width is None else int(width)
        out = torch.empty(len(slots), width, dtype=torch.int32)
        sl = (ctypes.c_int32 * max(1, len(slots)))(*slots)
        _lib.call("q3_kv_pages_table", self._h, sl, len(slots), width,
                  ctypes.c_void_p(out.data_ptr()))
        return out

    def layers(self, table: torch.Tensor) -> list:
        """The per-layer PagedLayer list for a batch whose block table is `table`."""
        return [PagedLayer(k, v, table) for k, v in zip(self.k, self.v)]

    def device_table(self, slots, width: int | None = None, out: torch.Tensor = None,
                     device=None) -> torch.Tensor:
        """table() copied to the device (into `out`, whose address a captured
        decode graph may hold, when given)."""
        host = self.table(slots, width)
        if out is None:
            dev = device if device is not None else (self.k[0].device if self.k else "cuda")
            return host.to(dev)
        out.copy_(host)
        return out

    @property
    def free_pages(self) -> int:
        free = ctypes.c_int64()
        _lib.call("q3_kv_pages_stats", self._h, 0, ctypes.byref(free), None)
        return int(free.value)

    def slot_pages(self, slot: int) -> int:
        n = ctypes.c_int64()
        _lib.call("q3_kv_pages_stats", self._h, int(slot), None, ctypes.byref(n))
        return int(n.value)

    def close(self) -> None:
        if self._h is not None and self._h.value:
            _lib.raw("q3_kv_pages_destroy")(self._h)
        self._h = None
        self.k, self.v = [], []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
