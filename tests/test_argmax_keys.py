"""The distributed greedy argmax's key scheme (csrc/misc.cu argmax_key),
restated bit for bit on the host: a per-rank key of (value, global index)
whose MAX over ranks decodes to torch.argmax of the concatenated row (first
index on ties).  CPU only; the kernels themselves are checked in
tests/test_kernels_gpu.py."""
import numpy as np
import pytest
import torch


def key(v: float, gidx: int) -> int:
    """int64 key: high word = the float's bits mapped to signed integer order,
    low word = 0xffffffff - index (smaller index wins a tie)."""
    u = int(np.array([np.float32(v) + np.float32(0.0)], dtype=np.float32).view(np.uint32)[0])
    ordv = (~u & 0xffffffff) if (u & 0x80000000) else (u | 0x80000000)
    hi = int(np.array([ordv ^ 0x80000000], dtype=np.uint32).view(np.int32)[0])
    return (hi << 32) | (0xffffffff - gidx)


def decode(k: int) -> int:
    return 0xffffffff - (k & 0xffffffff)


def slice_key(row: np.ndarray, offset: int) -> int:
    """What one rank's argmax_kernel<true> writes for its slice: the first
    maximum (NaN-free rows; an all -inf slice reports its first index)."""
    best, bi = -np.inf, None
    for j, f in enumerate(row):
        if f > best:
            best, bi = f, j
    return key(float(best), offset + (0 if bi is None else bi))


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("seed", range(4))
def test_max_of_slice_keys_is_the_first_argmax(tp, seed):
    rng = np.random.default_rng(seed)
    V = 64 * tp
    rows = [rng.standard_normal(V).astype(np.float32),
            -np.abs(rng.standard_normal(V)).astype(np.float32) - 1,      # all negative
            np.full(V, 2.5, np.float32),                                  # all equal
            np.round(rng.standard_normal(V) * 2).astype(np.float32),     # many ties
            np.full(V, -np.inf, np.float32),
            np.array([1e-45, -1e-45, 0.0, -0.0] * (V // 4), np.float32),  # subnormals, +-0
            np.concatenate([np.full(V // 2, -0.0, np.float32),             # -0 maximum first,
                            np.full(V // 2, 0.0, np.float32)])]             # +0 in a later slice
    for row in rows:
        n = V // tp
        k = max(slice_key(row[r * n:(r + 1) * n], r * n) for r in range(tp))
        want = int(torch.from_numpy(row.copy()).argmax())
        assert decode(k) == want, (row[:8], decode(k), want)


def test_keys_order_like_floats():
    vals = [-np.inf, -3.0, -1e-30, -1e-45, -0.0, 0.0, 1e-45, 1e-30, 2.0, np.inf]
    ks = [key(v, 7) for v in vals]
    assert ks == sorted(ks)
    assert key(-0.0, 7) == key(0.0, 7)                 # equal floats, equal keys
    assert key(1.0, 3) > key(1.0, 4) > key(0.999, 0)
