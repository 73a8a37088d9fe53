"""Shared helpers for the test suite (fixture loading, tolerance checks)."""
import os

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def bf16_from_np(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def as_tensor(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return bf16_from_np(a)
    return torch.from_numpy(a.copy())


def compare(name, got, want, max_abs=None, min_cos=None, rel_scale=False):
    """Assert max-abs (optionally relative to max|want|) and cosine similarity."""
    g = got.detach().double().cpu().flatten()
    w = want.detach().double().cpu().flatten()
    assert g.shape == w.shape, f"{name}: shape {tuple(got.shape)} vs {tuple(want.shape)}"
    assert torch.isfinite(g).all(), f"{name}: non-finite output"
    diff = (g - w).abs().max().item()
    scale = w.abs().max().item() if rel_scale else 1.0
    cos = torch.nn.functional.cosine_similarity(g, w, dim=0).item()
    if max_abs is not None:
        assert diff <= max_abs * scale, f"{name}: max|diff|={diff:.3e} > {max_abs * scale:.3e}"
    if min_cos is not None:
        assert cos >= min_cos, f"{name}: cosine {cos:.7f} < {min_cos}"
    return diff, cos
