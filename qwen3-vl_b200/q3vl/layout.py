"""Weight re-layouts between the reference's [in, out] convention and the
K-major [out, in] storage the q3vl kernels read.

The reference multiplies x @ W with W stored [in, out] (loader_fused.py:90,
101, 106, 109, 157).  The tensor-core and streaming kernels read weights as
[N, K] rows with contiguous K, so modules keep one K-major copy and expose the
[in, out] view (`.t()`) for API compatibility.

Gate/up for the fused SwiGLU epilogue are interleaved in blocks of 8 rows:
rows 16j..16j+7 are gate rows 8j..8j+7 and rows 16j+8..16j+15 the matching up
rows, so one 16-row block (decode kernel) or one 32-column TMEM chunk
(tcgen05 kernel) holds both halves of the same output features.
"""
from __future__ import annotations

import torch


def k_major(w_in_out: torch.Tensor) -> torch.Tensor:
    """[in, out] -> contiguous [out, in]."""
    return w_in_out.t().contiguous()


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gate, up [I, H] (K-major) -> [2I, H] in 8-row gate/up blocks."""
    if gate.shape != up.shape or gate.shape[0] % 8:
        raise ValueError("gate/up must share a shape with I % 8 == 0")
    I, H = gate.shape
    return torch.stack([gate.view(I // 8, 8, H), up.view(I // 8, 8, H)], dim=1).reshape(2 * I, H)


def deinterleave_gate_up(w: torch.Tensor):
    """Inverse of interleave_gate_up: [2I, H] -> (gate [I, H], up [I, H])."""
    I2, H = w.shape
    v = w.view(I2 // 16, 2, 8, H)
    return v[:, 0].reshape(I2 // 2, H), v[:, 1].reshape(I2 // 2, H)


def gate_up_from_fused(gate_up_in_out: torch.Tensor) -> torch.Tensor:
    """Reference fused [H, 2I] ([gate | up] columns, loader_fused.py:104-106) ->
    interleaved K-major [2I, H]."""
    H, I2 = gate_up_in_out.shape
    gate = gate_up_in_out[:, :I2 // 2].t()
    up = gate_up_in_out[:, I2 // 2:].t()
    return interleave_gate_up(gate.contiguous(), up.contiguous())


def fused_from_gate_up(w: torch.Tensor) -> torch.Tensor:
    """Interleaved K-major [2I, H] -> reference fused [H, 2I] ([gate | up])."""
    gate, up = deinterleave_gate_up(w)
    return torch.cat([gate, up], dim=0).t()
