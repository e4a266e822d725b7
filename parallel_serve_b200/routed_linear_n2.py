"""Drop-in for ``experiments/routed_linear_n2.py`` (the v1 routed linear).

``routed_linear_n2(x, W_stacked, split_point)`` has the v1 signature and
semantics (experiments/routed_linear_n2.py:118-153) and runs the same sm_100a
routed GEMM as :func:`parallel_serve_b200.routed_gemm.routed_gemm`.
"""
from __future__ import annotations

import torch

from .routed_gemm import routed_gemm

__all__ = ["routed_linear_n2", "reference_routed_linear"]


def routed_linear_n2(x: torch.Tensor, W_stacked: torch.Tensor, split_point: int) -> torch.Tensor:
    """out[:sp] = x[:sp] @ W[0]; out[sp:] = x[sp:] @ W[1] (one launch)."""
    return routed_gemm(x, W_stacked, split_point)


def reference_routed_linear(x: torch.Tensor, W_stacked: torch.Tensor, split_point: int) -> torch.Tensor:
    """Ground truth via 2x torch.mm (experiments/routed_linear_n2.py:156-160)."""
    y_a = x[:split_point] @ W_stacked[0]
    y_b = x[split_point:] @ W_stacked[1]
    return torch.cat([y_a, y_b], dim=0)
