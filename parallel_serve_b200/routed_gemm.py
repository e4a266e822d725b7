"""Routed two-model GEMM — drop-in for ``kernel/src/routed_gemm.py``.

``routed_gemm(x, W_stacked, split_point)`` keeps the reference signature and
meaning (kernel/src/routed_gemm.py:152-197): rows ``[0, split_point)`` of ``x``
are multiplied by ``W_stacked[0]``, the rest by ``W_stacked[1]``, one launch,
fp32 accumulation. It runs the sm_100a tcgen05 kernel of libparallel_serve.so
and accepts float16 (the build's decode dtype) or bfloat16 (the reference's).

Additions over the reference:
  * ``model_id=`` per-token ids in any order: the tokens are partitioned on the
    device (stable), gathered, multiplied, and the epilogue scatters rows back
    to the caller's order — no host sync.
  * ``counts=`` a device int32[2] split for rows already in routed order, so a
    CUDA graph captured once serves any split.
"""
from __future__ import annotations

import torch

from . import _lib
from . import ops

__all__ = ["routed_gemm", "reference_routed_gemm"]


def _validate(x: torch.Tensor, W_stacked: torch.Tensor) -> tuple[int, int, int]:
    if not (x.is_cuda and W_stacked.is_cuda):
        raise ValueError("inputs must be on CUDA")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"x dtype={x.dtype}, expected float16 or bfloat16")
    if W_stacked.dtype != x.dtype:
        raise TypeError(f"W dtype={W_stacked.dtype}, expected {x.dtype}")
    if x.dim() != 2:
        raise ValueError(f"x must be 2-D, got shape {tuple(x.shape)}")
    if W_stacked.dim() != 3 or W_stacked.shape[0] != 2:
        raise ValueError(f"W_stacked must be [2, K, N], got {tuple(W_stacked.shape)}")
    M, K = x.shape
    _, K_w, N = W_stacked.shape
    if K != K_w:
        raise ValueError(f"K mismatch: x has K={K}, W has K={K_w}")
    if K % 8 or N % 8:
        raise ValueError(f"K and N must be multiples of 8 (got K={K}, N={N})")
    if x.device != W_stacked.device:
        raise ValueError("x and W_stacked must be on the same device")
    return M, K, N


def routed_gemm(x: torch.Tensor, W_stacked: torch.Tensor, split_point: int | None = None, *,
                model_id: torch.Tensor | None = None, counts: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """y[:sp] = x[:sp] @ W[0], y[sp:] = x[sp:] @ W[1].

    Exactly one of ``split_point`` (host int), ``counts`` (device int32[2], rows
    already grouped model 0 first) or ``model_id`` (device int32[M], any order)
    selects the routing.
    """
    M, K, N = _validate(x, W_stacked)
    given = sum(v is not None for v in (split_point, model_id, counts))
    if given != 1:
        raise ValueError("pass exactly one of split_point, counts or model_id")
    if split_point is not None and not (0 <= split_point <= M):
        raise ValueError(f"split_point={split_point} out of range [0, {M}]")
    x = x.contiguous()
    W_stacked = W_stacked.contiguous()
    y = torch.empty((M, N), dtype=x.dtype, device=x.device) if out is None else out
    if model_id is not None:
        if model_id.shape != (M,):
            raise ValueError("model_id must have one entry per row of x")
        perm, cnt = ops.route_partition(model_id.to(torch.int32))
        xp = ops.gather_rows(x, perm)
        return ops.routed_gemm_raw(xp, W_stacked, y, counts=cnt, scatter=perm)
    if counts is not None:
        return ops.routed_gemm_raw(x, W_stacked, y, counts=counts)
    return ops.routed_gemm_raw(x, W_stacked, y, split_point=int(split_point))


def reference_routed_gemm(x: torch.Tensor, W_stacked: torch.Tensor, split_point: int) -> torch.Tensor:
    """Ground truth of the reference (kernel/src/routed_gemm.py:200-204): two torch.mm + cat."""
    y_a = x[:split_point] @ W_stacked[0]
    y_b = x[split_point:] @ W_stacked[1]
    return torch.cat([y_a, y_b], dim=0)
