"""Functional two-model decoder-layer forwards built only on parallel-serve kernels.

``block_forward`` is the layer of experiments/two_model_block.py:54-74 /
kernel/src/two_model_block_routed.py:122-153 in routed order:

    rms_norm -> QKV -> attention -> O (+ residual) -> rms_norm
             -> gate_up with fused SwiGLU -> down (+ residual)

Seven launches per layer (the reference issues about 15,
kernel/src/two_model_block_routed.py:26-28): the residual adds live in the
O / down GEMM epilogues and silu(gate) * up lives in the gate_up epilogue.
"""
from __future__ import annotations

import torch

from . import _lib, ops


def block_forward(x: torch.Tensor, W_qkv: torch.Tensor, W_o: torch.Tensor, W_gu: torch.Tensor,
                  W_d: torch.Tensor, ln1: torch.Tensor, ln2: torch.Tensor, n_heads: int, *,
                  split_point: int = 0, counts: torch.Tensor | None = None,
                  eps: float | None = None) -> torch.Tensor:
    """No-KV layer with the reference semantics: each model's tokens attend to
    their own segment of the batch (kernel/src/two_model_block_routed.py:100-120).

    ``W_*`` are stacked [2, K, N] (or single [K, N] with split_point == M),
    ``ln*`` are [2, H] (or [1, H]/[H] with split_point == M).
    """
    M, H = x.shape
    FF = W_d.shape[-2]
    if ln1.dim() == 1:
        ln1 = ln1.view(1, -1)
    if ln2.dim() == 1:
        ln2 = ln2.view(1, -1)
    kw = dict(split_point=split_point, counts=counts)
    h = ops.rmsnorm_routed(x, ln1, eps=eps, **kw)
    qkv = torch.empty(M, 3 * H, dtype=x.dtype, device=x.device)
    ops.routed_gemm_raw(h, W_qkv, qkv, **kw)
    attn = ops.segment_attention(qkv, n_heads, **kw)
    x1 = torch.empty_like(x)
    ops.routed_gemm_raw(attn, W_o, x1, residual=x, **kw)
    h2 = ops.rmsnorm_routed(x1, ln2, eps=eps, **kw)
    a = torch.empty(M, FF, dtype=x.dtype, device=x.device)
    ops.routed_gemm_raw(h2, W_gu, a, epilogue=_lib.PS_EPI_SWIGLU, **kw)
    y = torch.empty_like(x)
    ops.routed_gemm_raw(a, W_d, y, residual=x1, **kw)
    return y
