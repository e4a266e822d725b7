"""Drop-in for ``kernel/src/two_model_block_routed.py``.

``TwoModelBlockRouted(H, FF, n_heads, device="cuda", dtype=torch.bfloat16)``
with stacked ``nn.Parameter(requires_grad=False)`` weights ``W_qkv [2,H,3H]``,
``W_o [2,H,H]``, ``W_gu [2,H,2FF]``, ``W_d [2,FF,H]``, ``ln1``/``ln2 [2,H]``
(ones), and ``forward(x [M,H], split_point) -> [M,H]``
(kernel/src/two_model_block_routed.py:40-153). Weights may be re-pointed with
``b.W_qkv.data = ...`` as the reference benchmarks do
(kernel/benchmarks/bench_full_stack.py:116-131).

``forward`` also accepts ``counts=`` (device int32[2]) instead of a host split,
so one captured CUDA graph serves every split.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .layers import block_forward

__all__ = ["TwoModelBlockRouted"]


class TwoModelBlockRouted(nn.Module):
    """One transformer block fusing two models via the routed GEMM."""

    def __init__(self, H: int, FF: int, n_heads: int, device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.H = H
        self.FF = FF
        self.n_heads = n_heads
        if H % n_heads != 0:
            raise ValueError("H must be a multiple of n_heads")
        self.head_dim = H // n_heads
        self.W_qkv = nn.Parameter(torch.randn(2, H, 3 * H, device=device, dtype=dtype) * 0.02,
                                  requires_grad=False)
        self.W_o = nn.Parameter(torch.randn(2, H, H, device=device, dtype=dtype) * 0.02,
                                requires_grad=False)
        self.W_gu = nn.Parameter(torch.randn(2, H, 2 * FF, device=device, dtype=dtype) * 0.02,
                                 requires_grad=False)
        self.W_d = nn.Parameter(torch.randn(2, FF, H, device=device, dtype=dtype) * 0.02,
                                requires_grad=False)
        self.ln1 = nn.Parameter(torch.ones(2, H, device=device, dtype=dtype), requires_grad=False)
        self.ln2 = nn.Parameter(torch.ones(2, H, device=device, dtype=dtype), requires_grad=False)

    def forward(self, x: torch.Tensor, split_point: int | None = None, *,
                counts: torch.Tensor | None = None) -> torch.Tensor:
        """x: [M_total, H]; rows [0:split) use model A weights, the rest model B."""
        if x.dim() != 2 or x.shape[1] != self.H:
            raise ValueError(f"x must be [M, {self.H}], got {tuple(x.shape)}")
        M_total = x.shape[0]
        if counts is None:
            if split_point is None or not (0 <= split_point <= M_total):
                raise ValueError(f"split_point={split_point} out of range [0, {M_total}]")
        return block_forward(x.contiguous(), self.W_qkv.data.contiguous(),
                             self.W_o.data.contiguous(), self.W_gu.data.contiguous(),
                             self.W_d.data.contiguous(), self.ln1.data.contiguous(),
                             self.ln2.data.contiguous(), self.n_heads,
                             split_point=0 if split_point is None else split_point, counts=counts)
