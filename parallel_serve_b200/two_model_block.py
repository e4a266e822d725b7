"""Drop-in for ``experiments/two_model_block.py`` on parallel-serve kernels.

Same classes, constructor arguments, weight attributes and forward signatures
as the reference:

  * ``TransformerBlock(H, FF, n_heads, device, dtype)`` — one model's layer
    (experiments/two_model_block.py:42-74), weights ``W_qkv [H,3H]``, ``W_o``,
    ``W_gu [H,2FF]``, ``W_d [FF,H]``, ``ln1``/``ln2 [H]``, ``forward(x)``.
  * ``TwoModelBlockFused(block_a, block_b)`` — stacked weights, ``forward(x_stk)``
    with ``x_stk [2, M, H]`` (experiments/two_model_block.py:77-120).
  * ``TwoModelBlockBMM(block_a, block_b)`` — ``forward(x_cat, split)``, balanced
    split only, as in the reference (experiments/two_model_block.py:123-195).

Every GEMM is the sm_100a routed GEMM, attention is the segment-attention
kernel, norms / SwiGLU / residuals are the fused kernels of
:mod:`parallel_serve_b200.layers`. The serial ``TransformerBlock`` runs the
same kernels with every row routed to its single weight set, which is the
"serial two-model decode of the same kernels" baseline.
"""
from __future__ import annotations

import torch

from .layers import block_forward

H, N_HEADS, HEAD_DIM, FF = 4096, 32, 128, 11008
dtype = torch.float16

__all__ = ["TransformerBlock", "TwoModelBlockFused", "TwoModelBlockBMM", "H", "N_HEADS",
           "HEAD_DIM", "FF"]


class TransformerBlock(torch.nn.Module):
    """Single-model LLaMA-like decoder block (experiments/two_model_block.py:42-74)."""

    def __init__(self, H, FF, n_heads, device, dtype):
        super().__init__()
        self.H = H
        self.FF = FF
        self.n_heads = n_heads
        self.head_dim = H // n_heads
        self.W_qkv = torch.randn(H, 3 * H, device=device, dtype=dtype) * 0.02
        self.W_o = torch.randn(H, H, device=device, dtype=dtype) * 0.02
        self.W_gu = torch.randn(H, 2 * FF, device=device, dtype=dtype) * 0.02
        self.W_d = torch.randn(FF, H, device=device, dtype=dtype) * 0.02
        self.ln1 = torch.randn(H, device=device, dtype=dtype) * 0.01 + 1.0
        self.ln2 = torch.randn(H, device=device, dtype=dtype) * 0.01 + 1.0

    def forward(self, x):
        M = x.shape[0]
        return block_forward(x.contiguous(), self.W_qkv.contiguous(), self.W_o.contiguous(),
                             self.W_gu.contiguous(), self.W_d.contiguous(),
                             self.ln1.contiguous(), self.ln2.contiguous(), self.n_heads,
                             split_point=M)


class TwoModelBlockFused(torch.nn.Module):
    """Two-model block over a stacked [2, M, H] input (experiments/two_model_block.py:77-120)."""

    def __init__(self, block_a: TransformerBlock, block_b: TransformerBlock):
        super().__init__()
        self.H = block_a.H
        self.FF = block_a.FF
        self.n_heads = block_a.n_heads
        self.head_dim = block_a.head_dim
        self.W_qkv = torch.stack([block_a.W_qkv, block_b.W_qkv], dim=0).contiguous()
        self.W_o = torch.stack([block_a.W_o, block_b.W_o], dim=0).contiguous()
        self.W_gu = torch.stack([block_a.W_gu, block_b.W_gu], dim=0).contiguous()
        self.W_d = torch.stack([block_a.W_d, block_b.W_d], dim=0).contiguous()
        self.ln1 = torch.stack([block_a.ln1, block_b.ln1], dim=0).contiguous()
        self.ln2 = torch.stack([block_a.ln2, block_b.ln2], dim=0).contiguous()

    def forward(self, x_stk):
        """x_stk: [2, M_each, H] - pre-stacked input for both models"""
        two, M, Hx = x_stk.shape
        if two != 2 or Hx != self.H:
            raise ValueError(f"x_stk must be [2, M, {self.H}], got {tuple(x_stk.shape)}")
        y = block_forward(x_stk.reshape(2 * M, Hx).contiguous(), self.W_qkv, self.W_o, self.W_gu,
                          self.W_d, self.ln1, self.ln2, self.n_heads, split_point=M)
        return y.view(2, M, Hx)


class TwoModelBlockBMM(torch.nn.Module):
    """Two-model block over a flat [total, H] input (experiments/two_model_block.py:123-195)."""

    def __init__(self, block_a: TransformerBlock, block_b: TransformerBlock):
        super().__init__()
        self.H = block_a.H
        self.FF = block_a.FF
        self.n_heads = block_a.n_heads
        self.head_dim = block_a.head_dim
        self.W_qkv = torch.stack([block_a.W_qkv, block_b.W_qkv], dim=0).contiguous()
        self.W_o = torch.stack([block_a.W_o, block_b.W_o], dim=0).contiguous()
        self.W_gu = torch.stack([block_a.W_gu, block_b.W_gu], dim=0).contiguous()
        self.W_d = torch.stack([block_a.W_d, block_b.W_d], dim=0).contiguous()
        self.ln1 = torch.stack([block_a.ln1, block_b.ln1], dim=0).contiguous()
        self.ln2 = torch.stack([block_a.ln2, block_b.ln2], dim=0).contiguous()
        self.block_a = block_a
        self.block_b = block_b

    def forward(self, x_cat, split):
        """x_cat: [total, H], split: first split rows are model A, rest model B."""
        M_total = x_cat.shape[0]
        if split != M_total - split:
            raise ValueError("Balanced split only for this block (use TwoModelBlockRouted)")
        return block_forward(x_cat.contiguous(), self.W_qkv, self.W_o, self.W_gu, self.W_d,
                             self.ln1, self.ln2, self.n_heads, split_point=split)
