"""Route-A DeltaZip: base fp16 weights plus an int4, 2:4-sparse, group-quantised delta.

Route A of the reference serves the RL policy as ``W_base + deq(D)`` through an
external Marlin-24 kernel (docs/deltazip_progress_2026-04-17.md:154-162; only
numbers in the reference). Here:

* :func:`quantize_delta` — 2:4 magnitude pruning of D along K (keep the two
  largest |D| of every 4 consecutive k for each column, lower k first on ties),
  symmetric int4 with one fp16 scale per 128-group along K
  (scale = max|kept| / 7, q = round-half-even(D / scale) clipped to [-7, 7]).
* :func:`pack_delta` — the kernel's HBM format: for every 128-column tile and
  64-k block, 3328 bytes = 128 columns x [16 B: 32 kept int4 values in k order,
  8 B: their 2-bit positions inside each group of 4, 2 B: fp16 scale of the
  block's 128-group]. About 0.19 x the bytes of the fp16 base.
* :func:`deltazip_linear` — one sm_100a launch of ``ps_deltazip_linear``:
  rows before the split use ``W_base``, rows after it ``W_base + deq(D)``.

Packing is offline preprocessing (like loading a checkpoint) done with torch
ops on any device; the linear itself only runs the CUDA kernel.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr

GROUP = 128
TILE_N = 128
BLOCK_K = 64
PACK_BYTES = TILE_N * 16 + TILE_N * 8 + TILE_N * 2

__all__ = ["quantize_delta", "pack_delta", "deltazip_linear", "DeltaZipLinear", "dequantize"]


def quantize_delta(D: torch.Tensor, group: int = GROUP):
    """D [K, N] -> (q int8 [K, N] zero at pruned entries, keep bool [K, N],
    scales float16 [K / group, N])."""
    K, N = D.shape
    if K % group or K % 4:
        raise ValueError(f"K={K} must be a multiple of {group}")
    Dd = D.to(torch.float64)
    mag = Dd.abs().reshape(K // 4, 4, N)
    order = torch.sort(-mag, dim=1, stable=True).indices            # [K/4, 4, N]
    keep = torch.zeros_like(mag, dtype=torch.bool)
    keep.scatter_(1, order[:, :2, :], True)
    keep = keep.reshape(K, N)
    Dk = torch.where(keep, Dd, torch.zeros((), dtype=torch.float64, device=D.device))
    amax = Dk.abs().reshape(K // group, group, N).amax(dim=1)
    scales = torch.where(amax > 0, amax / 7.0, torch.ones_like(amax)).to(torch.float16)
    s = scales.to(torch.float64).repeat_interleave(group, dim=0)
    q = torch.clamp(torch.round(Dk / s), -7, 7).to(torch.int8)
    q = torch.where(keep, q, torch.zeros_like(q))
    return q, keep, scales


def dequantize(q: torch.Tensor, scales: torch.Tensor, group: int = GROUP) -> torch.Tensor:
    """deq(D) = q * scale (float32)."""
    return q.to(torch.float32) * scales.to(torch.float32).repeat_interleave(group, dim=0)


def pack_delta(q: torch.Tensor, keep: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """(q, keep, scales) -> packed uint8 [ceil(N/128), K/64, 3328] (see module doc)."""
    K, N = q.shape
    dev = q.device
    nt = (N + TILE_N - 1) // TILE_N
    Np = nt * TILE_N
    if Np != N:
        pad = Np - N
        q = torch.cat([q, torch.zeros(K, pad, dtype=q.dtype, device=dev)], dim=1)
        keep = torch.cat([keep, torch.zeros(K, pad, dtype=torch.bool, device=dev)], dim=1)
        # padded columns: keep the first two positions of each group (value 0)
        keep.view(K // 4, 4, Np)[:, :2, N:] = True
        scales = torch.cat([scales, torch.ones(K // GROUP, pad, dtype=scales.dtype, device=dev)], 1)
    KB = K // BLOCK_K
    # kept entries of every group of 4, in increasing k: positions and values
    kg = keep.reshape(K // 4, 4, Np)
    pos = torch.sort(torch.where(kg, torch.arange(4, device=dev)[None, :, None],
                                 torch.full((), 9, device=dev)), dim=1).values[:, :2, :]  # [K/4,2,Np]
    vals = torch.gather(q.reshape(K // 4, 4, Np).to(torch.int32), 1, pos)               # [K/4,2,Np]
    # per (column, 64-k block): 32 kept values (16 groups x 2)
    pos = pos.reshape(KB, 32, Np).permute(2, 0, 1)        # [Np, KB, 32]
    vals = vals.reshape(KB, 32, Np).permute(2, 0, 1)
    nib = (vals & 0xF).to(torch.uint8)                    # two's complement nibbles
    vbytes = nib[..., 0::2] | (nib[..., 1::2] << 4)       # [Np, KB, 16]
    p = pos.to(torch.int64)
    m = torch.zeros(Np, KB, 8, dtype=torch.int64, device=dev)
    for i in range(4):                                    # 4 positions per byte
        m |= p[..., i::4] << (2 * i)
    mbytes = m.to(torch.uint8)                            # [Np, KB, 8]
    sc = scales.reshape(K // GROUP, Np).repeat_interleave(GROUP // BLOCK_K, dim=0)  # [KB, Np]
    sbytes = sc.t().contiguous().view(torch.uint8).reshape(Np, KB, 2)
    out = torch.empty(nt, KB, PACK_BYTES, dtype=torch.uint8, device=dev)
    vb = vbytes.reshape(nt, TILE_N, KB, 16).permute(0, 2, 1, 3).reshape(nt, KB, TILE_N * 16)
    mb = mbytes.reshape(nt, TILE_N, KB, 8).permute(0, 2, 1, 3).reshape(nt, KB, TILE_N * 8)
    sb = sbytes.reshape(nt, TILE_N, KB, 2).permute(0, 2, 1, 3).reshape(nt, KB, TILE_N * 2)
    out[:, :, :TILE_N * 16] = vb
    out[:, :, TILE_N * 16:TILE_N * 24] = mb
    out[:, :, TILE_N * 24:] = sb
    return out


def _workspace(device, M, N):
    idx = torch.device(device).index or 0
    return _lib.workspace(device, lib.ps_deltazip_workspace_bytes(M, N, idx), "deltazip")


def deltazip_linear(x: torch.Tensor, W_base: torch.Tensor, packed: torch.Tensor,
                    split_point: int | None = None, *, counts: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """y[:sp] = x[:sp] @ W_base; y[sp:] = x[sp:] @ (W_base + deq(D)).

    ``split_point=None`` with no ``counts`` means every row is a policy row
    (Y = X @ W_base + X @ deq(D)).
    """
    if not (x.is_cuda and W_base.is_cuda and packed.is_cuda):
        raise ValueError("inputs must be on CUDA")
    if x.dtype != W_base.dtype or x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("x and W_base must both be float16 or both bfloat16")
    M, K = x.shape
    K2, N = W_base.shape
    if K != K2:
        raise ValueError(f"K mismatch: x has K={K}, W_base has K={K2}")
    if packed.numel() != lib.ps_deltazip_packed_bytes(K, N):
        raise ValueError("packed delta does not match W_base's shape")
    sp = 0 if split_point is None else int(split_point)
    x = x.contiguous()
    y = torch.empty(M, N, dtype=x.dtype, device=x.device) if out is None else out
    ws = _workspace(x.device, M, N)
    cp = None
    if counts is not None:
        if counts.dtype != torch.int32 or not counts.is_cuda:
            raise TypeError("counts must be a CUDA int32 tensor")
        cp = counts.data_ptr()
    check(lib.ps_deltazip_linear(ptr(x), ptr(W_base), ptr(packed), ptr(y), M, K, N, sp, cp,
                                 _lib.dtype_code(x.dtype), ptr(ws), ws.numel(),
                                 ptr(_lib.status_tensor(x.device)), _lib.stream_handle(x.device)),
          "ps_deltazip_linear")
    return y


class DeltaZipLinear(torch.nn.Module):
    """A base weight ``[K, N]`` plus the packed delta of one policy model."""

    def __init__(self, W_base: torch.Tensor, D: torch.Tensor | None = None,
                 packed: torch.Tensor | None = None):
        super().__init__()
        self.W_base = W_base.contiguous()
        if packed is None:
            q, keep, scales = quantize_delta(D)
            packed = pack_delta(q, keep, scales)
        self.packed = packed.to(W_base.device).contiguous()

    def forward(self, x, split_point: int | None = None, *, counts=None):
        return deltazip_linear(x, self.W_base, self.packed, split_point, counts=counts)
