"""``torch.ops.parallel_serve.*``: the C-ABI entry points as PyTorch custom operators.

The reference exposes its routed GEMM as a Python function over a Triton
kernel (kernel/src/routed_gemm.py:152). Here the same entry points are also
registered with the PyTorch dispatcher, each with a schema and a fake (meta)
implementation, so they appear as single operators to the profiler, to
``torch.compile`` graphs that contain them and to TorchScript-style callers:

  parallel_serve::routed_gemm(Tensor x, Tensor W_stacked, int split_point) -> Tensor
  parallel_serve::routed_gemm_counts(Tensor x, Tensor W_stacked, Tensor counts) -> Tensor
  parallel_serve::routed_gemm_model_id(Tensor x, Tensor W_stacked, Tensor model_id) -> Tensor
  parallel_serve::route_partition(Tensor model_id) -> (Tensor perm, Tensor counts)
  parallel_serve::rmsnorm_routed(Tensor x, Tensor w, Tensor counts, float eps) -> Tensor
  parallel_serve::decode_attention(Tensor q, Tensor? k0, Tensor? v0, Tensor? k1, Tensor? v1,
                                   Tensor pos, Tensor counts, int n_heads, int max_len) -> Tensor
  parallel_serve::deltazip_linear(Tensor x, Tensor W_base, Tensor packed, int split_point) -> Tensor

Every CUDA implementation is the same ctypes call into libparallel_serve.so
that the Python API makes (one kernel launch on the current stream, no host
synchronisation); there is no CPU implementation. Importing this module
registers the operators (the package imports it).
"""
from __future__ import annotations

import torch

from . import ops
from .deltazip import deltazip_linear as _deltazip_linear
from .routed_gemm import routed_gemm as _routed_gemm

__all__ = ["OPS"]

OPS = ("routed_gemm", "routed_gemm_counts", "routed_gemm_model_id", "route_partition",
       "rmsnorm_routed", "decode_attention", "deltazip_linear")


@torch.library.custom_op("parallel_serve::routed_gemm", mutates_args=(), device_types="cuda")
def routed_gemm(x: torch.Tensor, W_stacked: torch.Tensor, split_point: int) -> torch.Tensor:
    """y[:split_point] = x[:split_point] @ W[0], the rest @ W[1]."""
    return _routed_gemm(x, W_stacked, split_point)


@routed_gemm.register_fake
def _(x, W_stacked, split_point):
    return x.new_empty(x.shape[0], W_stacked.shape[-1])


@torch.library.custom_op("parallel_serve::routed_gemm_counts", mutates_args=(),
                         device_types="cuda")
def routed_gemm_counts(x: torch.Tensor, W_stacked: torch.Tensor,
                       counts: torch.Tensor) -> torch.Tensor:
    """Rows already grouped model 0 first; the split is read on the device."""
    return _routed_gemm(x, W_stacked, counts=counts)


@routed_gemm_counts.register_fake
def _(x, W_stacked, counts):
    return x.new_empty(x.shape[0], W_stacked.shape[-1])


@torch.library.custom_op("parallel_serve::routed_gemm_model_id", mutates_args=(),
                         device_types="cuda")
def routed_gemm_model_id(x: torch.Tensor, W_stacked: torch.Tensor,
                         model_id: torch.Tensor) -> torch.Tensor:
    """Per-token model ids in any order (partitioned, gathered and scattered back)."""
    return _routed_gemm(x, W_stacked, model_id=model_id)


@routed_gemm_model_id.register_fake
def _(x, W_stacked, model_id):
    return x.new_empty(x.shape[0], W_stacked.shape[-1])


@torch.library.custom_op("parallel_serve::route_partition", mutates_args=(), device_types="cuda")
def route_partition(model_id: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Stable partition by model id: (perm int32 [M], counts int32 [2])."""
    return ops.route_partition(model_id)


@route_partition.register_fake
def _(model_id):
    return (model_id.new_empty(model_id.shape[0], dtype=torch.int32),
            model_id.new_empty(2, dtype=torch.int32))


@torch.library.custom_op("parallel_serve::rmsnorm_routed", mutates_args=(), device_types="cuda")
def rmsnorm_routed(x: torch.Tensor, w: torch.Tensor, counts: torch.Tensor,
                   eps: float) -> torch.Tensor:
    """Per-model RMSNorm of rows in routed order (w is [2, H])."""
    return ops.rmsnorm_routed(x, w, counts=counts, eps=eps)


@rmsnorm_routed.register_fake
def _(x, w, counts, eps):
    return torch.empty_like(x)


@torch.library.custom_op("parallel_serve::decode_attention", mutates_args=(),
                         device_types="cuda")
def decode_attention(q: torch.Tensor, k0: torch.Tensor | None, v0: torch.Tensor | None,
                     k1: torch.Tensor | None, v1: torch.Tensor | None, pos: torch.Tensor,
                     counts: torch.Tensor, n_heads: int, max_len: int) -> torch.Tensor:
    """Two-model decode attention: token j (routed order) attends to positions
    0..pos[j] of its own model's pools [slots, n_heads, L_cap, 128]."""
    return ops.decode_attention(q, (k0, k1), (v0, v1), pos, n_heads=n_heads, max_len=max_len,
                                counts=counts)


@decode_attention.register_fake
def _(q, k0, v0, k1, v1, pos, counts, n_heads, max_len):
    return q.new_empty(q.shape[0], n_heads * 128)


@torch.library.custom_op("parallel_serve::deltazip_linear", mutates_args=(), device_types="cuda")
def deltazip_linear(x: torch.Tensor, W_base: torch.Tensor, packed: torch.Tensor,
                    split_point: int) -> torch.Tensor:
    """y[:split_point] = x @ W_base; the rest x @ (W_base + deq(D))."""
    return _deltazip_linear(x, W_base, packed, split_point)


@deltazip_linear.register_fake
def _(x, W_base, packed, split_point):
    return x.new_empty(x.shape[0], W_base.shape[-1])
