"""parallel-serve on B200 (sm_100a): the fused two-model decode path.

Two same-architecture models share one GPU (or a tensor-parallel 8xB200 box).
Their weights are stacked as ``W[2, K, N]``; every decode token carries a model
id and every projection runs as one routed GEMM over both models' tokens.

Public API (mirrors the reference's operator modules):
  routed_gemm, reference_routed_gemm             (kernel/src/routed_gemm.py)
  routed_linear_n2, reference_routed_linear      (experiments/routed_linear_n2.py)
  TransformerBlock, TwoModelBlockFused, TwoModelBlockBMM (experiments/two_model_block.py)
  TwoModelBlockRouted                            (kernel/src/two_model_block_routed.py)
  TwoModelDecoder                                (KV-cache decode loop, CUDA graphs,
                                                  contiguous or paged KV)
  deltazip_linear                                (Route-A base + int4 2:4 delta)
  pack_hf_llama, load_two_llama                  (experiments/real_weights_correctness.py:27-51)
  torch.ops.parallel_serve.*                     (the entry points as PyTorch custom operators)
"""
from __future__ import annotations

from . import _lib, ops  # noqa: F401  (loads libparallel_serve.so or raises)
from .routed_gemm import reference_routed_gemm, routed_gemm
from .routed_linear_n2 import reference_routed_linear, routed_linear_n2
from .two_model_block import TransformerBlock, TwoModelBlockBMM, TwoModelBlockFused
from .two_model_block_routed import TwoModelBlockRouted
from .deltazip import DeltaZipLinear, deltazip_linear
from .decoder import DecoderConfig, TwoModelDecoder
from .loader import decoder_config_from_hf, load_two_llama, pack_hf_llama
from . import torch_ops  # noqa: F401  (registers torch.ops.parallel_serve.*)

__all__ = [
    "routed_gemm", "reference_routed_gemm", "routed_linear_n2", "reference_routed_linear",
    "TransformerBlock", "TwoModelBlockFused", "TwoModelBlockBMM", "TwoModelBlockRouted",
    "deltazip_linear", "DeltaZipLinear", "DecoderConfig", "TwoModelDecoder",
    "pack_hf_llama", "load_two_llama", "decoder_config_from_hf",
]
