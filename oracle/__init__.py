"""CPU oracle for the fused two-model decode path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's algorithm for every function
on the path, each citing the reference file:line it follows. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it,
and only as the reference outputs for comparison / the timed CPU baseline. The product
(``parallel_serve_b200``) never imports it and has no CPU fallback.

Pinning: ``tests/golden/make_golden.py`` imports the reference's own Python
modules (``reference_routed_gemm``, ``TransformerBlock``, ``TwoModelBlockFused``,
``TwoModelBlockRouted`` with its routed GEMM replaced by the reference's own
``reference_routed_gemm``) on CPU and stores their outputs on seeded inputs as
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this oracle
against them. The decode-only parts the reference does not implement (KV
cache, RoPE, decode step, prefill) are restatements of the Llama decode math,
pinned in two ways: the no-KV special case (a cache holding exactly the
segment's keys reproduces the reference's SDPA), and ``tests/test_loader.py``,
which runs transformers' own Llama implementation (the model family the
reference serves) on small random models and checks ``decode_step`` and
``prefill`` against it. The DeltaZip dequantisation stays unpinned (the
reference's Marlin-24 kernel lives in a vLLM fork that is absent).
"""
from .ref_ops import *  # noqa: F401,F403
