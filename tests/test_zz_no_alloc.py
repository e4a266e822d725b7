"""The routed GEMM entry point that allocates nothing (ps_routed_gemm_noalloc).

It exists for callers that cannot give the library device memory: a serving
runtime whose pool owns all of the GPU's memory, a plugin host that forbids
allocation while it executes, a decode loop that cannot take the
synchronisation cudaMalloc may cause. Its scratch is a fixed array inside the
library, so this test checks, through the C ABI, that two calls in a row (the
second one reusing whatever the first left in that array) give the same
result as the regular ps_routed_gemm with a caller-provided workspace and as
the fp64 oracle, within the tolerance the other GPU tests use, and that a problem too big for the
array is refused with PS_ERR_SCRATCH_LIMIT. This file sorts last so a run
that stops at the first failure has run every other test before it.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _noalloc(x, W, y, M, K, N, split, counts=None, epilogue=0):
    from parallel_serve_b200 import _lib
    return _lib.lib.ps_routed_gemm_noalloc(
        _lib.ptr(x), _lib.ptr(W), _lib.ptr(y), M, K, N, split, _lib.ptr(counts), None, None,
        epilogue, _lib.dtype_code(x.dtype), _lib.ptr(_lib.status_tensor(x.device)),
        _lib.stream_handle(x.device))


def _regular(x, W, M, K, N, split, counts=None, epilogue=0):
    from parallel_serve_b200 import _lib
    ncols = N // 2 if epilogue else N
    y = torch.empty(M, ncols, dtype=x.dtype, device=x.device)
    nbytes = _lib.lib.ps_routed_gemm_workspace_bytes(M, N, epilogue, x.device.index or 0)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    rc = _lib.lib.ps_routed_gemm(
        _lib.ptr(x), _lib.ptr(W), _lib.ptr(y), M, K, N, split, _lib.ptr(counts), None, None,
        epilogue, _lib.dtype_code(x.dtype), _lib.ptr(ws), ws.numel(),
        _lib.ptr(_lib.status_tensor(x.device)), _lib.stream_handle(x.device))
    assert rc == _lib.PS_OK
    return y


def _oracle(x, W, M, split, counts, epilogue):
    """fp64 oracle of the routed GEMM (and SwiGLU) on the same fp16 inputs."""
    import oracle
    c0 = int(counts[0]) if counts is not None else split
    y = oracle.routed_gemm(to_np(x), to_np(W), c0)
    return oracle.swiglu(y) if epilogue else y


def _rel_beyond_fp16(out, ref) -> float:
    """max|err| / mean|ref| over the error beyond half an fp16 ulp of each
    reference value: silu(gate) * up is heavy-tailed (max / mean about 30),
    so the rounding of its largest fp16 outputs alone comes near 1e-2."""
    half_ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64) / 2
    excess = np.maximum(np.abs(out - ref) - half_ulp, 0.0)
    return float(excess.max() / (np.abs(ref).mean() + 1e-9))


@pytest.mark.parametrize("M,K,N,split,dev_counts,epi", [
    # a decode QKV projection with a host split
    (64, 4096, 12288, 24, False, 0),
    # a SwiGLU gate_up over a device-side split
    (48, 4096, 2 * 2752, 40, True, 1),
    # above 96 rows the partial tiles no longer fit beside a full grid, so the
    # call runs fewer CTAs (145 at 112 rows, 127 at 128): another stream-K cut,
    # and partial slots up to the end of the array
    (128, 4096, 4096, 70, True, 0),
    (112, 4096, 2 * 2752, 50, False, 1),
])
def test_noalloc_matches_regular_and_oracle_on_two_calls_in_a_row(M, K, N, split, dev_counts,
                                                                    epi):
    """Two calls in a row (the second one reuses whatever the first left in the
    shared array) each match ps_routed_gemm with a caller workspace and the fp64
    oracle, with a clean status word."""
    from parallel_serve_b200 import _lib
    dev = torch.device("cuda", 0)
    x = cpu_randn((M, K), 100 + M).to(dev)
    W = cpu_randn((2, K, N), 200 + M, 0.02).to(dev)
    counts = (torch.tensor([split, M - split], dtype=torch.int32, device=dev)
              if dev_counts else None)
    ncols = N // 2 if epi else N
    ref = _regular(x, W, M, K, N, split, counts, epi)
    want = _oracle(x, W, M, split, None if counts is None else counts.cpu(), epi)
    _lib.read_status(dev)   # start from a clear status word
    for call in range(2):
        y = torch.full((M, ncols), float("nan"), dtype=torch.float16, device=dev)
        rc = _noalloc(x, W, y, M, K, N, split, counts, epi)
        assert rc == _lib.PS_OK, _lib.lib.ps_error_string(rc).decode()
        torch.cuda.synchronize()
        assert _lib.read_status(dev) == 0, call
        assert torch.isfinite(y).all(), call
        out = to_np(y)
        assert rel_err(out, to_np(ref)) < TOL, call
        metric = _rel_beyond_fp16 if epi else rel_err
        assert metric(out, want) < TOL, call


def test_noalloc_rejects_problems_beyond_its_scratch():
    from parallel_serve_b200 import _lib
    dev = torch.device("cuda", 0)
    x = torch.zeros(16, 64, dtype=torch.float16, device=dev)
    W = torch.zeros(2, 64, 64, dtype=torch.float16, device=dev)
    y = torch.zeros(16, 64, dtype=torch.float16, device=dev)
    # 512 weight tiles x 33 token tiles > 16384 tiles: refused on the host,
    # before any launch, so the undersized buffers are never touched.
    rc = _noalloc(x, W, y, 4096, 64, 65536, 2048)
    assert rc == _lib.PS_ERR_SCRATCH_LIMIT
    assert "scratch" in _lib.lib.ps_error_string(rc).decode()
