"""GPU parity of the Route-A DeltaZip linear against the dense dequantised
oracle Y = X @ W_base + X @ deq(D), on the Llama-7B projection shapes with
1-64 tokens (W_base ~ N(0, 0.02), D ~ N(0, 0.002), 2:4 pruned, int4, fp16
scales per 128-group along K), plus the routed form where base-model rows
use W_base alone."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _setup(K, N, seed):
    from parallel_serve_b200 import deltazip as dzp
    Wb = cpu_randn((K, N), seed, 0.02)
    g = torch.Generator().manual_seed(seed + 1)
    D = torch.randn(K, N, generator=g, dtype=torch.float64) * 0.002
    q, keep, scales = dzp.quantize_delta(D)
    packed = dzp.pack_delta(q, keep, scales)
    deq = q.double().numpy() * np.repeat(scales.double().numpy(), 128, axis=0)
    return Wb, packed, deq


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 11008), (11008, 4096)])
def test_deltazip_policy_rows(K, N):
    from parallel_serve_b200 import deltazip_linear
    Wb, packed, deq = _setup(K, N, 1)
    Wd, pd = Wb.cuda(), packed.cuda()
    Wn = to_np(Wb)
    for M in (1, 2, 4, 8, 16, 32, 64):
        x = cpu_randn((M, K), 100 + M)
        y = deltazip_linear(x.cuda(), Wd, pd)
        xn = to_np(x)
        ref = xn @ Wn + xn @ deq
        assert rel_err(to_np(y), ref) < TOL, (K, N, M)


@pytest.mark.parametrize("M,c0", [(64, 32), (40, 8), (20, 20), (17, 0), (96, 48)])
def test_deltazip_routed_base_and_policy(M, c0):
    from parallel_serve_b200 import deltazip_linear
    K, N = 4096, 4096
    Wb, packed, deq = _setup(K, N, 2)
    x = cpu_randn((M, K), 7)
    y = deltazip_linear(x.cuda(), Wb.cuda(), packed.cuda(), c0)
    xn, Wn = to_np(x), to_np(Wb)
    ref = np.concatenate([xn[:c0] @ Wn, xn[c0:] @ (Wn + deq)])
    assert rel_err(to_np(y), ref) < TOL


def test_deltazip_device_counts():
    from parallel_serve_b200 import deltazip_linear
    K, N, M = 1024, 768, 24
    Wb, packed, deq = _setup(K, N, 3)
    x = cpu_randn((M, K), 9)
    for c0 in (0, 10, 24):
        counts = torch.tensor([c0, M - c0], dtype=torch.int32, device="cuda")
        y = deltazip_linear(x.cuda(), Wb.cuda(), packed.cuda(), counts=counts)
        xn, Wn = to_np(x), to_np(Wb)
        ref = np.concatenate([xn[:c0] @ Wn, xn[c0:] @ (Wn + deq)])
        assert rel_err(to_np(y), ref) < TOL, c0


def test_deltazip_bf16_dense_path():
    """bf16 runs the dense-expansion delta path (fp16 runs tcgen05.mma.sp)."""
    from parallel_serve_b200 import deltazip_linear
    K, N, M, c0 = 4096, 4096, 24, 8
    Wb, packed, deq = _setup(K, N, 5)
    Wb16 = Wb.to(torch.bfloat16)
    x = cpu_randn((M, K), 11, dtype=torch.bfloat16)
    y = deltazip_linear(x.cuda(), Wb16.cuda(), packed.cuda(), c0)
    xn, Wn = to_np(x), to_np(Wb16)
    ref = np.concatenate([xn[:c0] @ Wn, xn[c0:] @ (Wn + deq)])
    assert rel_err(to_np(y), ref) < 2e-2
