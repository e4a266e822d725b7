"""Kernels on two GPUs from ONE process.

A kernel's dynamic shared-memory opt-in (cudaFuncSetAttribute) belongs to one
device's context, so the first launch on a second device must raise its own
limit (ps_host.cu `allow_dynamic_smem`, keyed by function, device and size).
The routed GEMM (up to 227 KB of shared memory per CTA) and both decode
attention kernels (per-chunk and balanced split) run on cuda:0, cuda:1, then
cuda:0 again, each checked against the oracle, with a clean status word on
both devices.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

TOL = 1e-2


def test_routed_gemm_on_two_devices_in_one_process():
    import oracle
    from parallel_serve_b200 import _lib, routed_gemm
    M, K, N, split = 64, 4096, 1024, 24
    x = cpu_randn((M, K), 0)
    W = cpu_randn((2, K, N), 1, 0.02)
    ref = oracle.routed_gemm(to_np(x), to_np(W), split)
    for d in (0, 1, 0):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            y = routed_gemm(x.to(dev), W.to(dev), split)
            torch.cuda.synchronize(dev)
            assert _lib.read_status(dev) == 0, d
        assert rel_err(to_np(y), ref) < TOL, d


@pytest.mark.parametrize("chunk", [0, -1])   # per-chunk kernel / balanced split
def test_decode_attention_on_two_devices_in_one_process(chunk):
    import oracle
    from parallel_serve_b200 import _lib, ops
    nh, L_cap, slots = 2, 600, (3, 2)
    lens = [600, 1, 257, 64, 333]
    M, c0 = sum(slots), slots[0]
    k = [cpu_randn((s, nh, L_cap, 128), 40 + i) for i, s in enumerate(slots)]
    v = [cpu_randn((s, nh, L_cap, 128), 50 + i) for i, s in enumerate(slots)]
    q = cpu_randn((M, nh * 128), 60)
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32)
    Kc = np.stack([to_np(k[0][j]) if j < c0 else to_np(k[1][j - c0]) for j in range(M)])
    Vc = np.stack([to_np(v[0][j]) if j < c0 else to_np(v[1][j - c0]) for j in range(M)])
    ref = oracle.decode_attention(to_np(q).reshape(M, nh, 128), Kc, Vc, np.array(lens))
    for d in (0, 1, 0):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            out = ops.decode_attention(q.to(dev), tuple(t.to(dev) for t in k),
                                       tuple(t.to(dev) for t in v), pos.to(dev), n_heads=nh,
                                       max_len=L_cap, split_point=c0, chunk=chunk)
            torch.cuda.synchronize(dev)
            assert _lib.read_status(dev) == 0, d
        assert rel_err(to_np(out), ref.reshape(M, -1)) < TOL, d
