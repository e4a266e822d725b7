"""The C-ABI entry points registered as ``torch.ops.parallel_serve.*``.

CPU: every operator is registered with its schema and its fake (meta)
implementation gives the output shapes and dtypes without touching a GPU.
GPU (marked): each operator runs the CUDA kernel and matches the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from conftest import cpu_randn, rel_err, to_np


def test_every_operator_is_registered_with_a_schema():
    import parallel_serve_b200.torch_ops as tops
    for name in tops.OPS:
        op = getattr(torch.ops.parallel_serve, name)
        schema = str(op.default._schema)
        assert schema.startswith(f"parallel_serve::{name}("), schema


def test_fake_implementations_give_output_shapes():
    import parallel_serve_b200  # noqa: F401
    P = torch.ops.parallel_serve
    with FakeTensorMode():
        f16 = dict(dtype=torch.float16, device="cuda")
        i32 = dict(dtype=torch.int32, device="cuda")
        x, W = torch.empty(48, 512, **f16), torch.empty(2, 512, 384, **f16)
        cnt, ids = torch.empty(2, **i32), torch.empty(48, **i32)
        for y in (P.routed_gemm(x, W, 20), P.routed_gemm_counts(x, W, cnt),
                  P.routed_gemm_model_id(x, W, ids)):
            assert y.shape == (48, 384) and y.dtype == torch.float16
        perm, counts = P.route_partition(ids)
        assert perm.shape == (48,) and counts.shape == (2,) and perm.dtype == torch.int32
        assert P.rmsnorm_routed(x, torch.empty(2, 512, **f16), cnt, 1e-5).shape == (48, 512)
        q = torch.empty(6, 2 * 128, **f16)
        kv = torch.empty(3, 2, 64, 128, **f16)
        out = P.decode_attention(q, kv, kv, kv, kv, torch.empty(6, **i32), cnt, 2, 64)
        assert out.shape == (6, 256)
        packed = torch.empty(1, dtype=torch.uint8, device="cuda")
        assert P.deltazip_linear(x, torch.empty(512, 384, **f16), packed, 8).shape == (48, 384)


@pytest.mark.gpu
def test_operators_run_the_kernels_and_match_the_oracle():
    import oracle
    import parallel_serve_b200  # noqa: F401
    P = torch.ops.parallel_serve
    dev = torch.device("cuda", 0)
    M, K, N, c0 = 40, 1024, 768, 17
    x = cpu_randn((M, K), 1)
    W = cpu_randn((2, K, N), 2, 0.02)
    ref = oracle.routed_gemm(to_np(x), to_np(W), c0)
    xd, Wd = x.to(dev), W.to(dev)
    cnt = torch.tensor([c0, M - c0], dtype=torch.int32, device=dev)
    assert rel_err(to_np(P.routed_gemm(xd, Wd, c0)), ref) < 1e-2
    assert rel_err(to_np(P.routed_gemm_counts(xd, Wd, cnt)), ref) < 1e-2
    ids = torch.tensor([0] * c0 + [1] * (M - c0), dtype=torch.int32)
    order = torch.randperm(M, generator=torch.Generator().manual_seed(3))
    y = P.routed_gemm_model_id(xd[order.to(dev)], Wd, ids[order].to(dev))
    assert rel_err(to_np(y), ref[order.numpy()]) < 1e-2
    perm, counts = P.route_partition(ids[order].to(dev))
    assert np.array_equal(perm.cpu().numpy(), np.argsort(ids[order].numpy(), kind="stable"))
    assert counts.cpu().tolist() == [c0, M - c0]
    w = 1 + cpu_randn((2, K), 4, 0.1)
    h = P.rmsnorm_routed(xd, w.to(dev), cnt, 1e-5)
    want = np.concatenate([oracle.rms_norm(to_np(x)[:c0], to_np(w)[0], 1e-5),
                           oracle.rms_norm(to_np(x)[c0:], to_np(w)[1], 1e-5)])
    assert rel_err(to_np(h), want) < 1e-2
    from parallel_serve_b200 import _lib
    assert _lib.read_status(dev) == 0
