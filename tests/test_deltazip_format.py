"""DeltaZip packing on CPU: the package's torch quantizer equals the oracle's
numpy quantizer bit for bit, and the packed bytes decode (with the oracle's
independent reader) back to the same int4 values, positions and scales."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from parallel_serve_b200 import deltazip as dzp


@pytest.mark.parametrize("K,N", [(256, 128), (384, 200), (128, 8), (512, 264)])
def test_quantize_matches_oracle_and_roundtrips(K, N):
    g = torch.Generator().manual_seed(K + N)
    D = (torch.randn(K, N, generator=g, dtype=torch.float64) * 0.002).to(torch.float16)
    q, keep, scales = dzp.quantize_delta(D)
    q_ref, keep_ref, s_ref = oracle.deltazip_quantize(D.double().numpy())
    assert np.array_equal(q.numpy(), q_ref)
    assert np.array_equal(keep.numpy(), keep_ref)
    assert np.array_equal(scales.numpy(), s_ref.astype(np.float16))
    # exactly two kept entries in every group of 4 along K
    assert (keep.reshape(K // 4, 4, N).sum(1) == 2).all()
    packed = dzp.pack_delta(q, keep, scales)
    assert packed.numel() == ((N + 127) // 128) * (K // 64) * 3328
    q_back, s_back = oracle.deltazip_unpack(packed.numpy(), K, N)
    assert np.array_equal(q_back, q.numpy())
    assert np.array_equal(s_back, scales.numpy())


def test_dequant_is_sparse_and_close_to_delta():
    g = torch.Generator().manual_seed(0)
    D = torch.randn(256, 64, generator=g, dtype=torch.float64) * 0.002
    q, keep, scales = dzp.quantize_delta(D)
    deq = dzp.dequantize(q, scales).double()
    assert ((deq != 0).reshape(64, 4, 64).sum(1) <= 2).all()
    kept = torch.where(keep, D, torch.zeros_like(D))
    # symmetric int4 error <= half a step per entry
    step = scales.double().repeat_interleave(128, 0)
    assert ((deq - kept).abs() <= 0.5 * step + 1e-12).all()
