"""Failure detection on the device: a bounded wait that runs out.

Every wait inside the library's kernels is bounded by wall time; when one runs
out the kernel ORs PS_ERR_TIMEOUT into the status word and returns, so the
context stays usable and the host learns of the failure by reading the status
after a synchronize. Here the wait is made to run out without any fault: the
NVLink all-reduce is called as rank 0 of a world of 2 on ONE GPU, with both
"ranks'" symmetric regions in this GPU's own memory and nothing ever playing
rank 1, so rank 1's arrival flag is never set. (No second kernel is launched
to play rank 1: kernels that wait on one another must never share a GPU.)
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu


def _allreduce(peers, rank, world, slot_bytes, count, out, residual, epochs, algo):
    from parallel_serve_b200 import _lib
    dev = out.device
    arr = (ctypes.c_void_p * world)(*[p.data_ptr() for p in peers])
    return _lib.lib.ps_allreduce_sum(arr, rank, world, 0, slot_bytes, count, out.data_ptr(),
                                     None if residual is None else residual.data_ptr(),
                                     epochs.data_ptr(), out.shape[-1], None, algo,
                                     _lib.PS_DTYPE_F16, _lib.ptr(_lib.status_tensor(dev)),
                                     _lib.stream_handle(dev))


@pytest.mark.parametrize("algo", ["one_shot", "two_shot", "two_shot_ll"])
def test_peer_wait_runs_out_sets_timeout_and_context_survives(algo):
    from parallel_serve_b200 import _lib, routed_gemm
    import oracle
    dev = torch.device("cuda", 0)
    code = {"one_shot": _lib.PS_AR_ONE_SHOT, "two_shot": _lib.PS_AR_TWO_SHOT,
            "two_shot_ll": _lib.PS_AR_TWO_SHOT_LL}[algo]
    rows, H = 8, 512                         # count % (2 ranks x 256) == 0: two-shot applies
    count = rows * H
    slot_bytes = (count * 2 + 255) // 256 * 256
    region = _lib.lib.ps_symm_region_bytes(slot_bytes)
    # Both regions live on this GPU; nobody plays rank 1.
    peers = [torch.zeros(region, dtype=torch.uint8, device=dev) for _ in range(2)]
    epochs = torch.zeros(128, dtype=torch.int32, device=dev)
    out = torch.zeros(rows, H, dtype=torch.float16, device=dev)
    _lib.read_status(dev)                    # start from a clear status word

    t0 = time.monotonic()
    rc = _allreduce(peers, 0, 2, slot_bytes, count, out, None, epochs, code)
    assert rc == _lib.PS_OK
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    st = _lib.read_status(dev)
    assert st & _lib.PS_ERR_TIMEOUT, f"status 0x{st:x}"
    # the wait limit is 1 s per wait (two-shot: the first wait already fails)
    assert elapsed < 10.0, elapsed

    # The context is usable: a world-1 all-reduce of a slot adds it to the residual ...
    slot = cpu_randn((rows, H), 3)
    res = cpu_randn((rows, H), 4)
    off = _lib.lib.ps_symm_slot_offset(0, slot_bytes)
    peers[0][off:off + count * 2].copy_(slot.view(torch.uint8).flatten().to(dev))
    out1 = torch.empty(rows, H, dtype=torch.float16, device=dev)
    res_d = res.to(dev)
    rc = _allreduce(peers[:1], 0, 1, slot_bytes, count, out1, res_d, epochs, code)
    assert rc == _lib.PS_OK
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    assert torch.equal(out1.cpu(), (slot.float() + res.float()).half())

    # ... and a routed GEMM still matches the oracle.
    x = cpu_randn((32, 1024), 5)
    W = cpu_randn((2, 1024, 1024), 6, 0.02)
    y = routed_gemm(x.to(dev), W.to(dev), 12)
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    assert rel_err(to_np(y), oracle.routed_gemm(to_np(x), to_np(W), 12)) < 1e-2
    assert np.isfinite(to_np(y)).all()
