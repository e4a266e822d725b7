"""The vocab-parallel greedy pick (ps_argmax_tp) on one GPU (world 1: the
exchange runs through this rank's own symmetric region). The multi-rank
exchange is covered by the 2-GPU tensor-parallel tests and by bench.py's
parity gate at every GPU count."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import cpu_randn

pytestmark = pytest.mark.gpu


def test_pick_matches_argmax_scatter_and_length_update():
    from parallel_serve_b200 import _lib
    dev = torch.device("cuda", 0)
    M, V = 37, 4000
    logits = cpu_randn((M, V), 11)
    logits[3, 17] = logits[3, 2000] = 9.0          # tie: the lower index wins
    perm = torch.randperm(M, generator=torch.Generator().manual_seed(2)).to(torch.int32)
    slot_bytes = 256 * 1024
    region = torch.zeros(_lib.lib.ps_symm_region_bytes(slot_bytes), dtype=torch.uint8, device=dev)
    peers = (ctypes.c_void_p * 1)(region.data_ptr())
    epochs = torch.zeros(M, dtype=torch.int32, device=dev)
    nxt = torch.full((M,), -1, dtype=torch.int32, device=dev)
    tok = torch.full((M,), -1, dtype=torch.int32, device=dev)
    seq = torch.arange(M, dtype=torch.int32, device=dev)
    lg, pm = logits.to(dev), perm.to(dev)
    st = _lib.status_tensor(dev)
    _lib.read_status(dev)
    for call in range(2):                       # epochs advance call by call
        rc = _lib.lib.ps_argmax_tp(lg.data_ptr(), pm.data_ptr(), nxt.data_ptr(), tok.data_ptr(),
                                   seq.data_ptr(), M, V, peers, 0, 1, slot_bytes,
                                   epochs.data_ptr(), _lib.PS_DTYPE_F16, st.data_ptr(),
                                   _lib.stream_handle(dev))
        assert rc == _lib.PS_OK
        torch.cuda.synchronize()
        assert _lib.read_status(dev) == 0
        want = np.empty(M, dtype=np.int64)
        want[perm.numpy()] = logits.float().numpy().argmax(axis=1)
        assert np.array_equal(nxt.cpu().numpy(), want)
        assert np.array_equal(tok.cpu().numpy(), want)
        assert np.array_equal(seq.cpu().numpy(), np.arange(M) + call + 1)
        assert epochs.cpu().tolist() == [call + 1] * M
    assert want[perm[3].item()] == 17
