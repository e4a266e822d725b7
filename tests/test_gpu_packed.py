"""Packed weights (ps_pack_weights): the routed GEMM's HBM layout in which each
(model, weight tile, 128-k block) is one contiguous 32 KB block holding the
pipeline stage's swizzled shared-memory image.

* the packed bytes equal a numpy restatement of the layout (tails in K and N,
  SwiGLU's paired gate / up columns);
* a GEMM reading packed weights gives exactly the same result as one reading
  W [2, K, N] through the tensor map, for each epilogue mode;
* a decode step with packed weights equals one without, bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cpu_randn

pytestmark = pytest.mark.gpu


def pack_reference(W: np.ndarray, gated: bool) -> np.ndarray:
    """[nmat, K, N] (16-bit) -> packed bytes: per (m, tile n, k block kb) two
    halves of 128 k rows x 64 columns, 16-byte chunk c of row r stored at
    chunk c ^ (r % 8); zeros past K and N."""
    nmat, K, N = W.shape
    ff = N // 2
    nt = -(-ff // 64) if gated else -(-N // 128)
    KB = -(-K // 128)
    Wp = np.zeros((nmat, KB * 128, N + 128), dtype=W.dtype)
    Wp[:, :K, :N] = W
    out = np.zeros((nmat, nt, KB, 2, 128, 64), dtype=W.dtype)
    for n in range(nt):
        for h in range(2):
            if gated:
                c0 = (ff if h else 0) + 64 * n
                lim = (ff if h else 0) + ff
            else:
                c0 = 128 * n + 64 * h
                lim = N
            cols = np.arange(c0, c0 + 64)
            blk = Wp[:, :, np.minimum(cols, N + 127)]
            blk[:, :, cols >= lim] = 0
            out[:, n, :, h] = blk.reshape(nmat, KB, 128, 64)
    logical = out.reshape(nmat, nt, KB, 2, 128, 8, 8)
    r = np.arange(128)[:, None]
    pc = np.arange(8)[None, :]
    phys = logical[:, :, :, :, r, pc ^ (r & 7), :]
    return phys.reshape(-1).view(np.uint8)


def _pack(W: torch.Tensor, epilogue: int) -> torch.Tensor:
    from parallel_serve_b200 import _lib
    nmat, K, N = W.shape
    nbytes = _lib.lib.ps_packed_weights_bytes(nmat, K, N, epilogue)
    out = torch.full((nbytes,), 0xAB, dtype=torch.uint8, device=W.device)
    rc = _lib.lib.ps_pack_weights(W.data_ptr(), nmat, K, N, epilogue, out.data_ptr(), nbytes,
                                  _lib.stream_handle(W.device))
    assert rc == _lib.PS_OK
    return out


@pytest.mark.parametrize("K,N,gated", [(256, 384, False), (200, 136, False), (384, 2 * 344, True),
                                       (136, 2 * 88, True)])
def test_pack_matches_layout_restatement(K, N, gated):
    from parallel_serve_b200 import _lib
    W = cpu_randn((2, K, N), K + N)
    epi = _lib.PS_EPI_SWIGLU if gated else _lib.PS_EPI_STORE
    got = _pack(W.cuda(), epi).cpu().numpy()
    want = pack_reference(W.numpy(), gated)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("mode", ["store", "swiglu", "qkv"])
def test_gemm_with_packed_weights_is_bit_identical(mode):
    from parallel_serve_b200 import _lib, ops
    dev = torch.device("cuda", 0)
    M, c0, K = 40, 17, 1024
    nh = 2
    N = {"store": 1000, "swiglu": 2 * 704, "qkv": 3 * nh * 128}[mode]
    x = cpu_randn((M, K), 1).to(dev)
    W = cpu_randn((2, K, N), 2, 0.02).to(dev)
    counts = torch.tensor([c0, M - c0], dtype=torch.int32, device=dev)
    code = {"store": _lib.PS_EPI_STORE, "swiglu": _lib.PS_EPI_SWIGLU,
            "qkv": _lib.PS_EPI_QKV_ROPE}[mode]
    packed = _pack(W, _lib.PS_EPI_SWIGLU if mode == "swiglu" else _lib.PS_EPI_STORE)
    outs = []
    for use_packed in (False, True):
        ncol = N // 2 if mode == "swiglu" else (N // 3 if mode == "qkv" else N)
        y = torch.zeros(M, ncol, dtype=torch.float16, device=dev)
        kw = {}
        pools = None
        if mode == "qkv":
            L = 24
            pools = [torch.zeros(n, nh, L, 128, dtype=torch.float16, device=dev)
                     for n in (c0, c0, M - c0, M - c0)]
            cos, sin = ops.rope_tables(L, 128, 10000.0, dev)
            kw = dict(k_pools=(pools[0], pools[2]), v_pools=(pools[1], pools[3]),
                      pos=torch.arange(M, dtype=torch.int32, device=dev) % L, rope_cos=cos,
                      rope_sin=sin, n_heads=nh)
        e = ops.gemm_epilogue(code, **kw)
        e.w_packed = packed.data_ptr() if use_packed else None
        ws = ops.gemm_workspace(dev, M, N, 1 if mode == "swiglu" else 0)
        rc = _lib.lib.ps_routed_gemm_ex(x.data_ptr(), None if use_packed else W.data_ptr(),
                                        y.data_ptr(), M, K, N, 0, counts.data_ptr(), e,
                                        _lib.PS_DTYPE_F16, ws.data_ptr(), ws.numel(),
                                        _lib.status_tensor(dev).data_ptr(),
                                        _lib.stream_handle(dev))
        assert rc == _lib.PS_OK
        torch.cuda.synchronize()
        outs.append((y, pools))
    assert _lib.read_status(dev) == 0
    assert torch.equal(outs[0][0], outs[1][0])
    if mode == "qkv":
        for a, b in zip(outs[0][1], outs[1][1]):
            assert torch.equal(a, b)


def test_decode_step_packed_equals_unpacked():
    from parallel_serve_b200 import _lib
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    H, nh, FF, V, n_layers = 1024, 8, 2816, 4000, 2
    g = torch.Generator().manual_seed(9)

    def r(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(torch.float16)
    w = dict(layers=[dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF),
                          W_d=r(2, FF, H), ln1=1 + r(2, H, std=0.1), ln2=1 + r(2, H, std=0.1))
                     for _ in range(n_layers)],
             emb=r(2, V, H, std=1.0), ln_f=1 + r(2, H, std=0.1), W_lm=r(2, H, V))
    cfg = DecoderConfig(n_layers=n_layers, hidden=H, n_heads=nh, ffn=FF, vocab=V)
    mids = [0, 1, 1] * 8
    decs = [TwoModelDecoder(cfg, mids, 40, device="cuda", weights=w, packed=p)
            for p in (True, False)]
    assert decs[0].packed and not decs[1].packed
    for d in decs:
        d.fill_kv_random(32, seed=3)
        d.set_state(torch.arange(len(mids), dtype=torch.int32) * 7,
                    torch.full((len(mids),), 32, dtype=torch.int32))
        d.step_device("fused")
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0
    assert torch.equal(decs[0].logits, decs[1].logits)
    assert torch.equal(decs[0].next_tokens, decs[1].next_tokens)
