"""The projection chain (ps_routed_chain): a decode layer's O, gate_up, down
and next-QKV (or LM head) GEMMs, and under tensor parallelism the all-reduces
of the row-split ones, in one persistent launch with dataflow between them.

* Its GEMMs are the per-projection kernel's computation (same stream-K cut and
  summation order), so a decode step through chains must equal, bit for bit,
  the same step launched projection by projection (the path the other GPU
  tests pin to the oracle).
* Its all-reduce job is checked on one GPU with world 1 (the slot of this rank
  only) against the fp64 oracle of the layer; the multi-rank exchange is
  covered by the 2-GPU tensor-parallel tests and bench.py's parity gate.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu


def _decoder_pair(H, nh, FF, V, n_layers, mids, L0, seed, page_size=None):
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    g = torch.Generator().manual_seed(seed)

    def r(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(torch.float16)
    w = dict(layers=[dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF),
                          W_d=r(2, FF, H), ln1=1 + r(2, H, std=0.1), ln2=1 + r(2, H, std=0.1))
                     for _ in range(n_layers)],
             emb=r(2, V, H, std=1.0), ln_f=1 + r(2, H, std=0.1), W_lm=r(2, H, V))
    cfg = DecoderConfig(n_layers=n_layers, hidden=H, n_heads=nh, ffn=FF, vocab=V)
    L_cap = L0 + 8
    # the per-launch side keeps one CTA per SM for every projection, as the
    # chain does (its automatic per-shape grid cuts the split tiles differently)
    decs = [TwoModelDecoder(cfg, mids, L_cap, device="cuda", weights=w, chain=c,
                            page_size=page_size, auto_grid=False) for c in (True, False)]
    assert decs[0].use_chain and not decs[1].use_chain
    c0 = sum(1 for m in mids if m == 0)
    tok = torch.randint(0, V, (len(mids),), generator=g, dtype=torch.int32)
    for d in decs:   # lengths first: paged pools get their pages here
        d.set_state(tok, torch.full((len(mids),), L0, dtype=torch.int32))
    for li in range(n_layers):
        for m, n in ((0, c0), (1, len(mids) - c0)):
            if n:
                k, v = r(n, nh, L0, 128, std=1.0), r(n, nh, L0, 128, std=1.0)
                for d in decs:
                    d.write_kv(li, m, k.cuda(), v.cuda())
    return decs


@pytest.mark.parametrize("H,nh,FF,V,n_layers,mids,L0,page", [
    (256, 2, 512, 320, 2, [0, 1, 0, 1, 0, 1], 16, None),
    # Llama-7B layer shapes (stream-K split tiles in every projection), 48/16
    (4096, 32, 11008, 32000, 2, [0, 0, 0, 1] * 16, 64, None),
    # one model only; paged KV
    (1024, 8, 2816, 4000, 3, [1] * 24, 40, 16),
])
def test_chain_step_equals_per_launch_step_bitwise(H, nh, FF, V, n_layers, mids, L0, page):
    from parallel_serve_b200 import _lib
    chain, per = _decoder_pair(H, nh, FF, V, n_layers, mids, L0, seed=H + n_layers,
                               page_size=page)
    _lib.read_status(torch.device("cuda", 0))
    for step in range(2):          # the second step reuses the cleared counters / epoch
        for d in (chain, per):
            d.step_device("fused")
        torch.cuda.synchronize()
        assert _lib.read_status(torch.device("cuda", 0)) == 0, step
        assert torch.equal(chain.logits, per.logits), step
        assert torch.equal(chain.next_tokens, per.next_tokens), step
        assert torch.equal(chain.x, per.x), step
        for li in range(n_layers):       # every written position (the pools are not zeroed)
            for m in range(2):
                if chain.kpool[li][m] is not None:
                    kc, vc = chain.read_kv(li, m, L0 + step + 1)
                    kp, vp = per.read_kv(li, m, L0 + step + 1)
                    assert torch.equal(kc, kp) and torch.equal(vc, vp), (step, li, m)
    # a captured chain step replays identically
    for d in (chain, per):
        d.capture("fused")
        d.replay("fused")
    torch.cuda.synchronize()
    assert torch.equal(chain.logits, per.logits)
    assert _lib.read_status(torch.device("cuda", 0)) == 0


def test_chain_serial_mode_matches_per_launch():
    from parallel_serve_b200 import _lib
    chain, per = _decoder_pair(512, 4, 1024, 640, 2, [0, 1, 1, 0, 1, 1, 0, 0, 1], 24, seed=3)
    for d in (chain, per):
        d.step_device("serial")
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0
    assert torch.equal(chain.logits, per.logits)


def _job(**kw):
    from parallel_serve_b200 import _lib
    j = _lib.ChainJob()
    j.x_from = j.norm_from = j.res_from = -1
    for k, v in kw.items():
        setattr(j, k, v)
    return j


def test_chain_allreduce_job_world1_against_oracle():
    """O -> slot 0, all-reduce (world 1: residual + this rank's slot), gate_up
    with the folded norm from the all-reduce's sums of squares, down -> slot 1,
    all-reduce, LM head: the tensor-parallel chain layout on one rank."""
    import oracle
    from parallel_serve_b200 import _lib, ops
    from parallel_serve_b200._lib import ptr
    dev = torch.device("cuda", 0)
    H, FF, V, c0, M = 1024, 2816, 2048, 20, 44
    eps = 1e-5
    x0 = cpu_randn((M, H), 1)
    attn = cpu_randn((M, H), 2)
    Wo, Wgu = cpu_randn((2, H, H), 3, 0.02), cpu_randn((2, H, 2 * FF), 4, 0.02)
    Wd, Wlm = cpu_randn((2, FF, H), 5, 0.02), cpu_randn((2, H, V), 6, 0.02)
    x, a_ = x0.to(dev), torch.zeros(M, FF, dtype=torch.float16, device=dev)
    attn_d, Wo_d, Wgu_d, Wd_d, Wlm_d = (t.to(dev) for t in (attn, Wo, Wgu, Wd, Wlm))
    logits = torch.zeros(M, V, dtype=torch.float16, device=dev)
    sq_b = torch.zeros(M, H // 64, dtype=torch.float32, device=dev)
    sq_a = torch.zeros(M, H // 64, dtype=torch.float32, device=dev)
    counts = torch.tensor([c0, M - c0], dtype=torch.int32, device=dev)
    slot_bytes = (M * H * 2 + 255) // 256 * 256
    region = torch.zeros(_lib.lib.ps_symm_region_bytes(slot_bytes), dtype=torch.uint8,
                         device=dev)
    base = region.data_ptr()
    slot = [base + _lib.lib.ps_symm_slot_offset(s, slot_bytes) for s in (0, 1)]
    STORE, SWIGLU = _lib.PS_EPI_STORE, _lib.PS_EPI_SWIGLU
    e_o, e_d = ops.gemm_epilogue(STORE), ops.gemm_epilogue(STORE)
    e_gu = ops.gemm_epilogue(SWIGLU, in_sumsq=sq_b, norm_dim=H, eps=eps)
    e_lm = ops.gemm_epilogue(STORE, in_sumsq=sq_a, norm_dim=H, eps=eps)
    G, A = _lib.PS_JOB_GEMM, _lib.PS_JOB_ALLREDUCE
    jobs = [
        _job(kind=G, x=ptr(attn_d), W=ptr(Wo_d), y=slot[0], K=H, N=H, epi=e_o),
        _job(kind=A, src=0, slot=0, out=ptr(x), residual=ptr(x), out_sumsq=ptr(sq_b),
             row_elems=H),
        _job(kind=G, x=ptr(x), W=ptr(Wgu_d), y=ptr(a_), K=H, N=2 * FF, epi=e_gu, x_from=1,
             norm_from=1),
        _job(kind=G, x=ptr(a_), W=ptr(Wd_d), y=slot[1], K=FF, N=H, epi=e_d, x_from=2),
        _job(kind=A, src=3, slot=1, out=ptr(x), residual=ptr(x), out_sumsq=ptr(sq_a),
             row_elems=H, res_from=1),
        _job(kind=G, x=ptr(x), W=ptr(Wlm_d), y=ptr(logits), K=H, N=V, epi=e_lm, x_from=4,
             norm_from=4),
    ]
    arr = (_lib.ChainJob * len(jobs))(*jobs)
    ws = torch.zeros(_lib.lib.ps_routed_chain_workspace_bytes(M, len(jobs), 0),
                     dtype=torch.uint8, device=dev)
    peers = (ctypes.c_void_p * 1)(base)
    _lib.read_status(dev)
    rc = _lib.lib.ps_routed_chain(arr, len(jobs), M, ptr(counts), peers, 0, 1, slot_bytes,
                                  _lib.PS_DTYPE_F16, ptr(ws), ws.numel(),
                                  ptr(_lib.status_tensor(dev)), _lib.stream_handle(dev))
    assert rc == _lib.PS_OK, _lib.lib.ps_error_string(rc).decode()
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    # fp64 oracle with the kernel's fp16 roundings of x, a and the outputs
    r16 = "f16"
    xn = to_np(x0)
    x1 = oracle.round16(xn + oracle.round16(oracle.routed_gemm(to_np(attn), to_np(Wo), c0), r16),
                        r16)
    ones = np.ones((2, H))
    h = np.concatenate([oracle.rms_norm(x1[:c0], ones[0], eps), oracle.rms_norm(x1[c0:], ones[1],
                                                                               eps)])
    an = oracle.swiglu(oracle.routed_gemm(h, to_np(Wgu), c0), r16)
    x2 = oracle.round16(x1 + oracle.round16(oracle.routed_gemm(an, to_np(Wd), c0), r16), r16)
    h2 = np.concatenate([oracle.rms_norm(x2[:c0], ones[0], eps), oracle.rms_norm(x2[c0:], ones[1],
                                                                                eps)])
    want = oracle.routed_gemm(h2, to_np(Wlm), c0)
    assert rel_err(to_np(x), x2) < 1e-2
    assert rel_err(to_np(logits), want) < 1e-2
    sq_want = (oracle.round16(x2, r16) ** 2).reshape(M, H // 64, 64).sum(-1)
    assert rel_err(to_np(sq_a), sq_want) < 1e-3
    # a second launch (epoch 2, counters cleared by the first) gives the same logits
    first = logits.clone()
    x.copy_(x0.to(dev))
    rc = _lib.lib.ps_routed_chain(arr, len(jobs), M, ptr(counts), peers, 0, 1, slot_bytes,
                                  _lib.PS_DTYPE_F16, ptr(ws), ws.numel(),
                                  ptr(_lib.status_tensor(dev)), _lib.stream_handle(dev))
    assert rc == _lib.PS_OK
    torch.cuda.synchronize()
    assert _lib.read_status(dev) == 0
    assert torch.equal(logits, first)
