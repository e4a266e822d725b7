"""Paged KV cache on the GPU: paged decode attention, the QKV epilogue's paged
KV append and the paged decoder, against the contiguous kernels (bit-identical:
same math, same chunking) and the oracle (rel < 1e-2).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _paged_copy(pools_c, counts, page_size, seed):
    """Page pools holding the contiguous pools' histories, pages in shuffled order.
    Returns (k_pages, v_pages, block_table [M, max_pages] on the GPU)."""
    from parallel_serve_b200.paged_kv import BlockTable, PageAllocator
    k_c, v_c = pools_c
    L_cap = next(t for t in k_c if t is not None).shape[2]
    max_pages = -(-L_cap // page_size)
    n_pages = [c * max_pages + 3 for c in counts]               # a few spare pages
    alloc = tuple(PageAllocator(n, shuffle_seed=seed + m) for m, n in enumerate(n_pages))
    bt = BlockTable([0] * counts[0] + [1] * counts[1], alloc, max_pages, page_size, "cuda")
    bt.ensure(range(sum(counts)), L_cap)
    bt.sync()
    kp, vp = [], []
    for m in range(2):
        if counts[m] == 0:
            kp.append(None)
            vp.append(None)
            continue
        nh = k_c[m].shape[1]
        kk = torch.zeros(n_pages[m], nh, page_size, 128, dtype=k_c[m].dtype, device="cuda")
        vv = torch.zeros_like(kk)
        for s in range(counts[m]):
            j = s + (counts[0] if m else 0)
            for i, pg in enumerate(bt.pages_of(j)):
                n = min(page_size, L_cap - i * page_size)
                kk[pg, :, :n] = k_c[m][s, :, i * page_size:i * page_size + n]
                vv[pg, :, :n] = v_c[m][s, :, i * page_size:i * page_size + n]
        kp.append(kk)
        vp.append(vv)
    return tuple(kp), tuple(vp), bt


@pytest.mark.parametrize("page_size,chunk", [(16, 0), (16, 128), (64, 256), (256, 0), (8, 0)])
def test_paged_attention_bit_identical_to_contiguous(page_size, chunk):
    import oracle
    from parallel_serve_b200 import _lib, ops
    counts, nh, L_cap = (5, 3), 4, 700
    M = sum(counts)
    k_c = tuple(cpu_randn((c, nh, L_cap, 128), 10 + m).cuda() for m, c in enumerate(counts))
    v_c = tuple(cpu_randn((c, nh, L_cap, 128), 20 + m).cuda() for m, c in enumerate(counts))
    q = cpu_randn((M, nh * 128), 30).cuda()
    pos = torch.tensor([0, 5, 15, 16, 699, 130, 383, 64], dtype=torch.int32, device="cuda")
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    ref = ops.decode_attention(q, k_c, v_c, pos, n_heads=nh, max_len=L_cap, counts=cnt,
                               chunk=chunk)
    kp, vp, bt = _paged_copy((k_c, v_c), counts, page_size, seed=page_size)
    out = ops.paged_decode_attention(q, kp, vp, pos, bt.device, n_heads=nh, max_len=L_cap,
                                     counts=cnt, chunk=chunk)
    torch.cuda.synchronize()
    assert _lib.read_status(q.device) == 0
    assert torch.equal(out, ref)
    # and against the oracle, through the page layout
    p = pos.cpu().numpy()
    for j in range(M):
        m = 0 if j < counts[0] else 1
        K = oracle.gather_pages(to_np(kp[m]), bt.host[j], page_size, int(p[j]) + 1)
        V = oracle.gather_pages(to_np(vp[m]), bt.host[j], page_size, int(p[j]) + 1)
        o = oracle.sdpa(to_np(q[j]).reshape(nh, 1, 128), K, V)[:, 0]
        assert rel_err(to_np(out[j]).reshape(nh, 128), o) < TOL


def test_paged_attention_bad_page_sets_status():
    from parallel_serve_b200 import _lib, ops
    nh, ps = 2, 16
    kp = torch.zeros(4, nh, ps, 128, dtype=torch.float16, device="cuda")
    q = torch.zeros(2, nh * 128, dtype=torch.float16, device="cuda")
    pos = torch.tensor([20, 3], dtype=torch.int32, device="cuda")
    bt = torch.tensor([[0, 9], [1, -1]], dtype=torch.int32, device="cuda")    # page 9 > pool
    _lib.read_status(q.device)
    out = torch.full_like(q, 7.0)
    ops.paged_decode_attention(q, (kp, None), (kp, None), pos, bt, n_heads=nh, max_len=32,
                               split_point=2, out=out)
    assert _lib.read_status(q.device) & _lib.PS_ERR_BAD_INDEX
    assert (out[0] == 7.0).all()          # the bad row is skipped
    assert (out[1] == 0.0).all()          # the good row (zero K/V, zero q) is computed


def test_paged_qkv_epilogue_matches_contiguous():
    """The QKV epilogue writes the same k / v bits into pages as into contiguous pools."""
    from parallel_serve_b200 import _lib, ops
    counts, nh, L_cap, ps = (6, 4), 2, 64, 16
    M, H = sum(counts), nh * 128
    x = cpu_randn((M, H), 41).cuda()
    W = cpu_randn((2, H, 3 * H), 42, 0.02).cuda()
    pos = torch.tensor([0, 15, 16, 17, 63, 31, 1, 47, 48, 2], dtype=torch.int32, device="cuda")
    cnt = torch.tensor(counts, dtype=torch.int32, device="cuda")
    cos, sin = ops.rope_tables(L_cap)
    k_c = tuple(torch.zeros(c, nh, L_cap, 128, dtype=torch.float16, device="cuda") for c in counts)
    v_c = tuple(torch.zeros_like(t) for t in k_c)
    kp, vp, bt = _paged_copy((k_c, v_c), counts, ps, seed=5)     # zero pages, shuffled table
    q_c = torch.empty(M, H, dtype=torch.float16, device="cuda")
    e = ops.gemm_epilogue(_lib.PS_EPI_QKV_ROPE, k_pools=k_c, v_pools=v_c, pos=pos, rope_cos=cos,
                          rope_sin=sin, n_heads=nh)
    ops.routed_gemm_ex(x, W, q_c, e, counts=cnt)
    q_p = torch.empty_like(q_c)
    e = ops.gemm_epilogue(_lib.PS_EPI_QKV_ROPE, k_pools=kp, v_pools=vp, pos=pos, rope_cos=cos,
                          rope_sin=sin, n_heads=nh, block_table=bt.device)
    ops.routed_gemm_ex(x, W, q_p, e, counts=cnt)
    torch.cuda.synchronize()
    assert _lib.read_status(x.device) == 0
    assert torch.equal(q_p, q_c)
    for j in range(M):
        m, s = (0, j) if j < counts[0] else (1, j - counts[0])
        p = int(pos[j])
        pg = bt.pages_of(j)[p // ps]
        assert torch.equal(kp[m][pg, :, p % ps], k_c[m][s, :, p])
        assert torch.equal(vp[m][pg, :, p % ps], v_c[m][s, :, p])
        assert k_c[m][s, :, p].abs().sum() > 0
    for m in range(2):          # nothing else was written: one row per (token, head)
        assert int((kp[m].abs().sum(-1) > 0).sum()) == counts[m] * nh
        assert int((vp[m].abs().sum(-1) > 0).sum()) == counts[m] * nh


def _weights(n_layers, H, FF, V, seed):
    g = torch.Generator().manual_seed(seed)

    def r(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(torch.float16)
    layers = [dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF), W_d=r(2, FF, H),
                   ln1=(1 + r(2, H, std=0.1)), ln2=(1 + r(2, H, std=0.1)))
              for _ in range(n_layers)]
    return dict(layers=layers, emb=r(2, V, H, std=1.0), ln_f=(1 + r(2, H, std=0.1)),
                W_lm=r(2, H, V))


@pytest.mark.parametrize("page_size", [16, 32])
def test_paged_decoder_matches_contiguous_and_oracle(page_size):
    """4 greedy steps (crossing a page boundary) of a 2-layer decoder with paged
    KV give bit-identical logits to the contiguous-KV decoder, and match the
    oracle decode step; the last two steps replay a captured graph."""
    import oracle
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    n_layers, H, nh, FF, V, L0 = 2, 256, 2, 512, 384, 30
    ids = [0, 1, 1, 0, 1, 1]
    cfg = DecoderConfig(n_layers=n_layers, hidden=H, n_heads=nh, ffn=FF, vocab=V)
    w = _weights(n_layers, H, FF, V, 0)
    c = (ids.count(0), ids.count(1))
    L_cap = 64
    dec_c = TwoModelDecoder(cfg, ids, L_cap, weights=w)
    dec_p = TwoModelDecoder(cfg, ids, L_cap, weights=w, page_size=page_size)
    st = oracle.DecodeState(n_layers, c, nh, L_cap)
    tokens = np.array([(5 * i + 1) % V for i in range(len(ids))])
    seq = np.full(len(ids), L0)
    for dec in (dec_c, dec_p):
        dec.set_state(torch.from_numpy(tokens), torch.from_numpy(seq))
        dec.reserve(8)
    g = torch.Generator().manual_seed(1)
    for li in range(n_layers):
        for m in range(2):
            kk = torch.randn(c[m], nh, L0, 128, generator=g).to(torch.float16)
            vv = torch.randn(c[m], nh, L0, 128, generator=g).to(torch.float16)
            for dec in (dec_c, dec_p):
                dec.write_kv(li, m, kk.cuda(), vv.cuda())
            st.k[li][m][:, :, :L0] = to_np(kk)
            st.v[li][m][:, :, :L0] = to_np(vv)
    P = dict(layers=[{k: to_np(v) for k, v in L.items()} for L in w["layers"]],
             emb=to_np(w["emb"]), ln_f=to_np(w["ln_f"]), W_lm=to_np(w["W_lm"]))
    cos, sin = oracle.rope_tables(L_cap)
    perm, _ = oracle.route_partition(np.array(ids))
    for step in range(4):
        for dec in (dec_c, dec_p):
            if step < 2:
                dec.step_device("fused")
            else:
                if step == 2:
                    saved_len, saved_tok = dec.seq_len.clone(), dec.tokens.clone()
                    dec.capture("fused")      # capture ran one step: restore it
                    dec.seq_len.copy_(saved_len)
                    dec.tokens.copy_(saved_tok)
                dec.replay("fused")
        torch.cuda.synchronize()
        assert torch.equal(dec_p.logits, dec_c.logits), step
        nxt_ref, logits_ref = oracle.decode_step(tokens, np.array(ids), P, st, seq, nh, cos, sin,
                                                 1e-5)
        assert rel_err(to_np(dec_p.logits), logits_ref) < TOL, step
        srt = np.sort(logits_ref, axis=-1)
        clear = np.empty(len(ids), dtype=bool)
        clear[perm] = (srt[:, -1] - srt[:, -2]) > 0.05
        got = dec_p.next_tokens.cpu().numpy()
        assert np.array_equal(got[clear], nxt_ref[clear]), step
        tokens = nxt_ref
        for dec in (dec_c, dec_p):
            dec.tokens.copy_(torch.from_numpy(tokens).to(torch.int32))
    for li in range(n_layers):
        for m in range(2):
            kc, vc = dec_c.read_kv(li, m, L0 + 4)
            kq, vq = dec_p.read_kv(li, m, L0 + 4)
            assert torch.equal(kc, kq) and torch.equal(vc, vq)
    dec_c.check_status()
    dec_p.check_status()
