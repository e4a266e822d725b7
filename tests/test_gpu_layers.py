"""GPU parity of the per-layer kernels and the decode step against the CPU oracle.

Each kernel is called through the C ABI (via parallel_serve_b200.ops) on inputs
generated with a CPU generator, and compared to oracle/ref_ops.py with the
reference's metric rel = max|err| / mean|ref| (kernel/tests/test_correctness.py:34-38)
at the decode path's tolerance 1e-2 (the reference's own gate is 5e-2).
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu
TOL = 1e-2


def test_rmsnorm_routed():
    import oracle
    from parallel_serve_b200 import ops
    M, H, c0 = 37, 4096, 20
    x = cpu_randn((M, H), 1)
    w = (1.0 + cpu_randn((2, H), 2, 0.1))
    y = ops.rmsnorm_routed(x.cuda(), w.cuda(), split_point=c0, eps=1e-5)
    ref = np.concatenate([oracle.rms_norm(to_np(x[:c0]), to_np(w[0]), 1e-5, "f16"),
                          oracle.rms_norm(to_np(x[c0:]), to_np(w[1]), 1e-5, "f16")])
    assert rel_err(to_np(y), ref) < TOL


def test_swiglu():
    import oracle
    from parallel_serve_b200 import ops
    gu = cpu_randn((9, 2 * 1376), 3, 2.0)
    y = ops.swiglu(gu.cuda())
    assert rel_err(to_np(y), oracle.swiglu(to_np(gu), "f16")) < TOL


def test_gemm_swiglu_epilogue():
    import oracle
    from parallel_serve_b200 import _lib, ops
    for (M, K, FFn, c0) in [(64, 4096, 11008, 32), (40, 512, 1376, 9), (8, 256, 96, 8)]:
        x = cpu_randn((M, K), 4)
        W = cpu_randn((2, K, 2 * FFn), 5, 0.02)
        out = torch.empty(M, FFn, dtype=torch.float16, device="cuda")
        ops.routed_gemm_raw(x.cuda(), W.cuda(), out, split_point=c0, epilogue=_lib.PS_EPI_SWIGLU)
        gu = oracle.routed_gemm(to_np(x), to_np(W), c0)
        assert rel_err(to_np(out), oracle.swiglu(gu)) < TOL, (M, K, FFn, c0)


def test_gemm_residual_and_scatter():
    from parallel_serve_b200 import ops
    M, K, N, c0 = 24, 1024, 512, 10
    x = cpu_randn((M, K), 6)
    W = cpu_randn((2, K, N), 7, 0.02)
    res = cpu_randn((M, N), 8)
    perm = torch.randperm(M, generator=torch.Generator().manual_seed(0)).to(torch.int32)
    out = res.clone().cuda()
    ops.routed_gemm_raw(x.cuda(), W.cuda(), out, split_point=c0, scatter=perm.cuda(), residual=out)
    xn, Wn = to_np(x), to_np(W)
    ref = to_np(res).copy()
    for j in range(M):
        ref[int(perm[j])] += xn[j] @ Wn[0 if j < c0 else 1]
    assert rel_err(to_np(out), ref) < TOL


def test_gemm_device_counts_and_empty_model():
    from parallel_serve_b200 import ops
    M, K, N = 16, 512, 256
    x = cpu_randn((M, K), 9)
    W = cpu_randn((2, K, N), 10, 0.02)
    for c0 in (0, 5, 16):
        out = torch.zeros(M, N, dtype=torch.float16, device="cuda")
        counts = torch.tensor([c0, M - c0], dtype=torch.int32, device="cuda")
        ops.routed_gemm_raw(x.cuda(), W.cuda(), out, counts=counts)
        xn, Wn = to_np(x), to_np(W)
        ref = np.concatenate([xn[:c0] @ Wn[0], xn[c0:] @ Wn[1]])
        assert rel_err(to_np(out), ref) < TOL


def test_segment_attention_matches_sdpa():
    import oracle
    from parallel_serve_b200 import ops
    M, nh, c0 = 19, 3, 7
    qkv = cpu_randn((M, 3 * nh * 128), 11)
    out = ops.segment_attention(qkv.cuda(), nh, split_point=c0)
    ref = oracle.segment_attention(to_np(qkv), nh, c0)
    assert rel_err(to_np(out), ref) < TOL


def _pools(slots, nh, L_cap, seed):
    k = [cpu_randn((s, nh, L_cap, 128), seed + i) if s else None for i, s in enumerate(slots)]
    v = [cpu_randn((s, nh, L_cap, 128), seed + 10 + i) if s else None for i, s in enumerate(slots)]
    return k, v


@pytest.mark.parametrize("slots,L_cap,lens,chunk", [
    ((3, 2), 300, [5, 300, 64, 1, 129], 0),
    ((4, 4), 1100, [1025] * 8, 0),
    ((2, 1), 700, [700, 1, 333], 128),
    ((0, 3), 200, [200, 17, 64], 64),
])
def test_decode_attention(slots, L_cap, lens, chunk):
    import oracle
    from parallel_serve_b200 import ops
    nh = 2
    M = sum(slots)
    c0 = slots[0]
    k, v = _pools(slots, nh, L_cap, 20)
    q = cpu_randn((M, nh * 128), 30)
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32)
    kd = tuple(t.cuda() if t is not None else None for t in k)
    vd = tuple(t.cuda() if t is not None else None for t in v)
    out = ops.decode_attention(q.cuda(), kd, vd, pos.cuda(), n_heads=nh, max_len=L_cap,
                               split_point=c0, chunk=chunk)
    Kc = np.zeros((M, nh, L_cap, 128))
    Vc = np.zeros((M, nh, L_cap, 128))
    for j in range(M):
        m, sl = (0, j) if j < c0 else (1, j - c0)
        Kc[j] = to_np(k[m][sl])
        Vc[j] = to_np(v[m][sl])
    ref = oracle.decode_attention(to_np(q).reshape(M, nh, 128), Kc, Vc, np.array(lens))
    assert rel_err(to_np(out), ref.reshape(M, -1)) < TOL


@pytest.mark.parametrize("slots,nh,L_cap,chunk", [
    # few (token, head) items (4 heads per rank under 8-way tensor parallelism):
    # the balanced split over 3 CTAs per SM, forced (-1) and automatic (0),
    # uneven lengths so pieces straddle items
    ((12, 12), 4, 1100, -1),
    ((12, 12), 4, 1100, 0),
    ((1, 0), 1, 4000, -1),
    ((5, 9), 2, 300, -1),
])
def test_decode_attention_balanced_split(slots, nh, L_cap, chunk):
    import oracle
    from parallel_serve_b200 import _lib, ops
    M = sum(slots)
    c0 = slots[0]
    rng = np.random.default_rng(L_cap + M)
    lens = [int(x) for x in rng.integers(1, L_cap + 1, size=M)]
    lens[0] = L_cap
    k, v = _pools(slots, nh, L_cap, 60)
    q = cpu_randn((M, nh * 128), 61)
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32)
    kd = tuple(t.cuda() if t is not None else None for t in k)
    vd = tuple(t.cuda() if t is not None else None for t in v)
    for rep in range(2):   # the item counters are left at zero for the next call
        out = ops.decode_attention(q.cuda(), kd, vd, pos.cuda(), n_heads=nh, max_len=L_cap,
                                   split_point=c0, chunk=chunk)
        torch.cuda.synchronize()
        assert _lib.read_status(torch.device("cuda", 0)) == 0
        Kc = np.zeros((M, nh, L_cap, 128), dtype=np.float32)
        Vc = np.zeros((M, nh, L_cap, 128), dtype=np.float32)
        for j in range(M):
            m, sl = (0, j) if j < c0 else (1, j - c0)
            Kc[j] = to_np(k[m][sl])
            Vc[j] = to_np(v[m][sl])
        ref = oracle.decode_attention(to_np(q).reshape(M, nh, 128), Kc, Vc, np.array(lens))
        assert rel_err(to_np(out), ref.reshape(M, -1)) < TOL, rep


def test_decode_attention_balanced_split_tp8_shape():
    """One rank's shape under 8-way tensor parallelism at the decode benchmark:
    64 tokens (32 + 32), 4 heads, histories of ~2049 positions (256 items, the
    balanced split's case); checked against the per-chunk kernel on every
    token and against the oracle on a sample of tokens."""
    import oracle
    from parallel_serve_b200 import _lib, ops
    nh, L_cap, slots = 4, 2176, (32, 32)
    M, c0 = 64, 32
    g = torch.Generator(device="cuda").manual_seed(7)
    k = [torch.empty(s, nh, L_cap, 128, dtype=torch.float16, device="cuda").normal_(generator=g)
         for s in slots]
    v = [torch.empty(s, nh, L_cap, 128, dtype=torch.float16, device="cuda").normal_(generator=g)
         for s in slots]
    q = torch.empty(M, nh * 128, dtype=torch.float16, device="cuda").normal_(generator=g)
    lens = [2049 - (j % 7) * 3 for j in range(M)]
    pos = torch.tensor([L - 1 for L in lens], dtype=torch.int32, device="cuda")
    cnt = torch.tensor(slots, dtype=torch.int32, device="cuda")
    kw = dict(n_heads=nh, max_len=L_cap, counts=cnt)
    bal = ops.decode_attention(q, tuple(k), tuple(v), pos, chunk=0, **kw)
    ref = ops.decode_attention(q, tuple(k), tuple(v), pos, chunk=512, **kw)
    torch.cuda.synchronize()
    assert _lib.read_status(torch.device("cuda", 0)) == 0
    assert rel_err(to_np(bal), to_np(ref)) < TOL
    for j in (0, 5, 31, 32, 40, 63):
        m, sl = (0, j) if j < c0 else (1, j - c0)
        K = to_np(k[m][sl][:, :lens[j]])
        V = to_np(v[m][sl][:, :lens[j]])
        o = oracle.sdpa(to_np(q[j]).reshape(nh, 1, 128), K, V)[:, 0]
        assert rel_err(to_np(bal[j]).reshape(nh, 128), o) < TOL, j


def test_decode_attention_reproduces_reference_sdpa():
    """A cache holding exactly the segment's own keys reproduces the reference's
    no-KV per-model SDPA (kernel/src/two_model_block_routed.py:100-120)."""
    import oracle
    from parallel_serve_b200 import ops
    M, nh, c0 = 10, 2, 6
    H = nh * 128
    qkv = cpu_randn((M, 3 * H), 40)
    ref = oracle.segment_attention(to_np(qkv), nh, c0)
    slots = (c0, M - c0)
    q = qkv[:, :H].contiguous()
    Lc = max(c0, M - c0)
    kp, vp = [], []
    for m, (s0, s1) in enumerate(((0, c0), (c0, M))):
        n = s1 - s0
        kseg = qkv[s0:s1, H:2 * H].reshape(n, nh, 128).permute(1, 0, 2)  # [nh, n, 128]
        vseg = qkv[s0:s1, 2 * H:].reshape(n, nh, 128).permute(1, 0, 2)
        kpool = torch.zeros(slots[m], nh, Lc, 128, dtype=qkv.dtype)
        vpool = torch.zeros(slots[m], nh, Lc, 128, dtype=qkv.dtype)
        kpool[:, :, :n] = kseg
        vpool[:, :, :n] = vseg
        kp.append(kpool.cuda())
        vp.append(vpool.cuda())
    pos = torch.tensor([c0 - 1] * c0 + [M - c0 - 1] * (M - c0), dtype=torch.int32).cuda()
    out = ops.decode_attention(q.cuda(), tuple(kp), tuple(vp), pos, n_heads=nh,
                               max_len=Lc, split_point=c0)
    assert rel_err(to_np(out), ref) < TOL


def test_rope_kv_append():
    import oracle
    from parallel_serve_b200 import ops
    M, nh, L_cap, c0 = 6, 2, 40, 4
    H = nh * 128
    qkv = cpu_randn((M, 3 * H), 50)
    pos = torch.tensor([0, 3, 39, 7, 1, 22], dtype=torch.int32)
    k0 = torch.zeros(c0, nh, L_cap, 128, dtype=torch.float16, device="cuda")
    v0 = torch.zeros_like(k0)
    k1 = torch.zeros(M - c0, nh, L_cap, 128, dtype=torch.float16, device="cuda")
    v1 = torch.zeros_like(k1)
    cos, sin = ops.rope_tables(L_cap)
    q = torch.empty(M, H, dtype=torch.float16, device="cuda")
    ops.rope_kv_append(qkv.cuda(), q, (k0, k1), (v0, v1), cos, sin, pos.cuda(), n_heads=nh,
                       split_point=c0)
    c, s = oracle.rope_tables(L_cap)
    qn = to_np(qkv)
    p = pos.numpy().astype(np.int64)
    qref = oracle.apply_rope(qn[:, :H].reshape(M, nh, 128), p, c, s).reshape(M, H)
    kref = oracle.apply_rope(qn[:, H:2 * H].reshape(M, nh, 128), p, c, s)
    assert rel_err(to_np(q), qref) < TOL
    for j in range(M):
        kp, vp, sl = (k0, v0, j) if j < c0 else (k1, v1, j - c0)
        assert rel_err(to_np(kp[sl, :, p[j]]), kref[j]) < TOL
        assert np.array_equal(to_np(vp[sl, :, p[j]]).reshape(-1), qn[j, 2 * H:])


def _small_decoder_weights(n_layers, H, FF, V, seed):
    g = torch.Generator().manual_seed(seed)

    def r(*s, std=0.02):
        return (torch.randn(*s, generator=g) * std).to(torch.float16)
    layers = [dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF), W_d=r(2, FF, H),
                   ln1=(1 + r(2, H, std=0.1)), ln2=(1 + r(2, H, std=0.1)))
              for _ in range(n_layers)]
    return dict(layers=layers, emb=r(2, V, H, std=1.0), ln_f=(1 + r(2, H, std=0.1)),
                W_lm=r(2, H, V))


def _np_params(w):
    return dict(layers=[{k: to_np(v) for k, v in L.items()} for L in w["layers"]],
                emb=to_np(w["emb"]), ln_f=to_np(w["ln_f"]), W_lm=to_np(w["W_lm"]))


@pytest.mark.parametrize("fused_epilogues", [True, False])
@pytest.mark.parametrize("ids", [[0, 1] * 4, [1, 1, 0, 1, 0, 1, 1, 1], [0] * 5])
def test_decode_steps_match_oracle(ids, fused_epilogues):
    """3 greedy steps of a 2-layer two-model decoder (H=256, 2 heads) with a
    24-position prompt cache, fused and serial, against the oracle decode step;
    with the norm / RoPE / KV append fused into the GEMM epilogues or as
    separate launches."""
    import oracle
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    n_layers, H, nh, FF, V, L0 = 2, 256, 2, 512, 384, 24
    cfg = DecoderConfig(n_layers=n_layers, hidden=H, n_heads=nh, ffn=FF, vocab=V)
    w = _small_decoder_weights(n_layers, H, FF, V, 0)
    B = len(ids)
    c = (ids.count(0), ids.count(1))
    L_cap = L0 + 8
    for mode in ("fused", "serial"):
        dec = TwoModelDecoder(cfg, ids, L_cap, weights=w, fused_epilogues=fused_epilogues)
        assert dec.fused == fused_epilogues
        st = oracle.DecodeState(n_layers, c, nh, L_cap)
        g = torch.Generator().manual_seed(1)
        for li in range(n_layers):
            for m in range(2):
                if c[m]:
                    kk = (torch.randn(c[m], nh, L_cap, 128, generator=g)).to(torch.float16)
                    vv = (torch.randn(c[m], nh, L_cap, 128, generator=g)).to(torch.float16)
                    dec.kpool[li][m].copy_(kk)
                    dec.vpool[li][m].copy_(vv)
                    st.k[li][m][:] = to_np(kk)
                    st.v[li][m][:] = to_np(vv)
        tokens = np.array([(7 * i + 3) % V for i in range(B)])
        seq = np.full(B, L0)
        dec.set_state(torch.from_numpy(tokens), torch.from_numpy(seq))
        cos, sin = oracle.rope_tables(L_cap)
        P = _np_params(w)
        for step in range(3):
            dec.step_device(mode)
            torch.cuda.synchronize()
            nxt_ref, logits_ref = oracle.decode_step(tokens, np.array(ids), P, st, seq, nh, cos,
                                                     sin, 1e-5)
            assert rel_err(to_np(dec.logits), logits_ref) < TOL, (mode, step)
            got = dec.next_tokens.cpu().numpy()
            # greedy picks agree wherever the oracle's top-2 margin is not within fp16 noise
            srt = np.sort(logits_ref, axis=-1)
            clear = (srt[:, -1] - srt[:, -2]) > 0.05
            perm, _ = oracle.route_partition(np.array(ids))
            clear_orig = np.empty_like(clear)
            clear_orig[perm] = clear
            assert np.array_equal(got[clear_orig], nxt_ref[clear_orig]), (mode, step)
            tokens = nxt_ref
            dec.tokens.copy_(torch.from_numpy(tokens).to(torch.int32))
        assert dec.seq_len.cpu().numpy().tolist() == (np.full(B, L0 + 3)).tolist()
        dec.check_status()


def test_decode_graph_serves_any_split():
    """One captured graph replays correctly after the model ids change."""
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    cfg = DecoderConfig(n_layers=1, hidden=256, n_heads=2, ffn=256, vocab=256)
    w = _small_decoder_weights(1, 256, 256, 256, 3)
    dec = TwoModelDecoder(cfg, [0, 1, 0, 1], 16, weights=w)
    dec.fill_kv_random(8)
    dec.step_device("fused")
    dec.capture("fused")
    dec.seq_len.fill_(8)
    dec.tokens.copy_(torch.tensor([1, 2, 3, 4], dtype=torch.int32))
    dec.replay("fused")
    a = dec.logits.clone()
    dec.seq_len.fill_(8)
    dec.tokens.copy_(torch.tensor([1, 2, 3, 4], dtype=torch.int32))
    dec.step_device("fused")
    assert torch.equal(a, dec.logits)
    dec.check_status()


def test_kv_layers_alias_pool_sets():
    """kv_layers=2 over 3 layers: layer 2 shares layer 0's pools; the step runs
    clean and reads a full history in every layer."""
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    cfg = DecoderConfig(n_layers=3, hidden=256, n_heads=2, ffn=256, vocab=256)
    w = _small_decoder_weights(3, 256, 256, 256, 5)
    dec = TwoModelDecoder(cfg, [0, 1, 1], 32, weights=w, kv_layers=2)
    assert dec.kpool[2] is dec.kpool[0] and dec.vpool[2] is dec.vpool[0]
    assert dec.kpool[1] is not dec.kpool[0]
    dec.fill_kv_random(20)
    dec.step_device("fused")
    torch.cuda.synchronize()
    dec.check_status()
    assert np.isfinite(to_np(dec.logits)).all()
    with pytest.raises(ValueError):
        TwoModelDecoder(cfg, [0, 1], 16, weights=w, kv_layers=4)
