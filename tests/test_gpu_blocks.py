"""GPU parity of the reference-facing operator modules — the drop-in boundary.

* ``routed_gemm`` / ``routed_linear_n2`` (kernel/src/routed_gemm.py:152-197,
  experiments/routed_linear_n2.py:118-153) on every case of
  tests/golden/routed_gemm.npz;
* ``TransformerBlock``, ``TwoModelBlockFused``, ``TwoModelBlockBMM``
  (experiments/two_model_block.py:42-195) on tests/golden/blocks.npz and
  ``TwoModelBlockRouted`` (kernel/src/two_model_block_routed.py:40-153) on
  tests/golden/block_routed.npz — outputs of the reference's own Python
  modules (tests/golden/make_golden.py), weights assigned the way the
  reference's benchmarks assign them;
* one decoder layer, one decode step, at the Llama-7B shape (hidden 4096,
  32 heads, FF 11008; 16 sequences per model over a 1024-position N(0,1) KV
  cache) and at the Llama-13B shape (hidden 5120, 40 heads, FF 13824; 8
  sequences per model over 512 positions, a prefix of the 13B workload's
  4096 so the oracle finishes in seconds): fused against serial against the
  oracle's decode layer.

Metric rel = max|err| / mean|ref| (kernel/tests/test_correctness.py:34-38) at
the 1e-2 gate. The reference's blocks normalise with eps = finfo(dtype).eps
(F.rms_norm's default): the golden outputs were made in float64, these
kernels run fp16 with fp16's eps; the difference (1e-3 against mean squares
near 1) is far inside the gate.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, cpu_randn, rel_err, to_np

pytestmark = pytest.mark.gpu
TOL = 1e-2
F16 = torch.float16


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _t(a, dtype=F16):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


# ---------------------------------------------------------------- routed GEMM
@pytest.mark.parametrize("fn", ["routed_gemm", "routed_linear_n2"])
def test_routed_gemm_golden(fn):
    import parallel_serve_b200 as ps
    op = getattr(ps, fn)
    d = _load("routed_gemm.npz")
    for i in range(int(d["ncases"])):
        x, W, sp = _t(d[f"c{i}_x"]), _t(d[f"c{i}_W"]), int(d[f"c{i}_split"])
        y = op(x, W, sp)
        torch.cuda.synchronize()
        assert y.shape == (x.shape[0], W.shape[2]) and y.dtype == F16 and y.device == x.device
        assert rel_err(to_np(y), d[f"c{i}_y"]) < TOL, (fn, i)


def test_reference_routed_gemm_is_the_torch_restatement():
    from parallel_serve_b200.routed_gemm import reference_routed_gemm
    from parallel_serve_b200.routed_linear_n2 import reference_routed_linear
    d = _load("routed_gemm.npz")
    x, W, sp = _t(d["c1_x"], torch.float32), _t(d["c1_W"], torch.float32), int(d["c1_split"])
    for f in (reference_routed_gemm, reference_routed_linear):
        assert rel_err(to_np(f(x, W, sp)), d["c1_y"]) < 1e-5


def test_routed_gemm_rejects_what_the_reference_rejects():
    from parallel_serve_b200 import routed_gemm
    x = torch.zeros(8, 64, dtype=F16, device="cuda")
    W = torch.zeros(2, 64, 64, dtype=F16, device="cuda")
    with pytest.raises(ValueError):
        routed_gemm(x, W, 9)                     # split beyond M
    with pytest.raises(ValueError):
        routed_gemm(x, W[:, :32], 4)             # K mismatch
    with pytest.raises(ValueError):
        routed_gemm(x, W[:1], 4)                 # not two weight sets


# ---------------------------------------------------------------- blocks
_NAMES = ("W_qkv", "W_o", "W_gu", "W_d", "ln1", "ln2")


def _blocks(d):
    from parallel_serve_b200.two_model_block import TransformerBlock
    H, FF, nh = int(d["H"]), int(d["FF"]), int(d["n_heads"])
    out = []
    for tag in ("a", "b"):
        b = TransformerBlock(H, FF, nh, "cuda", F16)
        for n in _NAMES:                 # the reference assigns plain tensors
            setattr(b, n, _t(d[f"{tag}_{n}"]))
        out.append(b)
    return out


def test_transformer_block_golden():
    d = _load("blocks.npz")
    ba, bb = _blocks(d)
    for b, x, y in ((ba, "xa", "ya_serial"), (bb, "xb", "yb_serial")):
        out = b(_t(d[x]))
        torch.cuda.synchronize()
        assert out.shape == d[x].shape
        assert rel_err(to_np(out), d[y]) < TOL, x


def test_fused_and_bmm_blocks_golden():
    from parallel_serve_b200.two_model_block import TwoModelBlockBMM, TwoModelBlockFused
    d = _load("blocks.npz")
    ba, bb = _blocks(d)
    xa, xb = _t(d["xa"]), _t(d["xb"])
    M = xa.shape[0]
    y = TwoModelBlockFused(ba, bb)(torch.stack([xa, xb]))
    assert y.shape == (2, M, xa.shape[1])
    assert rel_err(to_np(y), d["y_fused"]) < TOL
    bmm = TwoModelBlockBMM(ba, bb)
    y2 = bmm(torch.cat([xa, xb]), M)
    assert rel_err(to_np(y2), d["y_fused"].reshape(2 * M, -1)) < TOL
    torch.cuda.synchronize()
    with pytest.raises(ValueError):              # the reference's BMM block is balanced-only
        bmm(torch.cat([xa, xb]), M - 1)


def test_routed_block_golden():
    from parallel_serve_b200 import TwoModelBlockRouted
    d = _load("block_routed.npz")
    H, FF, nh = int(d["H"]), int(d["FF"]), int(d["n_heads"])
    blk = TwoModelBlockRouted(H, FF, nh, device="cuda", dtype=F16)
    for n in _NAMES:                             # re-pointed as bench_full_stack.py does
        getattr(blk, n).data = _t(d[n])
    for i in range(int(d["ncases"])):
        x, sp = _t(d[f"r{i}_x"]), int(d[f"r{i}_split"])
        y = blk(x, sp)
        cnt = torch.tensor([sp, x.shape[0] - sp], dtype=torch.int32, device="cuda")
        y_dev = blk(x, counts=cnt)               # device split: same kernels, same bits
        torch.cuda.synchronize()
        assert rel_err(to_np(y), d[f"r{i}_y"]) < TOL, (i, sp)
        assert torch.equal(y, y_dev), (i, sp)
    with pytest.raises(ValueError):
        blk(x, x.shape[0] + 1)
    with pytest.raises(ValueError):
        blk(x[:, :128], 0)


# ---------------------------------------------------------------- one decoder layer
def _layer_weights(H, FF, V, seed):
    """One layer of both models, N(0, 0.02) fp16 from a CPU generator; norm
    weights near 1 so the folded-norm path is exercised."""
    g = torch.Generator().manual_seed(seed)

    def r(*s, std=0.02, mean=0.0):
        return (torch.randn(*s, generator=g) * std + mean).to(F16)
    layer = dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF), W_d=r(2, FF, H),
                 ln1=r(2, H, std=0.1, mean=1.0), ln2=r(2, H, std=0.1, mean=1.0))
    return dict(layers=[layer], emb=r(2, V, H, std=1.0), ln_f=r(2, H, std=0.1, mean=1.0),
                W_lm=r(2, H, V))


@pytest.mark.parametrize("shape", ["llama7b", "llama13b"])
def test_one_layer_decode_fused_vs_serial_vs_oracle(shape):
    import oracle
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    if shape == "llama7b":
        H, nh, FF, per_model, L0 = 4096, 32, 11008, 16, 1024
    else:
        H, nh, FF, per_model, L0 = 5120, 40, 13824, 8, 512
    V = 256
    ids = [i % 2 for i in range(2 * per_model)]          # interleaved, as model_id[i] = i % 2
    B, c = len(ids), (per_model, per_model)
    cfg = DecoderConfig(n_layers=1, hidden=H, n_heads=nh, ffn=FF, vocab=V)
    w = _layer_weights(H, FF, V, seed=11)
    L_cap = L0 + 8
    dec = TwoModelDecoder(cfg, ids, L_cap, weights=w)
    st = oracle.DecodeState(1, c, nh, L_cap)
    for m in range(2):
        kk = cpu_randn((c[m], nh, L0, 128), 100 + m)
        vv = cpu_randn((c[m], nh, L0, 128), 200 + m)
        dec.write_kv(0, m, kk.cuda(), vv.cuda())
        st.k[0][m][:, :, :L0] = to_np(kk)
        st.v[0][m][:, :, :L0] = to_np(vv)
    tokens = np.array([(37 * i + 5) % V for i in range(B)])
    seq = np.full(B, L0)
    outs = {}
    for mode in ("fused", "serial"):
        dec.set_state(torch.from_numpy(tokens), torch.from_numpy(seq))
        dec.step_device(mode)
        torch.cuda.synchronize()
        outs[mode] = to_np(dec.x)                        # layer output, routed order
    dec.check_status()
    # oracle: the same layer from the same embedding rows
    perm, counts = oracle.route_partition(np.array(ids))
    c0 = int(counts[0])
    mrow = (np.arange(B) >= c0).astype(np.int64)
    x0 = to_np(w["emb"])[mrow, tokens[perm]]
    P = {k: to_np(v) for k, v in w["layers"][0].items()}
    cos, sin = oracle.rope_tables(L_cap)
    ref = oracle.decode_layer(x0, P, st, 0, nh, c0, seq[perm].astype(np.int64), cos, sin, 1e-5)
    assert rel_err(outs["fused"], ref) < TOL
    assert rel_err(outs["serial"], ref) < TOL
    assert rel_err(outs["fused"], outs["serial"]) < TOL
