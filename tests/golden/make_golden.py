"""Generate the golden fixtures in this directory from the reference's own code.

Run once, where the reference sources are available (they are not on the GPU
machines):  python tests/golden/make_golden.py /path/to/reference

It imports, on CPU and in float64:
  kernel/src/routed_gemm.py           reference_routed_gemm      (:200-204)
  experiments/routed_linear_n2.py     reference_routed_linear    (:156-160)
  experiments/two_model_block.py      TransformerBlock (:42-74), TwoModelBlockFused (:77-120)
  kernel/src/two_model_block_routed.py TwoModelBlockRouted (:40-153), with its
                                       Triton routed_gemm swapped for the
                                       reference's own reference_routed_gemm
                                       (the Triton kernel needs a GPU)
and stores seeded inputs (rounded to float16 so a GPU fp16 run sees the same
bits) with the reference's outputs as compressed .npz files.

F.rms_norm is called by the reference without eps, i.e. eps = machine epsilon of
the computation dtype; each block fixture records the eps that applied.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

OUT = os.path.dirname(os.path.abspath(__file__))


def f16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float16).to(torch.float64)


def randn(g: torch.Generator, *shape, scale=1.0) -> torch.Tensor:
    return f16(torch.randn(*shape, generator=g, dtype=torch.float64) * scale)


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "kernel"))
    sys.path.insert(0, os.path.join(ref_root, "experiments"))
    import src.routed_gemm as rg  # noqa: E402
    import src.two_model_block_routed as tmbr  # noqa: E402
    import routed_linear_n2 as rl  # noqa: E402
    import two_model_block as tmb  # noqa: E402

    g = torch.Generator("cpu").manual_seed(1234)

    # ---- routed GEMM cases (shapes echo kernel/tests/test_correctness.py, shrunk)
    cases = [(32, 256, 384, 16), (37, 128, 136, 13), (16, 64, 64, 0), (16, 64, 64, 16),
             (1, 64, 128, 1), (300, 128, 256, 150), (64, 256, 128, 48), (64, 256, 128, 8)]
    arrs = {}
    for i, (M, K, N, sp) in enumerate(cases):
        x = randn(g, M, K)
        W = randn(g, 2, K, N, scale=0.02)
        y = rg.reference_routed_gemm(x, W, sp)
        y2 = rl.reference_routed_linear(x, W, sp)
        assert torch.equal(y, y2)
        arrs[f"c{i}_x"] = x.numpy().astype(np.float16)
        arrs[f"c{i}_W"] = W.numpy().astype(np.float16)
        arrs[f"c{i}_y"] = y.numpy().astype(np.float32)
        arrs[f"c{i}_split"] = np.array(sp)
    arrs["ncases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(OUT, "routed_gemm.npz"), **arrs)

    # ---- blocks: H=256, 2 heads of 128, FF=256
    Hs, nh, FFs = 256, 2, 256
    eps64 = float(torch.finfo(torch.float64).eps)

    def block(seed):
        torch.manual_seed(seed)
        b = tmb.TransformerBlock(Hs, FFs, nh, "cpu", torch.float64)
        for name in ("W_qkv", "W_o", "W_gu", "W_d", "ln1", "ln2"):
            setattr(b, name, f16(getattr(b, name)))
        return b

    ba, bb = block(1), block(2)
    arrs = {"H": np.array(Hs), "n_heads": np.array(nh), "FF": np.array(FFs), "eps": np.array(eps64)}
    for tag, b in (("a", ba), ("b", bb)):
        for name in ("W_qkv", "W_o", "W_gu", "W_d", "ln1", "ln2"):
            arrs[f"{tag}_{name}"] = getattr(b, name).numpy().astype(np.float16)
    M = 12
    xa = randn(g, M, Hs)
    xb = randn(g, M, Hs)
    with torch.no_grad():
        arrs["xa"] = xa.numpy().astype(np.float16)
        arrs["xb"] = xb.numpy().astype(np.float16)
        arrs["ya_serial"] = ba(xa).numpy().astype(np.float32)
        arrs["yb_serial"] = bb(xb).numpy().astype(np.float32)
        fused = tmb.TwoModelBlockFused(ba, bb)
        arrs["y_fused"] = fused(torch.stack([xa, xb])).numpy().astype(np.float32)
    np.savez_compressed(os.path.join(OUT, "blocks.npz"), **arrs)

    # ---- TwoModelBlockRouted, unbalanced split, routed GEMM = reference_routed_gemm
    tmbr.routed_gemm = rg.reference_routed_gemm
    torch.manual_seed(7)
    blk = tmbr.TwoModelBlockRouted(Hs, FFs, nh, device="cpu", dtype=torch.float64)
    with torch.no_grad():
        for name in ("W_qkv", "W_o", "W_gu", "W_d"):
            getattr(blk, name).data = f16(getattr(blk, name).data)
        blk.ln1.data = f16(torch.randn(2, Hs, generator=g, dtype=torch.float64) * 0.01 + 1.0)
        blk.ln2.data = f16(torch.randn(2, Hs, generator=g, dtype=torch.float64) * 0.01 + 1.0)
    arrs = {"H": np.array(Hs), "n_heads": np.array(nh), "FF": np.array(FFs), "eps": np.array(eps64)}
    for name in ("W_qkv", "W_o", "W_gu", "W_d", "ln1", "ln2"):
        arrs[name] = getattr(blk, name).data.numpy().astype(np.float16)
    for i, (Mt, sp) in enumerate([(20, 7), (20, 0), (20, 20), (33, 17)]):
        x = randn(g, Mt, Hs)
        with torch.no_grad():
            y = blk(x, sp)
        arrs[f"r{i}_x"] = x.numpy().astype(np.float16)
        arrs[f"r{i}_y"] = y.numpy().astype(np.float32)
        arrs[f"r{i}_split"] = np.array(sp)
    arrs["ncases"] = np.array(4)
    np.savez_compressed(os.path.join(OUT, "block_routed.npz"), **arrs)
    print("wrote", sorted(f for f in os.listdir(OUT) if f.endswith(".npz")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
