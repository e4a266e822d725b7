"""Timed CPU baseline of the decode step — the oracle restatement of the
reference's serial torch path, run on the host cores (test / benchmark
infrastructure only, never the product).

The reference path per layer is experiments/two_model_block.py:54-74 with
decode attention over a KV cache. One full Llama-7B-shape step over
32 layers does not fit host RAM in fp32 (52 GB of weights), so the sample is
ONE decoder layer (both models' weights, fp32, every sequence with its full KV
history) plus the LM head; the per-step time is layer_time x n_layers +
head_time, reported as an extrapolation.
"""
from __future__ import annotations

import os
import time

import numpy as np

from . import ref_ops as R


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [d.get("num_threads", 0) for d in threadpool_info() if d.get("user_api") == "blas"]
        return max(n) if n else (os.cpu_count() or 1)
    except Exception:
        return os.cpu_count() or 1


class DecodeSample:
    """One decode layer + LM head for B sequences (c0 on model 0) with KV
    length L, inputs generated once (weights, caches, hidden rows) so that
    repeated timings measure the computation alone.

    ``slice_factor`` S > 1 computes 1/S of the layer (n_heads/S heads, FF/S
    intermediate columns, V/S vocabulary columns; work is linear in each) and
    scales the time by S. ``run()`` returns seconds per layer, per head, the
    extrapolated step time (layer x n_layers + head) and tokens/s.
    """

    def __init__(self, B: int, c0: int, H: int, n_heads: int, FF: int, V: int, L: int,
                 n_layers: int, seed: int = 0, slice_factor: int = 1):
        rng = np.random.default_rng(seed)
        f32 = np.float32
        hd = H // n_heads
        S = max(1, int(slice_factor))
        nh = max(1, n_heads // S)
        FFs = max(8, FF // S)
        Vs = max(8, V // S)
        Hq = nh * hd  # q/k/v width actually computed

        def w(*shape, s=0.02):
            return (rng.standard_normal(shape, dtype=f32) * s).astype(f32)

        self.layer = dict(W_qkv=w(2, H, 3 * Hq), W_o=w(2, Hq, H), W_gu=w(2, H, 2 * FFs),
                          W_d=w(2, FFs, H), ln1=np.ones((2, H), f32), ln2=np.ones((2, H), f32))
        self.W_lm = w(2, H, Vs)
        self.lnf = np.ones((2, H), f32)
        # KV history stored in fp16 (as on the GPU), widened per sequence when used.
        self.K = rng.standard_normal((B, nh, L + 1, hd), dtype=f32).astype(np.float16)
        self.Vc = rng.standard_normal((B, nh, L + 1, hd), dtype=f32).astype(np.float16)
        self.x = rng.standard_normal((B, H), dtype=f32)
        self.cos, self.sin = R.rope_tables(L + 1, hd)
        self.pos = np.full(B, L, dtype=np.int64)
        self.B, self.c0, self.nh, self.hd, self.Hq, self.L = B, c0, nh, hd, Hq, L
        self.S, self.n_layers = S, n_layers
        self.sample = (f"1 of {n_layers} layers + LM head of one decode step (B={B}, KV {L}, "
                       f"fp32 numpy" + (f", 1/{S} of the heads/FF/vocab columns, x{S}" if S > 1
                                        else "") + f"); step time = layer x {n_layers} + head")
        self.run()  # warm-up (page-in, BLAS init)

    def _layer(self, x):
        B, c0, nh, hd, Hq, L, f32 = self.B, self.c0, self.nh, self.hd, self.Hq, self.L, np.float32
        layer = self.layer
        h = np.concatenate([R.rms_norm(x[:c0], layer["ln1"][0], 1e-5),
                            R.rms_norm(x[c0:], layer["ln1"][1], 1e-5)]).astype(f32)
        qkv = R.routed_gemm(h, layer["W_qkv"], c0)
        q = R.apply_rope(qkv[:, :Hq].reshape(B, nh, hd), self.pos, self.cos, self.sin).astype(f32)
        k = R.apply_rope(qkv[:, Hq:2 * Hq].reshape(B, nh, hd), self.pos, self.cos, self.sin)
        v = qkv[:, 2 * Hq:].reshape(B, nh, hd)
        out = np.empty((B, nh, hd), f32)
        for j in range(B):
            Kj = self.K[j].astype(f32)
            Vj = self.Vc[j].astype(f32)
            Kj[:, L] = k[j]
            Vj[:, L] = v[j]
            out[j] = R.sdpa(q[j][:, None, :], Kj, Vj)[:, 0, :]
        x = x + R.routed_gemm(out.reshape(B, Hq), layer["W_o"], c0)
        h = np.concatenate([R.rms_norm(x[:c0], layer["ln2"][0], 1e-5),
                            R.rms_norm(x[c0:], layer["ln2"][1], 1e-5)]).astype(f32)
        a = R.swiglu(R.routed_gemm(h, layer["W_gu"], c0)).astype(f32)
        return (x + R.routed_gemm(a, layer["W_d"], c0)).astype(f32)

    def _head(self, x):
        c0 = self.c0
        h = np.concatenate([R.rms_norm(x[:c0], self.lnf[0], 1e-5),
                            R.rms_norm(x[c0:], self.lnf[1], 1e-5)]).astype(np.float32)
        return R.routed_gemm(h, self.W_lm, c0).argmax(axis=-1)

    def run(self) -> dict:
        t0 = time.perf_counter()
        y = self._layer(self.x)
        t_layer = (time.perf_counter() - t0) * self.S
        t0 = time.perf_counter()
        self._head(y)
        t_head = (time.perf_counter() - t0) * self.S
        t_step = t_layer * self.n_layers + t_head
        return dict(t_layer=t_layer, t_head=t_head, t_step=t_step, tokens_per_s=self.B / t_step,
                    threads=blas_threads(), sample=self.sample)
