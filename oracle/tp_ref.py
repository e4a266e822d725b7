"""Tensor-parallel decode step restated on CPU (test infrastructure only).

Mirrors the sharded dataflow of the GPU decoder for one rank of a
`torch.distributed` group (gloo on CPU): replicated RMSNorm, column-split QKV
(each rank: its heads' slices of q, k and v) and gate_up (its FF slice of gate
and of up), attention over the rank's heads with its share of the KV cache,
row-split O and down producing partial sums that an all-reduce combines
(rank 0 contributes the residual), vocabulary-split LM head with a
(max logit, global index) all-gather for the greedy pick. The unsharded
reference for the same math is ``ref_ops.decode_step``
(experiments/two_model_block.py:54-74 plus the KV-cache decode).
"""
from __future__ import annotations

import numpy as np
import torch

from . import ref_ops as R


def _allreduce(a: np.ndarray, group) -> np.ndarray:
    import torch.distributed as dist
    t = torch.from_numpy(np.ascontiguousarray(a))
    dist.all_reduce(t, group=group)
    return t.numpy()


def _allgather(a: np.ndarray, world: int, group) -> np.ndarray:
    import torch.distributed as dist
    t = torch.from_numpy(np.ascontiguousarray(a))
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t, group=group)
    return np.stack([o.numpy() for o in out])


def tp_decode_step(tokens, model_id, shard: dict, kv_shard: R.DecodeState, seq_len, n_heads_local,
                   cos, sin, eps, rank: int, world: int, vocab_local: int, group=None):
    """One greedy step on this rank. ``shard`` holds the rank's weight shards
    (same keys as ref_ops.decode_step params); returns (next_tokens, logits shard)."""
    perm, counts = R.route_partition(model_id)
    c0 = int(counts[0])
    B = len(perm)
    m = (np.arange(B) >= c0).astype(np.int64)
    x = shard["emb"][m, tokens[perm]]
    pos = seq_len[perm].astype(np.int64)
    nh = n_heads_local
    Hl = nh * 128
    for li, w in enumerate(shard["layers"]):
        h = np.concatenate([R.rms_norm(x[:c0], w["ln1"][0], eps), R.rms_norm(x[c0:], w["ln1"][1], eps)])
        qkv = R.routed_gemm(h, w["W_qkv"], c0)
        q = R.apply_rope(qkv[:, :Hl].reshape(B, nh, 128), pos, cos, sin)
        k = R.apply_rope(qkv[:, Hl:2 * Hl].reshape(B, nh, 128), pos, cos, sin)
        v = qkv[:, 2 * Hl:].reshape(B, nh, 128)
        Lmax = int(pos.max()) + 1
        Kc = np.zeros((B, nh, Lmax, 128))
        Vc = np.zeros((B, nh, Lmax, 128))
        for j in range(B):
            mj = 0 if j < c0 else 1
            sl = j - (0 if mj == 0 else c0)
            kv_shard.k[li][mj][sl, :, pos[j]] = k[j]
            kv_shard.v[li][mj][sl, :, pos[j]] = v[j]
            Kc[j] = kv_shard.k[li][mj][sl, :, :Lmax]
            Vc[j] = kv_shard.v[li][mj][sl, :, :Lmax]
        attn = R.decode_attention(q, Kc, Vc, pos + 1).reshape(B, Hl)
        part = R.routed_gemm(attn, w["W_o"], c0) + (x if rank == 0 else 0.0)
        x = _allreduce(part, group)
        h = np.concatenate([R.rms_norm(x[:c0], w["ln2"][0], eps), R.rms_norm(x[c0:], w["ln2"][1], eps)])
        a = R.swiglu(R.routed_gemm(h, w["W_gu"], c0))
        part = R.routed_gemm(a, w["W_d"], c0) + (x if rank == 0 else 0.0)
        x = _allreduce(part, group)
    lnf = shard["ln_f"]
    h = np.concatenate([R.rms_norm(x[:c0], lnf[0], eps), R.rms_norm(x[c0:], lnf[1], eps)])
    logits = R.routed_gemm(h, shard["W_lm"], c0)
    best = np.stack([logits.max(axis=-1), logits.argmax(axis=-1) + rank * vocab_local], axis=-1)
    allb = _allgather(best, world, group)              # [world, B, 2]
    r = allb[:, :, 0].argmax(axis=0)                     # first rank on ties = lowest index
    pick = allb[r, np.arange(B), 1].astype(np.int64)
    nxt = np.empty(B, dtype=np.int64)
    nxt[perm] = pick
    seq_len += 1
    return nxt, logits
