"""Tensor-parallel sharding on CPU ranks (gloo, world size 2, 4 and 8).

Each rank shards the full weights with the GPU decoder's own sharding
functions (parallel_serve_b200.decoder.shard_columns / shard_rows) and runs
the sharded decode step restated on CPU (oracle/tp_ref.py) with real gloo
all-reduce / all-gather; rank 0 checks that the logits and greedy tokens equal
the unsharded oracle step. Also checks that a rank that dies is seen by the
others as a collective error within the process-group timeout (no hang).
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(n_layers, H, FF, V, seed):
    g = torch.Generator().manual_seed(seed)

    def r(*s, std=0.05):
        return torch.randn(*s, generator=g, dtype=torch.float64) * std
    layers = [dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF), W_d=r(2, FF, H),
                   ln1=1 + r(2, H, std=0.1), ln2=1 + r(2, H, std=0.1)) for _ in range(n_layers)]
    return dict(layers=layers, emb=r(2, V, H, std=1.0), ln_f=1 + r(2, H, std=0.1), W_lm=r(2, H, V))


def _worker(rank, world, port, cfg, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import oracle
        from oracle import tp_ref
        from parallel_serve_b200.decoder import shard_columns, shard_rows
        n_layers, H, nh, FF, V, L0, ids = cfg
        w = _weights(n_layers, H, FF, V, 0)
        shard = dict(
            layers=[dict(W_qkv=shard_columns(L["W_qkv"], world, rank, 3).numpy(),
                         W_o=shard_rows(L["W_o"], world, rank).numpy(),
                         W_gu=shard_columns(L["W_gu"], world, rank, 2).numpy(),
                         W_d=shard_rows(L["W_d"], world, rank).numpy(),
                         ln1=L["ln1"].numpy(), ln2=L["ln2"].numpy()) for L in w["layers"]],
            emb=w["emb"].numpy(), ln_f=w["ln_f"].numpy(),
            W_lm=shard_columns(w["W_lm"], world, rank, 1).numpy())
        full = dict(layers=[{k: v.numpy() for k, v in L.items()} for L in w["layers"]],
                    emb=w["emb"].numpy(), ln_f=w["ln_f"].numpy(), W_lm=w["W_lm"].numpy())
        B = len(ids)
        c = (ids.count(0), ids.count(1))
        L_cap = L0 + 4
        nhl = nh // world
        st_full = oracle.DecodeState(n_layers, c, nh, L_cap)
        st_shard = oracle.DecodeState(n_layers, c, nhl, L_cap)
        rng = np.random.default_rng(3)
        for li in range(n_layers):
            for m in range(2):
                kk = rng.standard_normal(st_full.k[li][m].shape)
                vv = rng.standard_normal(st_full.v[li][m].shape)
                st_full.k[li][m][:] = kk
                st_full.v[li][m][:] = vv
                st_shard.k[li][m][:] = kk[:, rank * nhl:(rank + 1) * nhl]
                st_shard.v[li][m][:] = vv[:, rank * nhl:(rank + 1) * nhl]
        cos, sin = oracle.rope_tables(L_cap)
        tokens = np.array([(5 * i + 1) % V for i in range(B)])
        seq_a = np.full(B, L0)
        seq_b = np.full(B, L0)
        ok = True
        for _ in range(2):
            nxt_tp, _ = tp_ref.tp_decode_step(tokens, np.array(ids), shard, st_shard, seq_a, nhl,
                                              cos, sin, 1e-5, rank, world, V // world)
            nxt_ref, _ = oracle.decode_step(tokens, np.array(ids), full, st_full, seq_b, nh, cos,
                                            sin, 1e-5)
            ok = ok and np.array_equal(nxt_tp, nxt_ref)
            tokens = nxt_ref
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_sharded_step_equals_unsharded(world):
    if world == 8:      # 1 head and 216 FF columns per rank, as one rank's FF tail at TP 8
        cfg = (1, 1024, 8, 1728, 64, 6, [0, 1, 1, 0, 1, 0])
    else:
        cfg = (2, 512, 4, 256, 64, 6, [0, 1, 1, 0, 1])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert all(res[r] for r in range(world)), res
    assert all(p.exitcode == 0 for p in procs)


@pytest.mark.parametrize("H,nh,FF,tp", [(4096, 32, 11008, t) for t in (2, 4, 8)] +
                         [(5120, 40, 13824, t) for t in (2, 4, 8)])
def test_shards_partition_llama_layers_exactly(H, nh, FF, tp):
    """Llama-7B and -13B layers at TP 2/4/8: each rank's QKV shard holds whole
    heads (its q, k and v columns of heads [r*nh/tp, (r+1)*nh/tp)), its gate_up
    shard the same FF range of gate and of up, its O / down shards the matching
    rows; over all ranks every column (row) is taken exactly once. Weights are
    coded by index, so the check is exact."""
    from parallel_serve_b200.decoder import shard_columns, shard_rows
    hl, ffl = nh // tp * 128, FF // tp
    qkv = torch.arange(3 * H, dtype=torch.float64).expand(2, 1, 3 * H)
    gu = torch.arange(2 * FF, dtype=torch.float64).expand(2, 1, 2 * FF)
    seen_qkv, seen_gu, seen_o, seen_d = [], [], [], []
    for r in range(tp):
        q = shard_columns(qkv, tp, r, 3)[0, 0].long()
        assert q.numel() == 3 * hl
        for g in range(3):              # q | k | v blocks, heads r*nh/tp ..
            assert torch.equal(q[g * hl:(g + 1) * hl], torch.arange(hl) + g * H + r * hl)
        g_u = shard_columns(gu, tp, r, 2)[0, 0].long()
        assert torch.equal(g_u[:ffl], torch.arange(ffl) + r * ffl)
        assert torch.equal(g_u[ffl:], torch.arange(ffl) + FF + r * ffl)
        o = shard_rows(torch.arange(H, dtype=torch.float64).view(1, H, 1).expand(2, H, 1), tp, r)
        d = shard_rows(torch.arange(FF, dtype=torch.float64).view(1, FF, 1).expand(2, FF, 1), tp, r)
        assert torch.equal(o[0, :, 0].long(), torch.arange(hl) + r * hl)     # rows of its heads
        assert torch.equal(d[0, :, 0].long(), torch.arange(ffl) + r * ffl)   # rows of its FF
        seen_qkv.append(q)
        seen_gu.append(g_u)
        seen_o.append(o[0, :, 0].long())
        seen_d.append(d[0, :, 0].long())
    for seen, n in ((seen_qkv, 3 * H), (seen_gu, 2 * FF), (seen_o, H), (seen_d, FF)):
        assert torch.equal(torch.cat(seen).sort().values, torch.arange(n))


def _dying_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    t = torch.ones(4)
    dist.all_reduce(t)                       # one good step
    if rank == 1:
        os._exit(3)                          # this rank dies between steps
    try:
        dist.all_reduce(t)                   # the survivor's next collective must fail, not hang
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__))


def test_dead_rank_is_detected_by_collective_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    rank, what = q.get(timeout=10)
    assert rank == 0 and what != "no error"
    assert procs[1].exitcode == 3
