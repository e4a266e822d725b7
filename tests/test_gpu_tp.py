"""Tensor-parallel decode on 2 GPUs against the single-process oracle.

Spawns one process per GPU; each builds the TwoModelDecoder shard of the same
seeded weights, runs two greedy steps (eager, then CUDA-graph replay) with the
row-split outputs summed by the NVLink peer-memory all-reduce, by NCCL, or by
the all-reduce jobs of the projection chain (one launch per layer), and
compares its logits slice (rel < 1e-2) and clear-margin greedy picks with
oracle.decode_step; with the NVLink all-reduce it then runs a paged routed
prefill and compares the last-token logits with oracle.prefill. The all-reduce itself is checked against a CPU sum over
eight calls (alternating slots, one-shot and two-shot), for bit-identical
results on both ranks, and for its per-row sums of squares (the folded
RMSNorm's input).
Skipped when fewer than 2 GPUs are visible.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, allreduce="nvlink"):
    import sys
    chain = allreduce.endswith("+chain")      # projection chains with the fused all-reduce
    allreduce = allreduce.replace("+chain", "")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        import oracle
        from conftest import rel_err, to_np
        from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
        n_layers, H, nh, FF, V, L0 = 2, 512, 4, 512, 256, 20
        ids = [0, 1, 0, 1, 1, 1]
        g = torch.Generator().manual_seed(0)

        def r(*s, std=0.02):
            return (torch.randn(*s, generator=g) * std).to(torch.float16)
        w = dict(layers=[dict(W_qkv=r(2, H, 3 * H), W_o=r(2, H, H), W_gu=r(2, H, 2 * FF),
                              W_d=r(2, FF, H), ln1=1 + r(2, H, std=0.1), ln2=1 + r(2, H, std=0.1))
                         for _ in range(n_layers)],
                 emb=r(2, V, H, std=1.0), ln_f=1 + r(2, H, std=0.1), W_lm=r(2, H, V))
        cfg = DecoderConfig(n_layers=n_layers, hidden=H, n_heads=nh, ffn=FF, vocab=V)
        L_cap = L0 + 4
        dec = TwoModelDecoder(cfg, ids, L_cap, device=dev, weights=w, tp_group=dist.group.WORLD,
                              allreduce=allreduce, chain=chain)
        assert dec.use_chain == chain
        c = (ids.count(0), ids.count(1))
        st = oracle.DecodeState(n_layers, c, nh, L_cap)
        gk = torch.Generator().manual_seed(1)
        nhl = nh // world
        for li in range(n_layers):
            for m in range(2):
                kk = torch.randn(c[m], nh, L_cap, 128, generator=gk).to(torch.float16)
                vv = torch.randn(c[m], nh, L_cap, 128, generator=gk).to(torch.float16)
                dec.kpool[li][m].copy_(kk[:, rank * nhl:(rank + 1) * nhl])
                dec.vpool[li][m].copy_(vv[:, rank * nhl:(rank + 1) * nhl])
                st.k[li][m][:] = to_np(kk)
                st.v[li][m][:] = to_np(vv)
        tokens = np.array([3, 50, 7, 99, 250, 1])
        seq = np.full(len(ids), L0)
        dec.set_state(torch.from_numpy(tokens), torch.from_numpy(seq))
        P = dict(layers=[{k: to_np(v) for k, v in L.items()} for L in w["layers"]],
                 emb=to_np(w["emb"]), ln_f=to_np(w["ln_f"]), W_lm=to_np(w["W_lm"]))
        cos, sin = oracle.rope_tables(L_cap)
        ok = True
        for step in range(2):
            if step == 0:
                dec.step_device("fused")
                saved = dec.seq_len.clone()
            else:
                dec.capture("fused")          # capture rewrites state: restore and replay
                dec.seq_len.copy_(saved)
                dec.tokens.copy_(torch.from_numpy(tokens).to(torch.int32))
                dec.replay("fused")
            torch.cuda.synchronize()
            nxt_ref, logits_ref = oracle.decode_step(tokens, np.array(ids), P, st, seq, nh, cos,
                                                     sin, 1e-5)
            lg = to_np(dec.logits)                       # this rank's vocab slice
            Vl = V // world
            e = rel_err(lg, logits_ref[:, rank * Vl:(rank + 1) * Vl])
            got = dec.next_tokens.cpu().numpy()
            srt = np.sort(logits_ref, axis=-1)
            clear = (srt[:, -1] - srt[:, -2]) > 0.05
            perm, _ = oracle.route_partition(np.array(ids))
            clear_orig = np.empty_like(clear)
            clear_orig[perm] = clear
            ok = ok and e < 1e-2 and np.array_equal(got[clear_orig], nxt_ref[clear_orig])
            tokens = nxt_ref
            dec.tokens.copy_(torch.from_numpy(tokens).to(torch.int32))
        dec.check_status()
        dec.close()
        if allreduce.startswith("nvlink"):
            # routed prefill under tensor parallelism (paged KV, chunks that
            # split sequences) against the oracle's teacher-forced prefill
            dec = TwoModelDecoder(cfg, ids, L_cap, device=dev, weights=w,
                                  tp_group=dist.group.WORLD, allreduce=allreduce, page_size=16,
                                  prefill_chunk=8)
            gp = torch.Generator().manual_seed(12)
            lens = [5, 3, 9, 1, 6, 4]
            prompts = [torch.randint(0, V, (n,), generator=gp).tolist() for n in lens]
            dec.prefill(prompts)
            torch.cuda.synchronize()
            st2 = oracle.DecodeState(n_layers, c, nh, L_cap)
            _, lref = oracle.prefill(prompts, np.array(ids), P, st2, nh, cos, sin, 1e-5)
            Vl = V // world
            ok = ok and rel_err(to_np(dec.logits), lref[:, rank * Vl:(rank + 1) * Vl]) < 1e-2
            dec.check_status()
            dec.close()
        q.put((rank, bool(ok)))
    except Exception as ex:  # noqa: BLE001
        q.put((rank, repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("allreduce", ["nvlink", "nvlink2", "nvlink-ll", "nccl", "nvlink+chain"])
def test_tp2_decode_matches_oracle(allreduce):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, allreduce)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert all(res[r] is True for r in range(world)), res


def _ar_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from parallel_serve_b200 import _lib
        from parallel_serve_b200.tp import NvlinkAllReduce
        rows, H = 64, 4096
        count = rows * H
        ar = NvlinkAllReduce(dist.group.WORLD, count, dev, torch.float16)
        ident = torch.arange(rows, dtype=torch.int32, device=dev)
        ok = True
        algos = (_lib.PS_AR_ONE_SHOT, _lib.PS_AR_TWO_SHOT, _lib.PS_AR_TWO_SHOT_LL)
        for call in range(12):                     # alternating slots, repeated epochs
            ar.algo = algos[(call // 2) % 3]
            slot = call % 2
            parts = [torch.randn(rows, H, generator=torch.Generator().manual_seed(100 * call + r)
                                 ).to(torch.float16) for r in range(world)]
            res = torch.randn(rows, H, generator=torch.Generator().manual_seed(999 + call)
                              ).to(torch.float16)
            mine = parts[rank].to(dev)
            # place this rank's partial in its local slot with the library's row copy
            _lib.check(_lib.lib.ps_gather_rows(mine.data_ptr(), ident.data_ptr(), ar.slot_ptr(slot),
                                               rows, H * 2, None, _lib.stream_handle(dev)), "copy")
            out = res.to(dev)
            sq = torch.full((rows, H // 256), -1.0, device=dev)
            ar(slot, count, out, residual=out, out_sumsq=sq if call % 3 else None)
            torch.cuda.synchronize()
            ref = res.double() + sum(p.double() for p in parts)
            err = (out.double().cpu() - ref).abs().max().item()
            ok = ok and err < 2e-2 and _lib.read_status(dev) == 0
            if call % 3:   # per-256-element sums of squares of the stored rows
                want = (out.double() ** 2).reshape(rows, H // 256, 256).sum(-1)
                ok = ok and torch.allclose(sq.double(), want, rtol=1e-5)
        # every rank must hold bit-identical results
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        ok = ok and all(torch.equal(g, gathered[0]) for g in gathered)
        # the three algorithms add in the same order: bit-identical outputs and sums of squares
        outs = []
        for k, algo in enumerate(algos):
            ar.algo = algo
            slot = k % 2
            _lib.check(_lib.lib.ps_gather_rows(mine.data_ptr(), ident.data_ptr(), ar.slot_ptr(slot),
                                               rows, H * 2, None, _lib.stream_handle(dev)), "copy")
            o = res.to(dev)
            sq = torch.zeros(rows, H // 256, device=dev)
            ar(slot, count, o, residual=o, out_sumsq=sq)
            torch.cuda.synchronize()
            outs.append((o, sq))
        ok = ok and _lib.read_status(dev) == 0
        ok = ok and all(torch.equal(o, outs[0][0]) and torch.equal(sq, outs[0][1]) for o, sq in outs)
        torch.cuda.synchronize()
        dist.barrier()
        ar.close()
        q.put((rank, bool(ok)))
    except Exception as ex:  # noqa: BLE001
        q.put((rank, repr(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nvlink_allreduce_matches_sum():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    res = dict(q.get(timeout=10) for _ in range(world))
    assert all(res[r] is True for r in range(world)), res
