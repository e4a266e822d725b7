#!/usr/bin/env python
"""Fused two-model Llama-7B-shape decode benchmark (tokens/s) on B200.

Workload (one "step"): one greedy decode step of two co-located 32-layer
Llama-7B-shape models (hidden 4096, 32 heads x 128, SwiGLU 11008, vocab
32000, fp16, random-init N(0, 0.02) weights) for 64 sequences split 32/32
between the models, each with a synthetic fp16 KV history of 2048 positions
(N(0, 1)) that grows by one per step. Every projection is one routed GEMM over
both models' tokens, attention is one fused decode kernel over both models'
KV pools, and the whole step replays as one CUDA graph. The per-step working
set (~95 GB of weights + KV) is far larger than L2, so no flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (launched by torchrun, one rank per GPU) the step is
tensor-parallel over NCCL: column-split QKV / gate_up, row-split O / down with
an all-reduce after each, vocab-split LM head. ``value`` is the whole job's
tokens/s (64 tokens per step / the max-over-ranks step time).

``--impl reference`` times the reference's serial per-model path restated on
the CPU (the oracle), on the host cores, as a bounded sample per step.

``--shape llama13b`` measures the large-batch Llama-13B-shape workload
instead (hidden 5120, 40 heads, FF 13824, 40 layers, 256 sequences per model
over 4096 KV positions). Its KV caches (44 GB per layer at one GPU) exceed
the memory of 8 GPUs at full depth, so when they do not fit, layers share KV
pool sets (``--kv-layers``): every layer still moves a full history's bytes,
the line's config says how many sets there were.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# model shapes: hidden, heads (x 128), SwiGLU width, vocabulary, layers, and the
# workload each is measured on (model-0/model-1 sequences, KV positions)
SHAPES = {
    "llama7b": dict(H=4096, heads=32, ff=11008, vocab=32000, layers=32, split="32/32", kv=2048,
                    name="Llama-7B"),
    "llama13b": dict(H=5120, heads=40, ff=13824, vocab=32000, layers=40, split="256/256",
                     kv=4096, name="Llama-13B"),
}
H, N_HEADS, FF, VOCAB, N_LAYERS = 4096, 32, 11008, 32000, 32
METRIC = "2-model decode tokens/s (Llama-7B shape, B=64)"


def apply_shape(args):
    """Fill the shape's dimensions and its workload defaults into the module
    constants and the unset arguments."""
    global H, N_HEADS, FF, VOCAB, N_LAYERS, METRIC
    sh = SHAPES[args.shape]
    H, N_HEADS, FF, VOCAB, N_LAYERS = sh["H"], sh["heads"], sh["ff"], sh["vocab"], sh["layers"]
    args.split = args.split or sh["split"]
    args.kv_len = args.kv_len or sh["kv"]
    args.layers = args.layers or N_LAYERS
    B = sum(split_counts(args.split))
    METRIC = f"2-model decode tokens/s ({sh['name']} shape, B={B})"
    args.shape_name = sh["name"]
    return args


def parse():
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--shape", choices=sorted(SHAPES), default="llama7b",
                   help="model shape; llama13b: hidden 5120, 40 heads, FF 13824, 40 layers, "
                        "256/256 sequences over 4096 KV positions")
    p.add_argument("--split", default=None,
                   help="model-0/model-1 sequences, e.g. 48/16 (default: the shape's)")
    p.add_argument("--kv-len", type=int, default=0, help="KV positions (default: the shape's)")
    p.add_argument("--layers", type=int, default=0, help="layers (default: the shape's)")
    p.add_argument("--kv-layers", type=int, default=0,
                   help="distinct KV pool sets, layer i using set i %% n (0: one per layer "
                        "when they fit in memory, else as many as fit)")
    p.add_argument("--no-serial", action="store_true", help="skip the serial same-kernel baseline")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    p.add_argument("--no-sweep", action="store_true",
                   help="skip the 48/16 and 56/8 split sweep (timed by default at N=1)")
    p.add_argument("--no-extra", action="store_true",
                   help="skip the single-routed-linear and DeltaZip blocks (timed by default "
                        "at N=1)")
    p.add_argument("--chain", action="store_true",
                   help="one projection chain launch per layer (O, gate_up, down, next QKV, "
                        "and the all-reduces under tensor parallelism) instead of one launch "
                        "per projection")
    p.add_argument("--no-gate", action="store_true",
                   help="skip the oracle parity gate before timing (the line then says so)")
    p.add_argument("--prefill-len", type=int, default=0,
                   help="also time a prefill of this many prompt tokens per sequence")
    p.add_argument("--prefill-chunk", type=int, default=1024,
                   help="prompt tokens per routed prefill launch")
    p.add_argument("--page-size", type=int, default=0,
                   help="paged KV cache with this page size (0: contiguous per-sequence caches)")
    p.add_argument("--allreduce", choices=["nvlink", "nvlink1", "nvlink2", "nvlink-ll", "nccl"],
                   default="nvlink",
                   help="collective for the row-split outputs under tensor parallelism")
    return apply_shape(p.parse_args())


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def split_counts(split: str) -> tuple[int, int]:
    a, b = (int(v) for v in split.split("/"))
    return a, b


def model_ids(c0: int, c1: int):
    """Interleave the two models' sequences over the batch (model 0 first where
    they differ), so the routed order is a real permutation."""
    ids = []
    a, b = c0, c1
    while a or b:
        if a:
            ids.append(0)
            a -= 1
        if b:
            ids.append(1)
            b -= 1
    return ids


# --------------------------------------------------------------- clocks ----
class ClockSampler:
    """SM clocks and clock-event reasons of the job's GPUs over the timed
    regions. NVML is read every 20 ms from a thread (a timed region at 8 GPUs
    can be shorter than nvidia-smi's start-up plus one sampling period);
    nvidia-smi's sampling loop is the fallback. Reading clocks changes no
    setting of the GPU. `nvml` replaces the NVML module (tests)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40))
    PERIOD_S = 0.02

    def __init__(self, nvml=None):
        self.proc = None
        self.mode = None
        self._nvml = nvml
        self.path = os.path.join("/tmp", f"ps_clocks_{os.getpid()}.csv")

    def _start_nvml(self) -> bool:
        import threading
        nv = self._nvml
        if nv is None:
            try:
                import pynvml as nv
            except Exception:
                return False
        try:
            nv.nvmlInit()
            handles = [nv.nvmlDeviceGetHandleByIndex(i) for i in range(nv.nvmlDeviceGetCount())]
            reasons_of = (getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None)
                          or nv.nvmlDeviceGetCurrentClocksThrottleReasons)
            sm_clock = getattr(nv, "NVML_CLOCK_SM", 1)
        except Exception:
            return False
        self._nv, self._samples, self._stop = nv, [], threading.Event()

        def loop():
            while True:
                for i, h in enumerate(handles):
                    try:
                        self._samples.append((i, float(nv.nvmlDeviceGetClockInfo(h, sm_clock)),
                                              float(nv.nvmlDeviceGetMaxClockInfo(h, sm_clock)),
                                              int(reasons_of(h))))
                    except Exception:
                        pass
                if self._stop.wait(self.PERIOD_S):
                    return
        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        self.mode = "nvml"
        return True

    def start(self):
        if self._start_nvml():
            return
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
            self.mode = "nvidia-smi"
        except Exception:
            self.proc = None

    @staticmethod
    def physical(indices):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if not vis:
            return indices
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        try:
            return {int(ids[i]) for i in indices if i < len(ids)}
        except ValueError:
            return None

    @staticmethod
    def _summary(sm, smax, reasons, source) -> dict:
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons), "source": source}

    def stop(self, gpu_indices=None) -> dict:
        if gpu_indices is not None:
            gpu_indices = self.physical(gpu_indices)
        if self.mode == "nvml":
            self._stop.set()
            self._thread.join(timeout=5)
            try:
                self._nv.nvmlShutdown()
            except Exception:
                pass
            sm, smax, reasons = [], [], set()
            for idx, clk, mx, mask in list(self._samples):
                if gpu_indices is not None and idx not in gpu_indices:
                    continue
                sm.append(clk)
                smax.append(mx)
                reasons.update(n for n, bit in self.REASONS if mask & bit)
            return self._summary(sm, smax, reasons, "nvml")
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    idx = int(parts[0])
                except ValueError:
                    continue
                if gpu_indices is not None and idx not in gpu_indices:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return self._summary(sm, smax, reasons, "nvidia-smi")


def workload_config(args, world: int, kv_layers: int | None = None) -> dict:
    """The line's `config`: the same dict for this arm and the reference arm."""
    c0, c1 = split_counts(args.split)
    B = c0 + c1
    cfg = {"workload": f"two-model {args.shape_name}-shape greedy decode, "
                       f"{args.layers} layers, B={B} ({args.split}), KV {args.kv_len}+, "
                       "CUDA graph per step",
           "global_batch": B, "seq_len": args.kv_len, "split": args.split,
           "parallelism": f"tp{world}",
           "kv_layout": (f"paged, {args.page_size}-position pages" if args.page_size
                         else "contiguous per sequence"),
           "l2": "working set per step >> L2 (weights + KV of all layers), no flush",
           "projections": ("one projection chain launch per layer" if getattr(args, "chain", False)
                           else "one launch per projection")}
    if kv_layers is not None and kv_layers < args.layers:
        cfg["kv_layers"] = (f"{kv_layers} KV pool sets shared by {args.layers} layers "
                            "(same bytes per layer; caches aliased to fit memory)")
    return cfg


def use_all_host_cores() -> int:
    """BLAS threads = the cores this process may run on. torchrun exports
    OMP_NUM_THREADS=1 for its ranks, which would leave the CPU reference on one
    core; the reference arm runs on rank 0 alone, so it takes them all. Call
    before numpy is imported (OpenBLAS reads the variables once)."""
    n = host_cores()
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = str(n)
    return n


# ------------------------------------------------------------ reference ----
def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    cores = use_all_host_cores()
    from threadpoolctl import threadpool_limits
    from oracle.cpu_baseline import DecodeSample
    c0, c1 = split_counts(args.split)
    B = c0 + c1
    # Size the per-step sample so that warm-up + K steps end within ~2 minutes:
    # 1/S of each layer's heads / FF / vocabulary columns, time x S.
    with threadpool_limits(limits=cores):
        probe = DecodeSample(B, c0, H, N_HEADS, FF, VOCAB, args.kv_len, args.layers,
                             slice_factor=16)
        per_full_step = probe.run()["t_layer"]  # time of one full layer
        del probe
        budget = 120.0 / max(1, args.steps + args.warmup)
        S = 1
        while S < 32 and per_full_step / S > budget:
            S *= 2
        sample = DecodeSample(B, c0, H, N_HEADS, FF, VOCAB, args.kv_len, args.layers,
                              slice_factor=S)
        times = []
        for i in range(args.warmup + args.steps):
            r = sample.run()
            if i >= args.warmup:
                times.append(r["t_step"])
    t = statistics.mean(times)
    value = B / t
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": r["threads"],
                         "kind": "port",
                         "sample": r["sample"] + f"; host CPU, {r['threads']} BLAS threads of "
                                                 f"{os.cpu_count()} cores (ms_per_step is that "
                                                 "extrapolated step)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- ours ----
def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    world, rank, local_rank = dist_env()
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
        group = dist.group.WORLD
    from parallel_serve_b200 import _lib
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder

    c0, c1 = split_counts(args.split)
    B = c0 + c1
    K, W = args.steps, args.warmup
    cfg = DecoderConfig(n_layers=args.layers, hidden=H, n_heads=N_HEADS, ffn=FF, vocab=VOCAB)
    L_cap = args.kv_len + W + K + 8
    ids = model_ids(c0, c1)
    peak, peak_kind = peaks()

    # Correctness first: no number is printed for a step that fails the gate.
    gate = None
    if not args.no_gate:
        gate = parity_gate(args, cfg, ids, group, world, rank, device, torch)
        if not gate["ok"]:
            if rank == 0:
                print(json.dumps({"metric": METRIC, "value": None, "unit": "tokens/s",
                                  "n_gpus": world, "error": "parity gate failed",
                                  "parity": gate}), flush=True)
            if world > 1:
                dist.barrier()
                dist.destroy_process_group()
            return 1
    kv_layers = args.kv_layers or kv_sets_that_fit(cfg, B, L_cap, world, args.page_size, torch,
                                                   device)
    dec = TwoModelDecoder(cfg, ids, L_cap, device=device, tp_group=group, seed=0,
                          allreduce=args.allreduce, page_size=args.page_size or None,
                          prefill_chunk=args.prefill_chunk, kv_layers=kv_layers,
                          chain=args.chain)
    g = torch.Generator().manual_seed(0)
    prompt_tok = torch.randint(0, VOCAB, (B,), generator=g, dtype=torch.int32)

    def reset():
        if reset.first:
            dec.fill_kv_random(args.kv_len, seed=1)
        else:
            dec.reset_lengths(args.kv_len)
        dec.reserve(W + K + 2)       # paged KV: pages for every step of a timed run
        reset.first = False
        dec.tokens.copy_(prompt_tok.to(device))
    reset.first = True

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # eager warm-up step (sets kernel attributes, checks status), then capture
    reset()
    dec.step_device("fused")
    torch.cuda.synchronize()
    dec.check_status()
    dec.capture("fused")
    if not args.no_serial:
        dec.step_device("serial")
        dec.capture("serial")
    barrier()

    def timed(mode: str) -> float:
        reset()
        for _ in range(W):
            dec.replay(mode)
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(K):
            dec.replay(mode)
        e.record()
        barrier()
        return max_over_ranks(s.elapsed_time(e) / 1e3)

    clocks = ClockSampler()
    if rank == 0:
        clocks.start()
    t_fused = timed("fused")
    dec.check_status()
    value = B * K / t_fused

    t_serial = timed("serial") if not args.no_serial else None

    # e2e: public host-buffer API (pinned H2D of the step's token ids, D2H of the picks)
    reset()
    tok_host = prompt_tok.clone().pin_memory()
    out_host = torch.empty(B, dtype=torch.int32).pin_memory()
    for _ in range(W):
        dec.step(tok_host, out_host)
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(K):
        dec.step(tok_host, out_host)
        tok_host.copy_(out_host)
    e.record()
    barrier()
    t_e2e = max_over_ranks(s.elapsed_time(e) / 1e3)

    # Clocks were sampled from the start of the fused timing through the e2e
    # loop (the timed regions), on the GPUs this job uses.
    clk = clocks.stop(gpu_indices=set(range(world))) if rank == 0 else None

    # --- per-kernel-class timing (same launches as the step, replayed alone) ---
    kinfo = kernel_rooflines(dec, torch, W, peak, barrier, max_over_ranks, t_fused / K)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        from threadpoolctl import threadpool_limits
        from oracle.cpu_baseline import DecodeSample
        with threadpool_limits(limits=host_cores()):
            r = DecodeSample(B, c0, H, N_HEADS, FF, VOCAB, args.kv_len, args.layers,
                             slice_factor=4).run()
        cpu = {"value": r["tokens_per_s"], "unit": "tokens/s", "cores": r["threads"],
               "kind": "port", "sample": r["sample"]}

    launches_per_step = dec.launches_per_step()
    dom = max((k for k in kinfo if "achieved_gbs" in kinfo[k]),
              key=lambda k: kinfo[k]["time_share"])
    roof = dict(kinfo[dom])
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": t_fused / K * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": workload_config(args, world, kv_layers),
        "parity": gate if gate is not None else "not run (--no-gate)",
        "e2e": {"value": B * K / t_e2e, "unit": "tokens/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B},
        "gpu_launches": launches_per_step * K,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": roof["achieved_gbs"],
                     "peak": peak, "unit": "GB/s", "frac": roof["achieved_gbs"] / peak,
                     "traffic": traffic_for(dom, roof["bytes_per_launch"]),
                     "peak_kind": peak_kind},
        "kernels": {k: {kk: vv for kk, vv in v.items()} for k, v in kinfo.items()},
        "clocks": clk,
    }
    if t_serial is not None:
        line["serial_same_kernels"] = {"value": B * K / t_serial, "unit": "tokens/s",
                                       "ms_per_step": t_serial / K * 1e3,
                                       "fused_over_serial": t_serial / t_fused}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if args.prefill_len > 0:
        # routed prefill of B prompts (random tokens) through the public API,
        # host arrays and their copies included; after the decode timings
        # because it rewrites the caches
        P = min(args.prefill_len, L_cap - 1)
        gp = torch.Generator().manual_seed(11)
        prompts = [torch.randint(0, VOCAB, (P,), generator=gp).tolist() for _ in range(B)]
        dec.prefill(prompts)
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        dec.prefill(prompts)
        e.record()
        barrier()
        t_pf = max_over_ranks(s.elapsed_time(e) / 1e3)
        line["prefill"] = {"value": B * P / t_pf, "unit": "prompt tokens/s", "ms": t_pf * 1e3,
                           "prompt_len": P, "sequences": B, "chunk_tokens": args.prefill_chunk}
        dec.check_status()
    dec.close()
    if world == 1 and not (args.no_sweep and args.no_extra):
        del dec
        torch.cuda.empty_cache()
    if world == 1 and not args.no_sweep and args.shape == "llama7b":
        line["split_sweep"] = {sp: split_tokens_per_s(cfg, sp, args, device, torch)
                               for sp in ("48/16", "56/8")}
    if world == 1 and not args.no_extra:
        line["routed_linear_cfg1"] = routed_linear_cfg1(torch, device, peak)
        line["deltazip"] = deltazip_table(torch, device, peak)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


GATE_LAYERS, GATE_KV, GATE_TOL = 2, 128, 1e-2


def parity_gate(args, cfg_full, ids, group, world, rank, device, torch) -> dict:
    """Correctness gate run before any timing, on this job's own tensor-parallel
    group: a 2-layer decoder with the bench's hidden size, heads per rank, FF,
    vocabulary, batch and split, the same collective (NVLink all-reduce) and the
    same vocab-split greedy pick, runs ONE captured decode step over a 128-position
    KV history; rank 0 gathers every rank's logits and compares them (and the
    picks) with the oracle's decode step (fp32 numpy on the host cores) on the
    identical weights and caches. Every rank takes the same collective steps.
    Follows the reference's one-layer fused-vs-serial gate before its timings
    (experiments/split_sweep_cudagraph.py:98-128), held to the 1e-2 tolerance."""
    import numpy as np
    import torch.distributed as dist
    from parallel_serve_b200.decoder import DecoderConfig, TwoModelDecoder
    H, nh, FFd, V = cfg_full.hidden, cfg_full.n_heads, cfg_full.ffn, cfg_full.vocab
    B = len(ids)
    if B > 128:      # the large-batch shape: gate a 64-sequence batch with the same ratio
        c0 = round(64 * sum(1 for m in ids if m == 0) / B)
        ids = model_ids(c0, 64 - c0)
        B = 64
    cfg = DecoderConfig(n_layers=GATE_LAYERS, hidden=H, n_heads=nh, ffn=FFd, vocab=V)
    L0, L_cap = GATE_KV, GATE_KV + 8
    # Identical full weights on every rank: one seeded device generator (the same
    # Philox stream on every GPU), sharded by the decoder.
    g = torch.Generator(device=device).manual_seed(1234)

    def rnd(*shape, std=0.02, mean=0.0):
        return torch.empty(*shape, dtype=torch.float16, device=device).normal_(mean, std,
                                                                               generator=g)
    w = dict(layers=[dict(W_qkv=rnd(2, H, 3 * H), W_o=rnd(2, H, H), W_gu=rnd(2, H, 2 * FFd),
                          W_d=rnd(2, FFd, H), ln1=rnd(2, H, std=0.1, mean=1.0),
                          ln2=rnd(2, H, std=0.1, mean=1.0)) for _ in range(GATE_LAYERS)],
             emb=rnd(2, V, H, std=1.0), ln_f=rnd(2, H, std=0.1, mean=1.0), W_lm=rnd(2, H, V))
    c0 = sum(1 for m in ids if m == 0)
    slots = (c0, B - c0)
    kv = [[(rnd(s, nh, L0, 128, std=1.0), rnd(s, nh, L0, 128, std=1.0)) if s else None
           for s in slots] for _ in range(GATE_LAYERS)]
    tokens = torch.randint(0, V, (B,), generator=torch.Generator().manual_seed(5),
                           dtype=torch.int32)
    dec = TwoModelDecoder(cfg, ids, L_cap, device=device, tp_group=group, weights=w,
                          allreduce=args.allreduce, page_size=args.page_size or None,
                          chain=args.chain)
    nl = dec.nh
    hs = slice(rank * nl, (rank + 1) * nl)

    def load_state():
        for li in range(GATE_LAYERS):
            for m in range(2):
                if kv[li][m] is not None:
                    k, v = kv[li][m]
                    dec.write_kv(li, m, k[:, hs].contiguous(), v[:, hs].contiguous())
        dec.set_state(tokens, torch.full((B,), L0, dtype=torch.int32))
    load_state()
    dec.step_device("fused")          # eager warm-up (kernel attributes, NCCL)
    torch.cuda.synchronize()
    load_state()
    dec.capture("fused")
    dec.replay("fused")               # the one captured step that is checked
    torch.cuda.synchronize()
    status = _lib_status(device)
    logits = dec.logits.contiguous()
    if world > 1:
        parts = [torch.empty_like(logits) for _ in range(world)]
        dist.all_gather(parts, logits, group=group)
        logits = torch.cat(parts, dim=1)
    picks = dec.next_tokens.clone()
    dec.close()
    out = {}
    if rank == 0:
        import oracle
        from threadpoolctl import threadpool_limits
        f32 = lambda t: t.float().cpu().numpy()  # noqa: E731
        P = dict(layers=[{k: f32(v) for k, v in L.items()} for L in w["layers"]],
                 emb=f32(w["emb"]), ln_f=f32(w["ln_f"]), W_lm=f32(w["W_lm"]))
        st = oracle.DecodeState(GATE_LAYERS, slots, nh, L_cap, dt=np.float32)
        for li in range(GATE_LAYERS):
            for m in range(2):
                if kv[li][m] is not None:
                    st.k[li][m][:, :, :L0] = f32(kv[li][m][0])
                    st.v[li][m][:, :, :L0] = f32(kv[li][m][1])
        cos, sin = oracle.rope_tables(L_cap)
        with threadpool_limits(limits=host_cores()):
            nxt, ref = oracle.decode_step(tokens.numpy().astype(np.int64), np.array(ids), P, st,
                                          np.full(B, L0), nh, cos, sin, float(cfg.eps))
        got = logits.double().cpu().numpy()
        err = oracle.rel_err(got, ref)
        top2 = np.sort(ref, axis=1)[:, -2:]
        gap = top2[:, 1] - top2[:, 0]
        clear = gap > 0.02 * np.abs(ref).mean()       # margin far above the logits' error
        # picks are in original batch order, ref rows in routed order
        perm = np.argsort(np.array(ids), kind="stable")
        got_picks = picks.cpu().numpy()[perm]
        ref_picks = ref.argmax(axis=1)
        match = int((got_picks[clear] == ref_picks[clear]).sum())
        ok = bool(err < GATE_TOL and match == int(clear.sum()) and status == 0)
        out = {"ok": ok, "rel_err": err, "tol": GATE_TOL, "picks_checked": int(clear.sum()),
               "picks_equal": match, "status": status,
               "case": (f"{GATE_LAYERS} layers, B={B} ({c0}/{B - c0}), KV {L0}, hidden {H}, "
                        f"{nl} heads per rank, FF {FFd}, vocab {V}, one captured step, "
                        f"tp{world} {args.allreduce if world > 1 else ''}").strip(),
               "oracle": "oracle.decode_step, fp32 numpy on the host cores"}
    flag = torch.tensor([1 if (rank != 0 or out.get("ok")) else 0], device=device)
    if world > 1:
        dist.broadcast(flag, 0, group=group)
    del dec, w, kv
    torch.cuda.empty_cache()
    out["ok"] = bool(flag.item())
    return out


def _lib_status(device) -> int:
    from parallel_serve_b200 import _lib
    return _lib.read_status(device)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def rotating_graph_time(torch, launches, reps=3):
    """Per-launch time of a list of launch closures (distinct weight sets, so
    no launch finds its weights in L2), captured as one CUDA graph and replayed
    `reps` times after a warm-up, CUDA events on the capturing stream."""
    for fn in launches:
        fn()
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for fn in launches:
            fn()
    gr.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        gr.replay()
    e.record()
    torch.cuda.synchronize()
    t = s.elapsed_time(e) / 1e3 / (reps * len(launches))
    del gr
    return t


def routed_linear_cfg1(torch, device, peak) -> dict:
    """The single routed linear: W [2, 4096, 4096] fp16 N(0, 0.02), 32 tokens
    N(0, 1), model_id[i] = i % 2 (16 tokens per model, interleaved). Timed two
    ways, each over 8 distinct weight sets (537 MB > L2) in one CUDA graph:
    the GEMM on tokens already in routed order (device counts), and the whole
    routed call (device partition, gather, GEMM with row scatter back)."""
    from parallel_serve_b200 import ops
    K = N = 4096
    M, sets = 32, 8
    g = torch.Generator(device=device).manual_seed(7)
    Ws = [torch.empty(2, K, N, dtype=torch.float16, device=device).normal_(0, 0.02, generator=g)
          for _ in range(sets)]
    x = torch.empty(M, K, dtype=torch.float16, device=device).normal_(0, 1, generator=g)
    ids = (torch.arange(M, dtype=torch.int32, device=device) % 2)
    ys = [torch.empty(M, N, dtype=torch.float16, device=device) for _ in range(sets)]
    ws = ops.gemm_workspace(device, M, N, 0)
    perm, counts = ops.route_partition(ids)
    xp = ops.gather_rows(x, perm)
    t_gemm = rotating_graph_time(torch, [
        (lambda W=W, y=y: ops.routed_gemm_raw(xp, W, y, counts=counts, workspace=ws))
        for W, y in zip(Ws, ys)])

    def full(W, y):
        p, c = ops.route_partition(ids)
        ops.gather_rows(x, p, out=xp)
        ops.routed_gemm_raw(xp, W, y, counts=c, scatter=p, workspace=ws)
    t_full = rotating_graph_time(torch, [(lambda W=W, y=y: full(W, y)) for W, y in zip(Ws, ys)])
    alg = 2 * K * N * 2 + 2 * M * K * 2 + M * N * 2
    return {"workload": "W [2,4096,4096] fp16, 32 tokens, model_id = i % 2",
            "gemm_us": t_gemm * 1e6, "gemm_gbs": alg / t_gemm / 1e9,
            "gemm_frac_of_peak": alg / t_gemm / 1e9 / peak,
            "routed_call_us": t_full * 1e6, "routed_call_gbs": alg / t_full / 1e9,
            "bytes_per_call": alg, "l2": "8 distinct weight sets rotated (537 MB > L2)"}


def deltazip_table(torch, device, peak) -> dict:
    """Route-A DeltaZip linear (base fp16 + int4 2:4 delta, all rows policy rows)
    on the Llama-7B projection shapes at M = 1, 16, 64, beside the routed GEMM
    reading the base weights alone (one model) on the same shape. Six distinct
    weight sets per shape (>= 200 MB) rotate through one CUDA graph."""
    from parallel_serve_b200 import deltazip as dzp, ops
    from parallel_serve_b200._lib import check, lib, ptr
    from parallel_serve_b200 import _lib
    out = {}
    sets = 6
    for K, N in ((4096, 4096), (4096, 11008), (11008, 4096)):
        g = torch.Generator(device=device).manual_seed(K + N)
        Wb = [torch.empty(K, N, dtype=torch.float16, device=device).normal_(0, 0.02, generator=g)
              for _ in range(sets)]
        D = torch.empty(K, N, dtype=torch.float32, device=device).normal_(0, 0.002, generator=g)
        q, keep, sc = dzp.quantize_delta(D)
        pk = dzp.pack_delta(q, keep, sc)
        del D, q, keep, sc
        packs = [pk] + [pk.clone() for _ in range(sets - 1)]
        dz_bytes = pk.numel()
        row = {}
        for M in (1, 16, 64):
            x = torch.empty(M, K, dtype=torch.float16, device=device).normal_(0, 1, generator=g)
            ys = [torch.empty(M, N, dtype=torch.float16, device=device) for _ in range(sets)]
            dws = torch.zeros(lib.ps_deltazip_workspace_bytes(M, N, device.index or 0),
                              dtype=torch.uint8, device=device)
            st = _lib.status_tensor(device)

            def dz(W, P, y, x=x, M=M, dws=dws):
                check(lib.ps_deltazip_linear(ptr(x), ptr(W), ptr(P), ptr(y), M, K, N, 0, None,
                                             _lib.PS_DTYPE_F16, ptr(dws), dws.numel(), ptr(st),
                                             _lib.stream_handle(device)), "ps_deltazip_linear")
            t_dz = rotating_graph_time(torch, [(lambda W=W, P=P, y=y: dz(W, P, y))
                                               for W, P, y in zip(Wb, packs, ys)])
            gws = ops.gemm_workspace(device, M, N, 0)
            t_b = rotating_graph_time(torch, [
                (lambda W=W, y=y, x=x, M=M, gws=gws:
                 ops.routed_gemm_raw(x, W, y, split_point=M, workspace=gws))
                for W, y in zip(Wb, ys)])
            a_dz = K * N * 2 + dz_bytes + M * (K + N) * 2
            a_b = K * N * 2 + M * (K + N) * 2
            row[str(M)] = {"deltazip_us": t_dz * 1e6, "deltazip_gbs": a_dz / t_dz / 1e9,
                           "deltazip_frac_of_peak": a_dz / t_dz / 1e9 / peak,
                           "base_gemm_us": t_b * 1e6, "base_gemm_gbs": a_b / t_b / 1e9,
                           "deltazip_over_base": t_dz / t_b}
        out[f"{K}x{N}"] = row
        del Wb, packs, pk
        torch.cuda.empty_cache()
    if _lib.read_status(device):
        raise RuntimeError("DeltaZip timing raised device status bits")
    return {"shapes": out, "bytes": "W_base 2KN + packed delta 0.406KN + x, y",
            "parity": "unpinned against the reference's Marlin-24 kernel (source absent); "
                      "pinned to the dense-dequant oracle by the GPU tests"}


def kv_sets_that_fit(cfg, B, L_cap, world, page_size, torch, device) -> int:
    """One KV pool set per layer when weights + all sets fit in this GPU's free
    memory with 8 GB to spare, else as many sets as fit (at least 1)."""
    nh, FFl, Vl = cfg.n_heads // world, cfg.ffn // world, cfg.vocab // world
    Hl, Hd = nh * 128, cfg.hidden
    weights = 2 * 2 * (cfg.n_layers * (Hd * 3 * Hl + Hl * Hd + Hd * 2 * FFl + FFl * Hd)
                       + Hd * Vl + cfg.vocab * Hd)
    if page_size:
        L_cap = -(-L_cap // page_size) * page_size
    per_set = B * nh * L_cap * 128 * 2 * 2
    free = torch.cuda.mem_get_info(device)[0]
    fit = int((free - weights - 8e9) // per_set)
    return max(1, min(cfg.n_layers, fit))


def traffic_for(kernel: str, alg_bytes: float):
    """DRAM bytes per launch from the committed ncu summary (profiles/traffic.json),
    scaled by algorithmic bytes when this launch processes a different amount
    of work than the captured one; None when no capture exists."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            rec = json.load(f).get(kernel)
        return rec["dram_bytes"] * alg_bytes / rec["alg_bytes"]
    except Exception:
        return None


def kernel_rooflines(dec, torch, W, peak, barrier, max_over_ranks, t_step) -> dict:
    """Time each kernel class of the step alone (same launches, same buffers,
    CUDA graph, CUDA events on the launch stream) and convert to achieved GB/s
    from algorithmic bytes. Under tensor parallelism the row-split outputs'
    all-reduces are a class of their own; `other` is the rest of the measured
    step time (`t_step`, seconds): partition, positions, embedding, greedy pick,
    the copy of the picks, and launch boundaries."""
    from parallel_serve_b200 import _lib, ops
    B, L = dec.B, dec.L_cap
    esz = 2
    c0, c1 = dec.counts_host
    models = (1 if c0 else 0) + (1 if c1 else 0)
    H, Hl, FFl, Vl = dec.cfg.hidden, dec.Hl, dec.FFl, dec.Vl
    seq = int(dec.seq_len[0].item())

    def graph_time(fn, reps=5):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        for _ in range(2):
            gr.replay()
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            gr.replay()
        e.record()
        barrier()
        t = max_over_ranks(s.elapsed_time(e) / 1e3) / reps
        del gr
        return t

    counts = dec.counts
    bt = None if dec.block_table is None else dec.block_table.device
    eps = float(dec.cfg.eps)
    STORE, SWIGLU, QKV = _lib.PS_EPI_STORE, _lib.PS_EPI_SWIGLU, _lib.PS_EPI_QKV_ROPE
    tp1 = dec.tp == 1

    # routed GEMMs: 4 per layer + LM head, with the step's epilogues (outputs
    # of the residual projections go to a scratch buffer)
    def gemms():
        if dec.fused:
            for li, Lw in enumerate(dec.layers):
                e = ops.gemm_epilogue(QKV, in_sumsq=dec.sq_a, norm_dim=H, eps=eps,
                                      k_pools=tuple(dec.kpool[li]), v_pools=tuple(dec.vpool[li]),
                                      pos=dec.pos, rope_cos=dec.rope_cos, rope_sin=dec.rope_sin,
                                      n_heads=dec.nh, block_table=bt)
                dec._gemm_ex(dec.x, Lw["W_qkv"], dec.q, counts, e)
                e = ops.gemm_epilogue(STORE, residual=dec.x_alt if tp1 else None,
                                      out_sumsq=dec.sq_b if tp1 else None)
                dec._gemm_ex(dec.attn, Lw["W_o"], dec.x_alt, counts, e)
                e = ops.gemm_epilogue(SWIGLU, in_sumsq=dec.sq_b, norm_dim=H, eps=eps)
                dec._gemm_ex(dec.x, Lw["W_gu"], dec.a, counts, e)
                e = ops.gemm_epilogue(STORE, residual=dec.x_alt if tp1 else None,
                                      out_sumsq=dec.sq_a if tp1 else None)
                dec._gemm_ex(dec.a, Lw["W_d"], dec.x_alt, counts, e)
            e = ops.gemm_epilogue(STORE, in_sumsq=dec.sq_a, norm_dim=H, eps=eps)
            dec._gemm_ex(dec.x, dec.W_lm, dec.logits, counts, e)
            return
        for Lw in dec.layers:
            dec._gemm(dec.h, Lw["W_qkv"], dec.qkv, counts)
            dec._gemm(dec.attn, Lw["W_o"], dec.x_alt, counts)
            dec._gemm(dec.h, Lw["W_gu"], dec.a, counts, epilogue=_lib.PS_EPI_SWIGLU)
            dec._gemm(dec.a, Lw["W_d"], dec.x_alt, counts)
        dec._gemm(dec.h, dec.W_lm, dec.logits, counts)
    n_gemm = 4 * len(dec.layers) + 1
    wbytes = models * esz * (len(dec.layers) * (H * 3 * Hl + Hl * H + H * 2 * FFl + FFl * H) + H * Vl)
    # activations per layer: x -> q,k,v; attn -> (+residual) x; x -> a; a -> (+residual) x
    res = 2 * H if (dec.fused and dec.tp == 1) else 0
    abytes = B * esz * (len(dec.layers) * (H + 3 * Hl + Hl + H + H + FFl + FFl + H + res) + H + Vl)
    chain = dec.use_chain and bool(dec.layers)
    if chain:
        # the step's own projection launches: layer 0's QKV and one chain per
        # layer (O, gate_up, down, next QKV / LM head and, under tensor
        # parallelism, the fused all-reduces), over a scratch residual stream
        n_gemm = 1 + len(dec.layers)
        t_g = graph_time(lambda: dec._layers_chain(slice(0, B), counts, attention=False,
                                                   xbuf=dec.x_alt))
    else:
        t_g = graph_time(gemms)


    def attns():   # the step's own attention launches (contiguous or paged KV)
        for li in range(len(dec.layers)):
            dec._attention(dec.q, tuple(dec.kpool[li]), tuple(dec.vpool[li]), dec.attn, dec.pos,
                           counts, bt)
    pos_mean = float(dec.pos.float().mean().item()) + 1.0
    kvbytes = len(dec.layers) * B * dec.nh * pos_mean * 128 * esz * 2
    qbytes = len(dec.layers) * B * Hl * esz * 2
    t_a = graph_time(attns)
    t_ar, n_ar = 0.0, 0
    if dec.tp > 1 and dec.ar is not None and not chain:
        def allreduces():   # the step's own all-reduce launches (2 per layer)
            for li in range(len(dec.layers)):
                for sq in (dec.sq_b, dec.sq_a):
                    slot = dec._slot
                    dec._slot ^= 1
                    dec.ar(slot, dec.x.numel(), dec.x, residual=dec.x, out_sumsq=sq)
        n_ar = 2 * len(dec.layers)
        t_ar = graph_time(allreduces)
    t_other = max(0.0, t_step - t_g - t_a - t_ar)
    t_step_est = t_g + t_a + t_ar + t_other
    extra = {}
    if n_ar:
        nbytes = dec.x.numel() * esz
        extra["allreduce"] = {"launches": n_ar, "avg_launch_us": t_ar / n_ar * 1e6,
                              "message_bytes": nbytes, "us_per_step": t_ar * 1e6,
                              "time_share": t_ar / t_step_est,
                              "kind": "one-shot NVLink peer all-reduce (+ residual, sums of "
                                      "squares)"}
    extra["other"] = {"us_per_step": t_other * 1e6, "time_share": t_other / t_step_est,
                      "what": "partition, positions, embedding, greedy pick"
                              + (" (vocab-split exchange)" if dec.tp > 1 else "")
                              + ", token copy, launch boundaries: step time minus the classes "
                                "above, each timed alone"}
    gname = "projection_chain" if chain else "routed_gemm"
    ginfo = {"launches": n_gemm, "avg_launch_us": t_g / n_gemm * 1e6,
             "bytes_per_launch": (wbytes + abytes) / n_gemm,
             "achieved_gbs": (wbytes + abytes) / t_g / 1e9,
             "frac_of_peak": (wbytes + abytes) / t_g / 1e9 / peak,
             "time_share": t_g / t_step_est, "us_per_step": t_g * 1e6}
    if chain:
        ginfo["what"] = ("layer 0's QKV GEMM + one persistent chain per layer: O, gate_up, down, "
                         "next QKV or LM head" + (", NVLink all-reduce of O and down"
                                                  if dec.tp > 1 else "")
                         + "; bytes = weights + activations")
    return extra | {
        gname: ginfo,
        "decode_attention": {"launches": len(dec.layers),
                             "avg_launch_us": t_a / len(dec.layers) * 1e6,
                             "bytes_per_launch": (kvbytes + qbytes) / len(dec.layers),
                             "achieved_gbs": (kvbytes + qbytes) / t_a / 1e9,
                             "frac_of_peak": (kvbytes + qbytes) / t_a / 1e9 / peak,
                             "time_share": t_a / t_step_est, "us_per_step": t_a * 1e6},
    }


def split_tokens_per_s(cfg, split, args, device, torch) -> dict:
    """Tokens/s of the fused and serial steps at another split (1 GPU)."""
    from parallel_serve_b200.decoder import TwoModelDecoder
    c0, c1 = split_counts(split)
    B = c0 + c1
    K, W = min(args.steps, 32), args.warmup
    dec = TwoModelDecoder(cfg, model_ids(c0, c1), args.kv_len + W + K + 8, device=device)
    dec.fill_kv_random(args.kv_len, seed=1)
    out = {}
    for mode in ("fused", "serial"):
        dec.step_device(mode)
        dec.capture(mode)
        dec.seq_len.fill_(args.kv_len)
        for _ in range(W):
            dec.replay(mode)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(K):
            dec.replay(mode)
        e.record()
        torch.cuda.synchronize()
        out[mode] = B * K / (s.elapsed_time(e) / 1e3)
        out[f"{mode}_ms_per_step"] = s.elapsed_time(e) / K
    dec.check_status()
    dec.release_graphs()
    out["fused_over_serial"] = out["fused"] / out["serial"]
    out["unit"] = "tokens/s"
    del dec
    torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    sys.exit(main())
