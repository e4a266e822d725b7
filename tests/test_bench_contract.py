"""bench.py's command-line contract, on the CPU: each model shape's workload
defaults, and the reference arm's single JSON line (the oracle's restatement
of the reference's serial torch path, timed on the host cores)."""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)


def _shape(name, **kw):
    import bench
    ns = argparse.Namespace(shape=name, split=kw.get("split"), kv_len=kw.get("kv_len", 0),
                            layers=kw.get("layers", 0))
    return bench, bench.apply_shape(ns)


def test_shape_defaults_and_overrides():
    bench, a = _shape("llama13b")
    assert (bench.H, bench.N_HEADS, bench.FF, bench.VOCAB) == (5120, 40, 13824, 32000)
    assert (a.split, a.kv_len, a.layers) == ("256/256", 4096, 40)
    assert bench.METRIC == "2-model decode tokens/s (Llama-13B shape, B=512)"
    bench, a = _shape("llama7b", split="48/16", kv_len=1024)
    assert (bench.H, bench.N_HEADS, bench.FF) == (4096, 32, 11008)
    assert (a.split, a.kv_len, a.layers) == ("48/16", 1024, 32)
    assert bench.METRIC == "2-model decode tokens/s (Llama-7B shape, B=64)"
    assert bench.model_ids(3, 1) == [0, 1, 0, 0]


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--layers", "1", "--kv-len", "64"],
                       cwd=ROOT, capture_output=True, text=True, timeout=900,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


class _FakeNvml:
    """Two GPUs: GPU 0 at 1800 of 1965 MHz under the power cap, GPU 1 idle at
    max; reads only (the sampler changes no GPU setting)."""
    NVML_CLOCK_SM = 1

    def __init__(self):
        self.calls = []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetCount(self):
        return 2

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetClockInfo(self, h, kind):
        assert kind == self.NVML_CLOCK_SM
        return 1800 if h == 0 else 1965

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return 0x4 if h == 0 else 0x1          # sw_power_cap / GPU idle


def test_clock_sampler_reads_nvml_during_the_timed_region(monkeypatch):
    import time
    import bench
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    fake = _FakeNvml()
    c = bench.ClockSampler(nvml=fake)
    c.start()
    time.sleep(0.1)                              # a timed region shorter than 200 ms
    got = c.stop(gpu_indices={0})
    assert got["source"] == "nvml" and got["samples"] >= 2
    assert got["sm_mhz"] == 1800 and got["sm_max_mhz"] == 1965
    assert got["reasons"] == ["sw_power_cap"]
    assert fake.calls == ["init", "shutdown"]
    # CUDA_VISIBLE_DEVICES maps the job's device 0 to physical GPU 1
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "1")
    c = bench.ClockSampler(nvml=_FakeNvml())
    c.start()
    time.sleep(0.05)
    got = c.stop(gpu_indices={0})
    assert got["sm_mhz"] == 1965 and got["reasons"] == []
