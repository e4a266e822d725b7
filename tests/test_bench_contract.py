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
