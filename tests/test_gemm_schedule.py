"""The routed GEMM's tile schedule, checked on the CPU through the library's
schedule-introspection entry points, which run the kernel's own schedule
functions (sched_from_counts, seg_range, tile_of, the stream-K fix-up
bookkeeping) on the host.

For every shape and grid size:
* each (tile, k-block) iteration is worked by exactly one CTA;
* split tiles occur only in the stream-K part. Their contributors are exactly
  the CTA range the last-arriving CTA sums, and each contributor's partial
  slot is the one that CTA's fix-up reads. No CTA puts two tiles in one slot;
* tiles cover each model's tokens once per weight tile, and never mix the
  two models;
* with several token tiles per model and data-parallel rounds, the token
  tiles of one weight tile run in the same round (weights read once).
"""
from __future__ import annotations

import ctypes
import random

import numpy as np
import pytest

GRIDS = (148, 147, 132, 7, 1)


def _lib():
    from parallel_serve_b200 import _lib
    return _lib.lib


def _sched(L, c0, c1, K, N, epi, grid):
    info = (ctypes.c_int32 * 10)()
    assert L.ps_routed_gemm_schedule(c0, c1, K, N, epi, grid, info) == 0
    keys = ("T0", "T1", "nt", "ntiles", "KB", "I", "C", "R", "base", "grid")
    return dict(zip(keys, list(info)))


def _work(L, c0, c1, K, N, epi, grid, cta):
    n = L.ps_routed_gemm_cta_work(c0, c1, K, N, epi, grid, cta, None, 0)
    assert n >= 0
    buf = (ctypes.c_int32 * (6 * max(n, 1)))()
    assert L.ps_routed_gemm_cta_work(c0, c1, K, N, epi, grid, cta, buf, n) == n
    return np.frombuffer(buf, dtype=np.int32)[:6 * n].reshape(n, 6)


def _tile(L, c0, c1, K, N, epi, grid, t):
    out = (ctypes.c_int32 * 6)()
    assert L.ps_routed_gemm_tile(c0, c1, K, N, epi, grid, t, out) == 0
    return list(out)


def _check(c0, c1, K, N, epi, grid):
    L = _lib()
    s = _sched(L, c0, c1, K, N, epi, grid)
    KB, I = s["KB"], s["I"]
    seen = np.zeros(I, dtype=np.int32)
    contrib: dict[int, list] = {}
    round_of: dict[int, int] = {}
    for b in range(grid):
        slots = {}
        for t, kb0, kb1, slot, bf, bl in _work(L, c0, c1, K, N, epi, grid, b):
            seen[t * KB + kb0:t * KB + kb1] += 1
            if slot < 0:
                assert (kb0, kb1) == (0, KB)
                if t < s["R"] * grid:
                    assert t % grid == b           # data-parallel: tile b + r * grid
                    round_of[t] = t // grid
            else:
                assert t >= s["R"] * grid and not (kb0 == 0 and kb1 == KB)
                assert slot not in slots, (b, slot, t)
                slots[slot] = t
                contrib.setdefault(t, []).append((b, slot, kb1 - kb0, bf, bl))
    assert (seen == 1).all()
    for t, lst in contrib.items():
        assert sum(x[2] for x in lst) == KB
        bf, bl = lst[0][3], lst[0][4]
        assert all((x[3], x[4]) == (bf, bl) for x in lst)
        assert sorted(x[0] for x in lst) == list(range(bf, bl + 1))
    # tiles: each model's tokens once per weight tile, models never mixed
    if s["ntiles"]:
        rows = {}
        for t in range(s["ntiles"]):
            m, row0, ntok, col0, col1, out0 = _tile(L, c0, c1, K, N, epi, grid, t)
            lo, hi = (0, c0) if m == 0 else (c0, c0 + c1)
            assert lo <= row0 and row0 + ntok <= hi and 0 < ntok <= 128
            rows.setdefault((m, out0), []).append((row0, ntok))
        for (m, _), lst in rows.items():
            lst.sort()
            assert sum(n for _, n in lst) == (c0 if m == 0 else c1)
            assert all(lst[i][0] + lst[i][1] == lst[i + 1][0] for i in range(len(lst) - 1))
        # weights read once: a weight tile's token tiles share a data-parallel round
        s["pairs_checked"] = 0
        if s["R"] and s["T0"] == 2 and s["T1"] in (0, 2) and grid % 2 == 0:
            for t, r in round_of.items():
                partner = t ^ 1                    # token tiles 0 / 1 of one weight tile
                if partner in round_of:
                    assert round_of[partner] == r
                    s["pairs_checked"] += 1
    return s


CASES = [  # (c0, c1, K, N, epilogue)  decode, 13B, prefill-chunk and edge shapes
    (32, 32, 4096, 12288, 0), (32, 32, 4096, 4096, 0), (32, 32, 4096, 22016, 1),
    (32, 32, 11008, 4096, 0), (48, 16, 4096, 32000, 0), (256, 256, 5120, 15360, 0),
    (256, 256, 5120, 27648, 1), (256, 256, 13824, 5120, 0), (512, 512, 4096, 12288, 0),
    (700, 324, 4096, 22016, 1), (1024, 0, 11008, 4096, 0), (0, 1024, 4096, 4096, 0),
    (300, 0, 128, 256, 0), (129, 1, 5120, 1920, 0), (1, 0, 64, 128, 0), (0, 0, 64, 128, 0),
]


@pytest.mark.parametrize("case", CASES)
def test_schedule_invariants(case):
    for grid in GRIDS:
        _check(*case, grid)


def test_schedule_invariants_random_shapes():
    rng = random.Random(0)
    for _ in range(150):
        epi = 1 if rng.random() < 0.3 else 0
        N = 16 * rng.randint(1, 900) if epi else 8 * rng.randint(1, 1800)
        _check(rng.randint(0, 1100), rng.randint(0, 1100), 8 * rng.randint(1, 1500), N, epi,
               rng.choice(GRIDS))


def test_decode_keeps_pure_stream_k_and_large_batches_get_rounds():
    L = _lib()
    assert _sched(L, 32, 32, 4096, 12288, 0, 148)["R"] == 0
    s = _sched(L, 256, 256, 5120, 15360, 0, 148)
    assert (s["T0"], s["T1"], s["ntiles"], s["R"]) == (2, 2, 480, 3)
    assert _check(256, 256, 5120, 15360, 0, 148)["pairs_checked"] == 3 * 148


def test_schedule_entry_points_reject_bad_arguments():
    L = _lib()
    info = (ctypes.c_int32 * 10)()
    assert L.ps_routed_gemm_schedule(-1, 4, 64, 128, 0, 148, info) != 0
    assert L.ps_routed_gemm_schedule(4, 4, 64, 130, 0, 148, info) != 0     # N % 8
    assert L.ps_routed_gemm_schedule(4, 4, 64, 136, 1, 148, info) != 0     # SwiGLU N % 16
    assert L.ps_routed_gemm_schedule(4, 4, 64, 128, 0, 0, info) != 0       # grid
    assert L.ps_routed_gemm_cta_work(4, 4, 64, 128, 0, 148, 148, None, 0) < 0
    out = (ctypes.c_int32 * 6)()
    assert L.ps_routed_gemm_tile(4, 4, 64, 128, 0, 148, 2, out) != 0        # only tiles 0, 1
