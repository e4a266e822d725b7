"""Host bookkeeping of the paged KV cache (CPU): page allocation, block tables
and the oracle's page gather."""
from __future__ import annotations

import numpy as np
import pytest


def test_allocator_hands_out_each_page_once():
    from parallel_serve_b200.paged_kv import PageAllocator
    a = PageAllocator(10, shuffle_seed=3)
    got = a.alloc(4) + a.alloc(6)
    assert sorted(got) == list(range(10)) and got != list(range(10))
    with pytest.raises(MemoryError):
        a.alloc(1)
    a.release(got[:3])
    assert a.n_free == 3 and sorted(a.alloc(3)) == sorted(got[:3])
    with pytest.raises(ValueError):
        a.release([10])


def test_block_table_grows_per_model_pool():
    from parallel_serve_b200.paged_kv import BlockTable, PageAllocator
    alloc = (PageAllocator(8), PageAllocator(8, shuffle_seed=1))
    bt = BlockTable([0, 0, 1], alloc, max_pages=4, page_size=16)
    bt.ensure(range(3), 17)                      # 2 pages each
    assert bt.host[:, :2].min() >= 0 and (bt.host[:, 2:] == -1).all()
    assert len(set(bt.pages_of(0)) | set(bt.pages_of(1))) == 4       # model 0 pages distinct
    assert alloc[0].n_free == 4 and alloc[1].n_free == 6
    bt.ensure([2], 64)
    assert len(bt.pages_of(2)) == 4 and bt.pages_of(2)[:2] == bt.host[2, :2].tolist()
    with pytest.raises(ValueError):
        bt.ensure([0], 65)                       # beyond max_pages * page_size
    bt.release([2])
    assert alloc[1].n_free == 8 and (bt.host[2] == -1).all()
    bt.sync()
    assert bt.device.tolist() == bt.host.tolist()


def test_gather_pages_restates_the_layout():
    import oracle
    rng = np.random.default_rng(0)
    ps, heads, d = 4, 2, 3
    pool = rng.standard_normal((6, heads, ps, d))
    row = [5, 0, 3]
    hist = oracle.gather_pages(pool, row, ps, 10)
    assert hist.shape == (heads, 10, d)
    assert np.array_equal(hist[:, 4:8], pool[0]) and np.array_equal(hist[:, 8:10], pool[3][:, :2])
    assert oracle.gather_pages(pool, row, ps, 0).shape == (heads, 0, d)


def test_prefill_layout_chunks_keep_routing_and_causality():
    """The routed prefill's host layout: model-0 tokens first in every chunk,
    positions in order per sequence, KV rows and last-token picks right,
    whatever the chunk size."""
    from parallel_serve_b200.decoder import prefill_layout
    prompts = [[5, 6, 7], [1], [9, 9, 9, 9, 9], [2, 3]]        # original order
    ids = np.array([1, 0, 1, 0])
    perm = np.argsort(ids, kind="stable")                      # routed J -> sequence
    c0 = int((ids == 0).sum())
    for chunk in (1, 2, 3, 4, 7, 64):
        for paged in (False, True):
            chunks = prefill_layout(prompts, perm, c0, chunk, paged)
            toks = [t for ch in chunks for t in ch["tok"]]
            assert toks == [t for J in perm for t in prompts[J]]
            poss = [p for ch in chunks for p in ch["pos"]]
            assert poss == [p for J in perm for p in range(len(prompts[J]))]
            assert all(len(ch["tok"]) <= chunk for ch in chunks)
            seen_last = {}
            for ch in chunks:
                for i, J in ch["last"]:
                    seen_last[J] = (ch["pos"][i], ch["kv_rows"][i])
            assert sorted(seen_last) == list(range(len(perm)))
            for J, (p, r) in seen_last.items():
                assert p == len(prompts[perm[J]]) - 1
                assert r == (J if paged else (J - c0 if J >= c0 else J))
            # the model-0 count of each chunk matches the routed order
            pos_model = [0 if J < c0 else 1 for J in range(len(perm)) for _ in prompts[perm[J]]]
            start = 0
            for ch in chunks:
                n = len(ch["tok"])
                assert ch["n0"] == pos_model[start:start + n].count(0)
                start += n
