"""GPU decode with real-layout weights: two HF Llama models packed by the
loader drive TwoModelDecoder (fp16, fused epilogues, optionally paged KV) from
HF's own prompt caches; its logits must match transformers' Llama (float32,
CPU) continuing the same sequences, rel < 1e-2."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytest.importorskip("transformers")
pytestmark = pytest.mark.gpu

from conftest import rel_err, to_np  # noqa: E402
from hf_llama_pair import CFG, make_model, prefill, step  # noqa: E402


@pytest.mark.parametrize("page_size", [None, 16])
def test_decoder_matches_transformers_llama(page_size):
    import oracle
    from parallel_serve_b200.decoder import TwoModelDecoder
    from parallel_serve_b200.loader import decoder_config_from_hf, pack_hf_llama
    models = (make_model(0), make_model(1))
    cfg = decoder_config_from_hf(CFG)
    w = pack_hf_llama(models[0].state_dict(), models[1].state_dict())
    ids = [1, 0, 1, 1, 0, 0]
    L0, L_cap = 9, 32
    dec = TwoModelDecoder(cfg, ids, L_cap, weights=w, page_size=page_size)
    perm, counts = oracle.route_partition(np.array(ids))
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 384, (L0,), generator=g) for _ in ids]
    hist = {m: [[None] * int(counts[m]) for _ in range(cfg.n_layers)] for m in range(2)}
    caches = {}
    for j in range(len(ids)):
        s = int(perm[j])
        m = ids[s]
        kv, caches[s] = prefill(models[m], prompts[s])
        sl = j - (0 if m == 0 else int(counts[0]))
        for li, (k, v) in enumerate(kv):
            hist[m][li][sl] = (k, v)
    tokens = np.array([23 * (i + 3) % 384 for i in range(len(ids))])
    dec.set_state(torch.from_numpy(tokens), torch.full((len(ids),), L0))
    dec.reserve(4)
    for m in range(2):
        for li in range(cfg.n_layers):
            k = torch.stack([kv[0] for kv in hist[m][li]]).half().cuda()
            v = torch.stack([kv[1] for kv in hist[m][li]]).half().cuda()
            dec.write_kv(li, m, k, v)
    for _ in range(3):
        dec.step_device("fused")
        torch.cuda.synchronize()
        lg = to_np(dec.logits)
        ref = np.stack([step(models[ids[int(perm[j])]], caches[int(perm[j])],
                             int(tokens[int(perm[j])])).double().numpy() for j in range(len(ids))])
        assert rel_err(lg, ref) < 1e-2
        nxt = np.empty(len(ids), dtype=np.int64)
        nxt[perm] = ref.argmax(-1)
        tokens = nxt                        # continue both on the reference's greedy picks
        dec.tokens.copy_(torch.from_numpy(tokens).to(torch.int32))
    dec.check_status()
