"""Loader parity on CPU: HF Llama state dicts -> stacked two-model weights, and
the oracle decode step on those weights against transformers' own Llama
(float32) continuing from the same prompt cache. This pins the oracle's RoPE
convention, cache attention and block order to an independent implementation
of the model family the reference serves (Llama-2-7B / Vicuna-7B)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytest.importorskip("transformers")

from hf_llama_pair import CFG, make_model, prefill, step  # noqa: E402


def test_pack_layout():
    from parallel_serve_b200.loader import decoder_config_from_hf, pack_hf_llama
    a, b = make_model(0), make_model(1)
    sa, sb = a.state_dict(), b.state_dict()
    w = pack_hf_llama(sa, sb, dtype=torch.float32)
    L = w["layers"][1]
    p = "model.layers.1."
    assert L["W_qkv"].shape == (2, 256, 768) and L["W_gu"].shape == (2, 256, 1024)
    assert torch.equal(L["W_qkv"][1][:, 256:512], sb[p + "self_attn.k_proj.weight"].t())
    assert torch.equal(L["W_gu"][0][:, 512:], sa[p + "mlp.up_proj.weight"].t())
    assert torch.equal(L["W_d"][0], sa[p + "mlp.down_proj.weight"].t())
    assert torch.equal(w["W_lm"][1], sb["lm_head.weight"].t())
    assert w["emb"].shape == (2, 384, 256) and w["W_lm"].is_contiguous()
    cfg = decoder_config_from_hf(CFG)
    assert (cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.ffn, cfg.vocab) == (2, 256, 2, 512, 384)
    with pytest.raises(ValueError):
        decoder_config_from_hf(dict(CFG, num_key_value_heads=1))


def test_oracle_decode_matches_transformers_llama():
    import oracle
    from parallel_serve_b200.loader import pack_hf_llama
    models = (make_model(0), make_model(1))
    w = pack_hf_llama(models[0].state_dict(), models[1].state_dict(), dtype=torch.float64)
    P = dict(layers=[{k: v.numpy() for k, v in L.items()} for L in w["layers"]],
             emb=w["emb"].numpy(), ln_f=w["ln_f"].numpy(), W_lm=w["W_lm"].numpy())
    ids = np.array([0, 1, 1, 0, 1])
    L0, L_cap, nh = 7, 16, 2
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 384, (L0,), generator=g) for _ in ids]
    perm, counts = oracle.route_partition(ids)
    st = oracle.DecodeState(2, tuple(int(c) for c in counts), nh, L_cap)
    caches = []
    for j in range(len(ids)):                       # routed row j = sequence perm[j]
        s = int(perm[j])
        kv, cache = prefill(models[ids[s]], prompts[s])
        caches.append(cache)
        m = int(ids[s])
        sl = j - (0 if m == 0 else int(counts[0]))
        for li, (k, v) in enumerate(kv):
            st.k[li][m][sl, :, :L0] = k.double().numpy()
            st.v[li][m][sl, :, :L0] = v.double().numpy()
    cos, sin = oracle.rope_tables(L_cap)
    seq = np.full(len(ids), L0)
    tokens = np.array([17 * (i + 1) % 384 for i in range(len(ids))])
    for _ in range(3):
        nxt, logits = oracle.decode_step(tokens, ids, P, st, seq, nh, cos, sin, CFG["rms_norm_eps"])
        for j in range(len(ids)):
            s = int(perm[j])
            ref = step(models[ids[s]], caches[j], int(tokens[s])).double().numpy()
            assert oracle.rel_err(logits[j], ref) < 1e-4
        tokens = nxt


def test_oracle_prefill_matches_transformers_llama():
    """The oracle's teacher-forced prefill gives transformers' last-token logits
    and prompt caches for prompts of different lengths on both models."""
    import oracle
    from parallel_serve_b200.loader import pack_hf_llama
    models = (make_model(2), make_model(3))
    w = pack_hf_llama(models[0].state_dict(), models[1].state_dict(), dtype=torch.float64)
    P = dict(layers=[{k: v.numpy() for k, v in L.items()} for L in w["layers"]],
             emb=w["emb"].numpy(), ln_f=w["ln_f"].numpy(), W_lm=w["W_lm"].numpy())
    ids = np.array([1, 0, 1, 0])
    lens = [6, 3, 1, 9]
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 384, (n,), generator=g).tolist() for n in lens]
    perm, counts = oracle.route_partition(ids)
    st = oracle.DecodeState(2, tuple(int(c) for c in counts), 2, 16)
    cos, sin = oracle.rope_tables(16)
    nxt, logits = oracle.prefill(prompts, ids, P, st, 2, cos, sin, CFG["rms_norm_eps"])
    for J in range(len(ids)):
        s = int(perm[J])
        m = int(ids[s])
        kv, _ = prefill(models[m], torch.tensor(prompts[s]))
        with torch.no_grad():
            ref = models[m](torch.tensor([prompts[s]])).logits[0, -1].double().numpy()
        assert oracle.rel_err(logits[J], ref) < 1e-4
        assert nxt[s] == int(ref.argmax())
        sl = J - (0 if m == 0 else int(counts[0]))
        for li, (k, v) in enumerate(kv):
            assert oracle.rel_err(st.k[li][m][sl, :, :lens[s]], k.double().numpy()) < 1e-4
            assert oracle.rel_err(st.v[li][m][sl, :, :lens[s]], v.double().numpy()) < 1e-4
