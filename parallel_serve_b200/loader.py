"""Real-weight loader: two Hugging Face Llama checkpoints -> stacked two-model weights.

The reference packs each model's HF ``[out, in]`` projections into its
``x @ W`` layout and stacks the two models (experiments/real_weights_correctness.py:
27-51): ``W_qkv = cat(q, k, v).T`` ``[H, 3H]``, ``W_o = o.T``,
``W_gu = cat(gate, up).T`` ``[H, 2 FF]``, ``W_d = down.T``; norms as they are.
``pack_hf_llama`` does the same for every layer of two state dicts (plus the
embedding, final norm and LM head the decode step needs) and returns the
``weights`` dict ``TwoModelDecoder`` takes. HF Llama stores q / k in the
rotate-half RoPE layout, which is the layout these kernels use, so no
permutation is applied. Grouped-query checkpoints (fewer KV heads than query
heads) are rejected: the decode kernels implement multi-head attention, as
Llama-2-7B and Vicuna-7B use.
"""
from __future__ import annotations

import glob
import json
import os
from typing import Mapping

import torch

from .decoder import DecoderConfig

_P = "model.layers.{i}."


def decoder_config_from_hf(hf: Mapping | object, dtype: torch.dtype = torch.float16) -> DecoderConfig:
    """DecoderConfig from a HF LlamaConfig (object or config.json dict)."""
    get = (lambda k, d=None: hf.get(k, d)) if isinstance(hf, Mapping) else \
        (lambda k, d=None: getattr(hf, k, d))
    H, nh = int(get("hidden_size")), int(get("num_attention_heads"))
    nkv = int(get("num_key_value_heads") or nh)
    if nkv != nh:
        raise ValueError(f"grouped-query attention ({nkv} KV heads for {nh} query heads) "
                         "is not supported by the decode kernels")
    theta = get("rope_theta")
    if theta is None:
        rp = get("rope_parameters") or get("rope_scaling") or {}
        theta = rp.get("rope_theta", 10000.0) if isinstance(rp, Mapping) else 10000.0
    return DecoderConfig(n_layers=int(get("num_hidden_layers")), hidden=H, n_heads=nh,
                         ffn=int(get("intermediate_size")), vocab=int(get("vocab_size")),
                         eps=float(get("rms_norm_eps", 1e-5)), rope_theta=float(theta),
                         dtype=dtype)


def _layer(sd: Mapping[str, torch.Tensor], i: int) -> dict:
    p = _P.format(i=i)
    q, k, v, o = (sd[p + f"self_attn.{n}_proj.weight"] for n in "qkvo")
    gate, up, down = (sd[p + f"mlp.{n}_proj.weight"] for n in ("gate", "up", "down"))
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("grouped-query attention is not supported by the decode kernels")
    return dict(W_qkv=torch.cat([q, k, v], dim=0).t(), W_o=o.t(),
                W_gu=torch.cat([gate, up], dim=0).t(), W_d=down.t(),
                ln1=sd[p + "input_layernorm.weight"], ln2=sd[p + "post_attention_layernorm.weight"])


def pack_hf_llama(state_a: Mapping[str, torch.Tensor], state_b: Mapping[str, torch.Tensor],
                  n_layers: int | None = None, dtype: torch.dtype = torch.float16) -> dict:
    """Stacked weights of two same-architecture HF Llama state dicts (model 0 =
    ``state_a``, model 1 = ``state_b``) in the layout of TwoModelDecoder:
    ``{"emb": [2,V,H], "ln_f": [2,H], "W_lm": [2,H,V], "layers": [{W_qkv [2,H,3H],
    W_o [2,H,H], W_gu [2,H,2FF], W_d [2,FF,H], ln1 [2,H], ln2 [2,H]}, ...]}``
    (contiguous, on the state dicts' device, in ``dtype``)."""
    if n_layers is None:
        n_layers = 1 + max(int(k.split(".")[2]) for k in state_a if k.startswith("model.layers."))

    def stack(a, b):
        if a.shape != b.shape:
            raise ValueError(f"the two models differ in shape: {tuple(a.shape)} vs {tuple(b.shape)}")
        return torch.stack([a.to(dtype), b.to(dtype)]).contiguous()

    layers = []
    for i in range(n_layers):
        la, lb = _layer(state_a, i), _layer(state_b, i)
        layers.append({k: stack(la[k], lb[k]) for k in la})

    def lm_head(sd):
        w = sd.get("lm_head.weight")
        return (sd["model.embed_tokens.weight"] if w is None else w).t()   # tied embeddings
    return dict(layers=layers,
                emb=stack(state_a["model.embed_tokens.weight"], state_b["model.embed_tokens.weight"]),
                ln_f=stack(state_a["model.norm.weight"], state_b["model.norm.weight"]),
                W_lm=stack(lm_head(state_a), lm_head(state_b)))


def load_hf_state_dict(path: str) -> dict[str, torch.Tensor]:
    """Tensors of a HF checkpoint directory (``*.safetensors`` through the
    ``safetensors`` package when it is installed, else ``pytorch_model*.bin``)."""
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    out: dict[str, torch.Tensor] = {}
    if files:
        try:
            from safetensors.torch import load_file
        except ImportError as ex:
            raise ImportError("reading .safetensors needs the safetensors package") from ex
        for f in files:
            out.update(load_file(f))
        return out
    files = sorted(glob.glob(os.path.join(path, "pytorch_model*.bin")))
    if not files:
        raise FileNotFoundError(f"no *.safetensors or pytorch_model*.bin under {path}")
    for f in files:
        out.update(torch.load(f, map_location="cpu", weights_only=True))
    return out


def load_two_llama(path_a: str, path_b: str, dtype: torch.dtype = torch.float16):
    """(DecoderConfig, weights) of two HF Llama checkpoint directories."""
    with open(os.path.join(path_a, "config.json")) as f:
        cfg_a = json.load(f)
    with open(os.path.join(path_b, "config.json")) as f:
        cfg_b = json.load(f)
    ca, cb = decoder_config_from_hf(cfg_a, dtype), decoder_config_from_hf(cfg_b, dtype)
    if (ca.n_layers, ca.hidden, ca.n_heads, ca.ffn, ca.vocab) != \
            (cb.n_layers, cb.hidden, cb.n_heads, cb.ffn, cb.vocab):
        raise ValueError("the two checkpoints must share one architecture")
    return ca, pack_hf_llama(load_hf_state_dict(path_a), load_hf_state_dict(path_b),
                             ca.n_layers, dtype)
