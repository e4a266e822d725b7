"""Two small random Hugging Face Llama models (transformers, CPU float32) as an
independent implementation of the decode step for the loader tests: the same
architecture as Llama-2-7B (multi-head attention, head_dim 128, rotate-half
RoPE, RMSNorm, SwiGLU) at a size that runs in seconds."""
from __future__ import annotations

import torch

CFG = dict(vocab_size=384, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
           num_attention_heads=2, num_key_value_heads=2, rms_norm_eps=1e-5, rope_theta=10000.0,
           max_position_embeddings=256, tie_word_embeddings=False)


def make_model(seed: int):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    m = LlamaForCausalLM(LlamaConfig(**CFG)).eval()
    g = torch.Generator().manual_seed(seed + 100)
    with torch.no_grad():          # non-trivial norm weights, so folding them is exercised
        for name, p in m.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
            elif p.dim() == 2:     # round to fp16 so both paths start from the same weights
                p.copy_(p.half().float())
    return m


def prefill(model, prompt: torch.Tensor):
    """HF prefill of one sequence: (per-layer K and V [heads, L, 128] after RoPE,
    the cache object for continuing)."""
    with torch.no_grad():
        out = model(prompt[None], use_cache=True)
    kv = [(l.keys[0].clone(), l.values[0].clone()) for l in out.past_key_values.layers]
    return kv, out.past_key_values


def step(model, cache, token: int) -> torch.Tensor:
    """Logits [V] of the next position after feeding `token` with the cache."""
    with torch.no_grad():
        out = model(torch.tensor([[token]]), past_key_values=cache, use_cache=True)
    return out.logits[0, -1]
