"""numpy restatement of the reference's hot path (test infrastructure only).

Conventions: arrays are float64 unless a ``dt`` argument says otherwise;
``round16`` emulates a 16-bit storage rounding (float16 / bfloat16) where the
reference's torch ops round intermediates. Tokens are in routed order (model
0 first) wherever ``c0`` (the model-0 count) is given.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "round16", "routed_gemm", "route_partition", "rms_norm", "silu", "swiglu", "sdpa",
    "segment_attention", "transformer_block", "routed_block", "rope_tables", "apply_rope",
    "decode_attention", "gather_pages", "decode_layer", "DecodeState", "decode_step", "prefill",
    "deltazip_quantize", "deltazip_dequant", "deltazip_linear", "deltazip_unpack", "rel_err",
]


def round16(a: np.ndarray, kind: str | None) -> np.ndarray:
    """Round to float16 or bfloat16 precision (round-to-nearest-even), keep dtype."""
    if kind is None:
        return a
    if kind == "f16":
        return a.astype(np.float16).astype(a.dtype)
    if kind == "bf16":
        f = np.asarray(a, dtype=np.float32)
        u = f.view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        return u.astype(np.uint32).view(np.float32).astype(a.dtype)
    raise ValueError(kind)


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """The reference's metric: max|err| / mean|ref| (kernel/tests/test_correctness.py:34-38)."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(out - ref).max() / (np.abs(ref).mean() + 1e-9))


# ----------------------------------------------------------------- routing --
def routed_gemm(x: np.ndarray, W: np.ndarray, split_point: int) -> np.ndarray:
    """y[:sp] = x[:sp] @ W[0]; y[sp:] = x[sp:] @ W[1] (kernel/src/routed_gemm.py:200-204)."""
    return np.concatenate([x[:split_point] @ W[0], x[split_point:] @ W[1]], axis=0)


def route_partition(model_id: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Stable partition by model id: perm (routed -> original index) and counts.

    The reference keeps tokens pre-sorted and passes a host split
    (kernel/src/routed_gemm.py:157); with per-token ids the equivalent order is
    a stable argsort, so rows of each model keep their relative order.
    """
    ids = np.asarray(model_id)
    perm = np.argsort(ids, kind="stable").astype(np.int32)
    c0 = int((ids == 0).sum())
    return perm, np.array([c0, ids.size - c0], dtype=np.int32)


# ----------------------------------------------------------- layer pieces --
def rms_norm(x: np.ndarray, w: np.ndarray, eps: float, r16: str | None = None) -> np.ndarray:
    """F.rms_norm as called at experiments/two_model_block.py:56,69.

    torch computes x * rsqrt(mean(x^2) + eps) in fp32 for 16-bit inputs, rounds
    to the input dtype, then multiplies by the weight (rounded again).
    """
    xf = x.astype(np.float64)
    r = 1.0 / np.sqrt((xf * xf).mean(axis=-1, keepdims=True) + eps)
    y = round16(xf * r, r16)
    return round16(y * w, r16)


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def swiglu(gu: np.ndarray, r16: str | None = None) -> np.ndarray:
    """silu(gate) * up on gu = [gate | up] (experiments/two_model_block.py:70-72)."""
    FF = gu.shape[-1] // 2
    g, u = gu[..., :FF], gu[..., FF:]
    return round16(round16(silu(g), r16) * u, r16)


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None) -> np.ndarray:
    """Non-causal scaled-dot-product attention over the last two dims [.., M, d]
    (F.scaled_dot_product_attention as called at experiments/two_model_block.py:65)."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    s = q @ np.swapaxes(k, -1, -2) * scale
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return p @ v


def segment_attention(qkv: np.ndarray, n_heads: int, c0: int) -> np.ndarray:
    """Per-model attention over each model's own segment
    (kernel/src/two_model_block_routed.py:100-120)."""
    M, H3 = qkv.shape
    H = H3 // 3
    hd = H // n_heads
    out = np.empty((M, H), dtype=qkv.dtype)
    for s0, s1 in ((0, c0), (c0, M)):
        if s1 <= s0:
            continue
        q, k, v = (qkv[s0:s1, i * H:(i + 1) * H].reshape(s1 - s0, n_heads, hd).transpose(1, 0, 2)
                   for i in range(3))
        out[s0:s1] = sdpa(q, k, v).transpose(1, 0, 2).reshape(s1 - s0, H)
    return out


def transformer_block(x: np.ndarray, w: dict, n_heads: int, eps: float,
                      r16: str | None = None) -> np.ndarray:
    """One model's layer (experiments/two_model_block.py:54-74): rms_norm -> QKV ->
    SDPA over the batch -> O + residual -> rms_norm -> gate_up -> silu*up -> down + residual."""
    return routed_block(x, {k: np.asarray(v)[None] for k, v in w.items()}, n_heads,
                        x.shape[0], eps, r16)


def routed_block(x: np.ndarray, w: dict, n_heads: int, c0: int, eps: float,
                 r16: str | None = None) -> np.ndarray:
    """Two-model routed layer (kernel/src/two_model_block_routed.py:122-153) with
    stacked weights w[name] = [2, K, N] (ln: [2, H]) and rows [0, c0) on model 0."""
    M = x.shape[0]
    ln1 = w["ln1"]
    ln2 = w["ln2"]
    h = np.concatenate([rms_norm(x[:c0], ln1[0], eps, r16),
                        rms_norm(x[c0:], ln1[-1], eps, r16)], axis=0)
    qkv = round16(routed_gemm(h, w["W_qkv"] if w["W_qkv"].shape[0] == 2 else
                              np.concatenate([w["W_qkv"]] * 2), c0), r16)
    attn = round16(segment_attention(qkv, n_heads, c0), r16)
    Wo = w["W_o"] if w["W_o"].shape[0] == 2 else np.concatenate([w["W_o"]] * 2)
    x = round16(x + round16(routed_gemm(attn, Wo, c0), r16), r16)
    h = np.concatenate([rms_norm(x[:c0], ln2[0], eps, r16),
                        rms_norm(x[c0:], ln2[-1], eps, r16)], axis=0)
    Wgu = w["W_gu"] if w["W_gu"].shape[0] == 2 else np.concatenate([w["W_gu"]] * 2)
    gu = round16(routed_gemm(h, Wgu, c0), r16)
    a = swiglu(gu, r16)
    Wd = w["W_d"] if w["W_d"].shape[0] == 2 else np.concatenate([w["W_d"]] * 2)
    del M
    return round16(x + round16(routed_gemm(a, Wd, c0), r16), r16)


# ------------------------------------------------------------------ decode --
def rope_tables(max_pos: int, head_dim: int = 128, theta: float = 10000.0):
    """cos/sin [max_pos, head_dim/2] for the rotate-half convention, theta^(-2i/d)."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    inv = theta ** (-2.0 * i / head_dim)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang), np.sin(ang)


def apply_rope(x: np.ndarray, pos: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Rotate-half RoPE on x [M, n_heads, d] at per-row positions pos [M]."""
    d2 = x.shape[-1] // 2
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    x1, x2 = x[..., :d2], x[..., d2:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def decode_attention(q: np.ndarray, K: np.ndarray, V: np.ndarray, lens: np.ndarray,
                     scale: float | None = None) -> np.ndarray:
    """q [M, nh, d]; K/V [M, nh, Lmax, d] (row j = token j's cache); attend over
    positions [0, lens[j]) — SDPA with one query per sequence."""
    M, nh, d = q.shape
    out = np.empty_like(q)
    for j in range(M):
        L = int(lens[j])
        out[j] = sdpa(q[j][:, None, :], K[j, :, :L], V[j, :, :L], scale)[:, 0, :]
    return out


def gather_pages(pool: np.ndarray, table_row, page_size: int, L: int) -> np.ndarray:
    """Contiguous history [heads, L, d] of one sequence from a page pool
    [pages, heads, page_size, d] and its block-table row (page of positions
    [i*page_size, (i+1)*page_size) = table_row[i]). The reference has no paged
    cache; this restates the layout the paged kernels read."""
    if L == 0:
        return np.zeros((pool.shape[1], 0, pool.shape[3]), dtype=pool.dtype)
    out = [pool[int(table_row[i])][:, :min(page_size, L - i * page_size)]
           for i in range(-(-L // page_size))]
    return np.concatenate(out, axis=1)


class DecodeState:
    """Per-model KV pools [slots, nh, L_cap, d] for every layer plus lengths."""

    def __init__(self, n_layers: int, slots: tuple[int, int], n_heads: int, L_cap: int,
                 head_dim: int = 128, dt=np.float64):
        self.k = [[np.zeros((slots[m], n_heads, L_cap, head_dim), dt) for m in range(2)]
                  for _ in range(n_layers)]
        self.v = [[np.zeros((slots[m], n_heads, L_cap, head_dim), dt) for m in range(2)]
                  for _ in range(n_layers)]


def decode_layer(x: np.ndarray, w: dict, st: DecodeState, layer: int, n_heads: int, c0: int,
                 pos: np.ndarray, cos: np.ndarray, sin: np.ndarray, eps: float,
                 r16: str | None = None, slots: np.ndarray | None = None) -> np.ndarray:
    """One decode step of one layer for tokens in routed order (model 0 first).

    Same block order as experiments/two_model_block.py:54-74; attention is
    decode attention over the cache: RoPE on q and the new k at position pos[j],
    append k/v to the model's pool at slot (j - offset, or slots[j]), attend
    over [0, pos[j]].
    """
    M, H = x.shape
    hd = H // n_heads
    ln1, ln2 = w["ln1"], w["ln2"]
    h = np.concatenate([rms_norm(x[:c0], ln1[0], eps, r16),
                        rms_norm(x[c0:], ln1[1], eps, r16)], axis=0)
    qkv = round16(routed_gemm(h, w["W_qkv"], c0), r16)
    q = qkv[:, :H].reshape(M, n_heads, hd)
    k = qkv[:, H:2 * H].reshape(M, n_heads, hd)
    v = qkv[:, 2 * H:].reshape(M, n_heads, hd)
    q = round16(apply_rope(q, pos, cos, sin), r16)
    k = round16(apply_rope(k, pos, cos, sin), r16)
    Lmax = int(pos.max()) + 1 if M else 0
    Kc = np.zeros((M, n_heads, Lmax, hd))
    Vc = np.zeros((M, n_heads, Lmax, hd))
    for j in range(M):
        m = 0 if j < c0 else 1
        sl = int(slots[j]) if slots is not None else j - (0 if m == 0 else c0)
        st.k[layer][m][sl, :, pos[j]] = k[j]
        st.v[layer][m][sl, :, pos[j]] = v[j]
        Kc[j] = st.k[layer][m][sl, :, :Lmax]
        Vc[j] = st.v[layer][m][sl, :, :Lmax]
    attn = round16(decode_attention(q, Kc, Vc, pos + 1).reshape(M, H), r16)
    x = round16(x + round16(routed_gemm(attn, w["W_o"], c0), r16), r16)
    h = np.concatenate([rms_norm(x[:c0], ln2[0], eps, r16),
                        rms_norm(x[c0:], ln2[1], eps, r16)], axis=0)
    gu = round16(routed_gemm(h, w["W_gu"], c0), r16)
    a = swiglu(gu, r16)
    return round16(x + round16(routed_gemm(a, w["W_d"], c0), r16), r16)


def decode_step(tokens: np.ndarray, model_id: np.ndarray, params: dict, st: DecodeState,
                seq_len: np.ndarray, n_heads: int, cos: np.ndarray, sin: np.ndarray,
                eps: float, r16: str | None = None):
    """One greedy decode step for a batch in original order.

    params: emb [2, V, H], layers (list of dicts), ln_f [2, H], W_lm [2, H, V].
    Returns (next_tokens [B], logits in routed order [B, V]); seq_len += 1.
    """
    perm, counts = route_partition(model_id)
    c0 = int(counts[0])
    m = (np.arange(len(perm)) >= c0).astype(np.int64)
    x = params["emb"][m, tokens[perm]]
    pos = seq_len[perm].astype(np.int64)
    for li, w in enumerate(params["layers"]):
        x = decode_layer(x, w, st, li, n_heads, c0, pos, cos, sin, eps, r16)
    lnf = params["ln_f"]
    h = np.concatenate([rms_norm(x[:c0], lnf[0], eps, r16),
                        rms_norm(x[c0:], lnf[1], eps, r16)], axis=0)
    logits = round16(routed_gemm(h, params["W_lm"], c0), r16)
    nxt = np.empty(len(perm), dtype=np.int64)
    nxt[perm] = logits.argmax(axis=-1)
    seq_len += 1
    return nxt, logits


def prefill(prompts: list, model_id: np.ndarray, params: dict, st: DecodeState, n_heads: int,
            cos: np.ndarray, sin: np.ndarray, eps: float, r16: str | None = None):
    """Teacher-forced prompt processing (a prefill for the decode loop; the
    reference only measures decode): every prompt token of every sequence goes
    through the layers at its own position, in position order, with k/v
    appended to its sequence's slot, so causality is that of a decode loop.
    prompts: token lists in original batch order, any lengths >= 1.
    Returns (first generated token per sequence [B], last-token logits in
    routed order [B, V])."""
    perm, counts = route_partition(model_id)
    c0 = int(counts[0])
    B = len(perm)
    m_of = (np.arange(B) >= c0).astype(np.int64)
    slot_of = np.arange(B) - np.where(m_of == 1, c0, 0)
    lens = np.array([len(prompts[int(perm[J])]) for J in range(B)])
    last = np.zeros((B, params["emb"].shape[2]))
    for t in range(int(lens.max())):
        rows = np.nonzero(lens > t)[0]                       # routed order: model 0 first
        toks = np.array([prompts[int(perm[J])][t] for J in rows])
        x = params["emb"][m_of[rows], toks]
        c0_t = int((m_of[rows] == 0).sum())
        pos = np.full(len(rows), t, dtype=np.int64)
        for li, w in enumerate(params["layers"]):
            x = decode_layer(x, w, st, li, n_heads, c0_t, pos, cos, sin, eps, r16,
                             slots=slot_of[rows])
        done = lens[rows] == t + 1
        last[rows[done]] = x[done]
    lnf = params["ln_f"]
    h = np.concatenate([rms_norm(last[:c0], lnf[0], eps, r16),
                        rms_norm(last[c0:], lnf[1], eps, r16)], axis=0)
    logits = round16(routed_gemm(h, params["W_lm"], c0), r16)
    nxt = np.empty(B, dtype=np.int64)
    nxt[perm] = logits.argmax(axis=-1)
    return nxt, logits


# ------------------------------------------------------- DeltaZip Route A --
def deltazip_quantize(D: np.ndarray, group: int = 128):
    """Route-A delta compression (the reference only reports numbers for it,
    docs/deltazip_progress_2026-04-17.md:154-162):

    2:4 magnitude pruning along K (keep the 2 largest |D| of every 4
    consecutive k for each n), then symmetric int4 with one fp16 scale per
    128-group along K (scale = max|kept| / 7 over the group, q = round(D/scale)
    clipped to [-7, 7]). Returns (q int8 [K, N] with zeros at pruned entries,
    keep mask bool [K, N], scales float [K/group, N] rounded to fp16).
    """
    K, N = D.shape
    g4 = np.abs(D).reshape(K // 4, 4, N)
    order = np.argsort(-g4, axis=1, kind="stable")
    keep = np.zeros_like(g4, dtype=bool)
    np.put_along_axis(keep, order[:, :2, :], True, axis=1)
    keep = keep.reshape(K, N)
    Dk = np.where(keep, D, 0.0)
    amax = np.abs(Dk).reshape(K // group, group, N).max(axis=1)
    scales = round16(np.where(amax > 0, amax / 7.0, 1.0), "f16")
    q = np.clip(np.rint(Dk / np.repeat(scales, group, axis=0)), -7, 7).astype(np.int8)
    q = np.where(keep, q, 0).astype(np.int8)
    return q, keep, scales


def deltazip_dequant(q: np.ndarray, scales: np.ndarray, group: int = 128) -> np.ndarray:
    """deq(D)[k, n] = q[k, n] * scale[k // group, n] (zero at pruned positions)."""
    return q.astype(np.float64) * np.repeat(scales.astype(np.float64), group, axis=0)


def deltazip_linear(X: np.ndarray, W_base: np.ndarray, q: np.ndarray, scales: np.ndarray,
                    group: int = 128) -> np.ndarray:
    """Y = X @ W_base + X @ deq(D)."""
    return X @ W_base + X @ deltazip_dequant(q, scales, group)


def deltazip_unpack(packed: np.ndarray, K: int, N: int, group: int = 128):
    """Decode the kernel's packed delta format back to (q int8 [K, N], scales
    float16 [K / group, N]) — an independent reader of the layout: per
    128-column tile t and 64-k block b, 3328 bytes = 128 x 16 B kept int4
    values (k order, low nibble first), 128 x 8 B 2-bit positions, 128 x fp16
    scale."""
    pk = np.asarray(packed, dtype=np.uint8).reshape(-1, K // 64, 3328)
    nt = pk.shape[0]
    q = np.zeros((K, nt * 128), dtype=np.int8)
    scales = np.zeros((K // group, nt * 128), dtype=np.float16)
    for t in range(nt):
        for b in range(K // 64):
            blk = pk[t, b]
            vals = blk[:2048].reshape(128, 16)
            meta = blk[2048:3072].reshape(128, 8)
            sc = blk[3072:].view(np.float16)
            scales[(b * 64) // group, t * 128:(t + 1) * 128] = sc
            for j in range(32):
                nib = (vals[:, j // 2] >> (4 * (j % 2))) & 0xF
                v = np.where(nib >= 8, nib.astype(np.int16) - 16, nib.astype(np.int16))
                p = (meta[:, j // 4] >> (2 * (j % 4))) & 0x3
                k = b * 64 + 4 * (j // 2) + p.astype(np.int64)
                q[k, np.arange(t * 128, (t + 1) * 128)] = v.astype(np.int8)
    return q[:, :N], scales[:, :N]
