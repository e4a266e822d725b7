"""Thin Python wrappers over the C ABI, one per kernel.

Each wrapper validates shapes / dtypes on the host (raising ``ValueError`` or
``TypeError`` the way the reference's asserts reject bad input,
kernel/src/routed_gemm.py:163-174), allocates outputs through the torch
caching allocator on the input's device, and launches on the current torch
stream with no host synchronisation, so every call is CUDA-graph capturable.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import check, lib, ptr


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("parallel-serve ops take CUDA tensors")


def _need_contig(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_contiguous():
            raise ValueError("parallel-serve ops take contiguous tensors")


def _counts_arg(counts: torch.Tensor | None) -> int | None:
    if counts is None:
        return None
    if counts.dtype != torch.int32 or counts.numel() < 2 or not counts.is_cuda:
        raise TypeError("counts must be a CUDA int32 tensor of 2 elements")
    return counts.data_ptr()


def route_partition(model_id: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Stable partition of per-token model ids (0/1) -> (perm[M], counts[2]), int32 on device."""
    _need_cuda(model_id)
    if model_id.dtype != torch.int32 or model_id.dim() != 1:
        raise TypeError("model_id must be a 1-D int32 CUDA tensor")
    model_id = model_id.contiguous()
    M = model_id.numel()
    perm = torch.empty(M, dtype=torch.int32, device=model_id.device)
    counts = torch.empty(2, dtype=torch.int32, device=model_id.device)
    check(lib.ps_route_partition(ptr(model_id), M, ptr(perm), ptr(counts),
                                 ptr(_lib.status_tensor(model_id.device)),
                                 _lib.stream_handle(model_id.device)), "ps_route_partition")
    return perm, counts


def gather_rows(src: torch.Tensor, perm: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(src, perm)
    _need_contig(src, perm)
    M = perm.numel()
    if src.shape[0] != M:
        raise ValueError("gather_rows: src must have one row per perm entry")
    out = torch.empty_like(src) if out is None else out
    row_bytes = src[0].numel() * src.element_size() if M else 16
    check(lib.ps_gather_rows(ptr(src), ptr(perm), ptr(out), M, row_bytes,
                             ptr(_lib.status_tensor(src.device)), _lib.stream_handle(src.device)),
          "ps_gather_rows")
    return out


def scatter_rows(src: torch.Tensor, perm: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(src, perm)
    _need_contig(src, perm)
    M = perm.numel()
    out = torch.empty_like(src) if out is None else out
    row_bytes = src[0].numel() * src.element_size() if M else 16
    check(lib.ps_scatter_rows(ptr(src), ptr(perm), ptr(out), M, row_bytes,
                              ptr(_lib.status_tensor(src.device)), _lib.stream_handle(src.device)),
          "ps_scatter_rows")
    return out


def gemm_workspace(device: torch.device, M: int, N: int, epilogue: int) -> torch.Tensor:
    idx = torch.device(device).index or 0
    nbytes = lib.ps_routed_gemm_workspace_bytes(M, N, epilogue, idx)
    return _lib.workspace(device, nbytes, "gemm")


def routed_gemm_raw(x: torch.Tensor, W: torch.Tensor, out: torch.Tensor, *, split_point: int = 0,
                    counts: torch.Tensor | None = None, scatter: torch.Tensor | None = None,
                    residual: torch.Tensor | None = None, epilogue: int = _lib.PS_EPI_STORE,
                    workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Launch ps_routed_gemm with every option exposed (no allocation besides workspace)."""
    M, K = x.shape
    N = W.shape[-1]
    ws = workspace if workspace is not None else gemm_workspace(x.device, M, N, epilogue)
    check(lib.ps_routed_gemm(ptr(x), ptr(W), ptr(out), M, K, N, split_point, _counts_arg(counts),
                             ptr(scatter), ptr(residual), epilogue, _lib.dtype_code(x.dtype),
                             ptr(ws), ws.numel(), ptr(_lib.status_tensor(x.device)),
                             _lib.stream_handle(x.device)), "ps_routed_gemm")
    return out


def gemm_epilogue(mode: int = _lib.PS_EPI_STORE, *, scatter: torch.Tensor | None = None,
                  residual: torch.Tensor | None = None, in_sumsq: torch.Tensor | None = None,
                  norm_dim: int = 0, eps: float = 0.0, out_sumsq: torch.Tensor | None = None,
                  k_pools: tuple = (None, None),
                  v_pools: tuple = (None, None), pos: torch.Tensor | None = None,
                  rope_cos: torch.Tensor | None = None, rope_sin: torch.Tensor | None = None,
                  n_heads: int = 0, block_table: torch.Tensor | None = None,
                  kv_rows: torch.Tensor | None = None,
                  max_model_rows: int = 0, max_ctas: int = 0) -> _lib.GemmEpilogue:
    """Build a ps_gemm_epilogue_t. ``in_sumsq`` is [rows, parts] fp32 (partial sums
    of squares of x's rows). The descriptor holds references to every tensor
    it points to, so they live at least as long as the descriptor."""
    e = _lib.GemmEpilogue()
    e._keep = (scatter, residual, in_sumsq, out_sumsq, k_pools, v_pools, pos, rope_cos, rope_sin,
               block_table, kv_rows)
    e.mode = mode
    e.scatter_rows, e.residual = ptr(scatter), ptr(residual)
    e.in_sumsq, e.norm_dim, e.eps = ptr(in_sumsq), int(norm_dim), float(eps)
    e.in_parts = 0 if in_sumsq is None else (in_sumsq.shape[-1] if in_sumsq.dim() > 1 else 1)
    e.out_sumsq = ptr(out_sumsq)
    e.max_model_rows = int(max_model_rows)
    e.max_ctas = int(max_ctas)
    if mode == _lib.PS_EPI_QKV_ROPE:
        k0, k1, v0, v1, L_cap, s0, s1 = _pool_args(k_pools, v_pools, n_heads)
        e.k_pool0, e.v_pool0, e.k_pool1, e.v_pool1 = ptr(k0), ptr(v0), ptr(k1), ptr(v1)
        e.pos, e.rope_cos, e.rope_sin = ptr(pos), ptr(rope_cos), ptr(rope_sin)
        e.n_heads, e.L_cap, e.slots0, e.slots1 = n_heads, L_cap, s0, s1
        e.apply_rope = 1 if rope_cos is not None else 0
        if block_table is not None:     # page pools: [pages, n_heads, page_size, 128]
            if block_table.dtype != torch.int32 or block_table.dim() != 2:
                raise ValueError("block_table must be int32 [M, max_pages]")
            e.block_table, e.max_pages, e.page_size = ptr(block_table), block_table.shape[1], L_cap
            e.table_rows = block_table.shape[0]
        e.kv_rows = ptr(kv_rows)
    return e


def routed_gemm_ex(x: torch.Tensor, W: torch.Tensor, out: torch.Tensor,
                   epi: _lib.GemmEpilogue, *, split_point: int = 0,
                   counts: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Launch ps_routed_gemm_ex (routed GEMM + fused decode-layer epilogue)."""
    M, K = x.shape
    N = W.shape[-1]
    ws = workspace if workspace is not None else gemm_workspace(
        x.device, M, N, 1 if epi.mode == _lib.PS_EPI_SWIGLU else 0)
    check(lib.ps_routed_gemm_ex(ptr(x), ptr(W), ptr(out), M, K, N, split_point,
                                _counts_arg(counts), ctypes.byref(epi), _lib.dtype_code(x.dtype),
                                ptr(ws), ws.numel(), ptr(_lib.status_tensor(x.device)),
                                _lib.stream_handle(x.device)), "ps_routed_gemm_ex")
    return out


def rmsnorm_routed(x: torch.Tensor, w: torch.Tensor, *, split_point: int = 0,
                   counts: torch.Tensor | None = None, eps: float | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-model RMSNorm. ``w`` is [2, H] (or [1, H] when every row is model 0).

    ``eps=None`` follows F.rms_norm: the machine epsilon of x's dtype.
    """
    _need_cuda(x, w)
    _need_contig(x, w)
    M, H = x.shape
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    out = torch.empty_like(x) if out is None else out
    check(lib.ps_rmsnorm_routed(ptr(x), ptr(w), ptr(out), M, H, split_point, _counts_arg(counts),
                                float(eps), _lib.dtype_code(x.dtype),
                                ptr(_lib.status_tensor(x.device)), _lib.stream_handle(x.device)),
          "ps_rmsnorm_routed")
    return out


def swiglu(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _need_cuda(gu)
    _need_contig(gu)
    M, N2 = gu.shape
    FF = N2 // 2
    out = torch.empty(M, FF, dtype=gu.dtype, device=gu.device) if out is None else out
    check(lib.ps_swiglu(ptr(gu), ptr(out), M, FF, _lib.dtype_code(gu.dtype),
                        _lib.stream_handle(gu.device)), "ps_swiglu")
    return out


def segment_attention(qkv: torch.Tensor, n_heads: int, *, split_point: int = 0,
                      counts: torch.Tensor | None = None, out: torch.Tensor | None = None,
                      scale: float | None = None) -> torch.Tensor:
    """Reference no-KV attention: each token attends to its own model's segment."""
    _need_cuda(qkv)
    _need_contig(qkv)
    M, H3 = qkv.shape
    H = H3 // 3
    if H != n_heads * 128:
        raise ValueError("segment_attention supports head_dim 128 only")
    scale = 1.0 / math.sqrt(128) if scale is None else scale
    out = torch.empty(M, H, dtype=qkv.dtype, device=qkv.device) if out is None else out
    check(lib.ps_segment_attention(ptr(qkv), ptr(out), M, n_heads, split_point, _counts_arg(counts),
                                   float(scale), _lib.dtype_code(qkv.dtype),
                                   ptr(_lib.status_tensor(qkv.device)),
                                   _lib.stream_handle(qkv.device)), "ps_segment_attention")
    return out


def _pool_args(k_pools, v_pools, n_heads: int):
    """Validate the two models' K / V pools [slots, n_heads, L_cap, 128] (same
    L_cap, dtype and device; a model without slots passes None)."""
    k0, k1 = k_pools
    v0, v1 = v_pools
    live = [t for t in (k0, k1, v0, v1) if t is not None]
    if not live:
        raise ValueError("at least one model needs a KV pool")
    L_cap = live[0].shape[2]
    for t in live:
        if t.dim() != 4 or t.shape[1] != n_heads or t.shape[2] != L_cap or t.shape[3] != 128:
            raise ValueError("KV pools must be [slots, n_heads, L_cap, 128] with one L_cap")
        if not (t.is_cuda and t.is_contiguous()):
            raise ValueError("KV pools must be contiguous CUDA tensors")
    if (k0 is None) != (v0 is None) or (k1 is None) != (v1 is None):
        raise ValueError("each model needs both a K and a V pool (or neither)")
    s0 = 0 if k0 is None else k0.shape[0]
    s1 = 0 if k1 is None else k1.shape[0]
    if k0 is not None and v0.shape != k0.shape or k1 is not None and v1.shape != k1.shape:
        raise ValueError("K and V pools of a model must have the same shape")
    return k0, k1, v0, v1, L_cap, s0, s1


def rope_tables(max_pos: int, head_dim: int = 128, theta: float = 10000.0,
                device: torch.device | str = "cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin tables [max_pos, head_dim/2] (fp32), rotate-half convention.

    angle[p, i] = p * theta^(-2i/head_dim), evaluated in float64 then rounded.
    """
    i = torch.arange(head_dim // 2, dtype=torch.float64)
    inv = theta ** (-2.0 * i / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return (ang.cos().to(torch.float32).to(device).contiguous(),
            ang.sin().to(torch.float32).to(device).contiguous())


def rope_kv_append(qkv: torch.Tensor, q_out: torch.Tensor, k_pools: tuple, v_pools: tuple,
                   rope_cos: torch.Tensor | None, rope_sin: torch.Tensor | None,
                   pos: torch.Tensor, *, n_heads: int, split_point: int = 0,
                   counts: torch.Tensor | None = None, slot: torch.Tensor | None = None) -> None:
    """RoPE q and the new k, append k / v to the token's model pool at pos[j].

    Pools are [slots, n_heads, L_cap, 128]; ``k_pools = (k_pool_model0, k_pool_model1)``,
    either may be None when that model has no slots.
    """
    M = qkv.shape[0]
    k0, k1, v0, v1, L_cap, s0, s1 = _pool_args(k_pools, v_pools, n_heads)
    apply = rope_cos is not None
    check(lib.ps_rope_kv_append(ptr(qkv), ptr(q_out), ptr(k0), ptr(v0), ptr(k1), ptr(v1),
                                ptr(rope_cos), ptr(rope_sin), ptr(pos), ptr(slot),
                                _counts_arg(counts), split_point, M, n_heads, L_cap, s0, s1,
                                1 if apply else 0, _lib.dtype_code(qkv.dtype),
                                ptr(_lib.status_tensor(qkv.device)),
                                _lib.stream_handle(qkv.device)), "ps_rope_kv_append")


def attention_workspace(device: torch.device, M: int, n_heads: int, max_len: int,
                        chunk: int = 0) -> torch.Tensor:
    with torch.cuda.device(device):
        nbytes = lib.ps_decode_attention_workspace_bytes(M, n_heads, max_len, chunk)
    return _lib.workspace(device, nbytes, "attn")


def decode_attention(q: torch.Tensor, k_pools: tuple, v_pools: tuple, pos: torch.Tensor, *,
                     n_heads: int, max_len: int, split_point: int = 0,
                     counts: torch.Tensor | None = None, slot: torch.Tensor | None = None,
                     out: torch.Tensor | None = None, chunk: int = 0,
                     scale: float | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Two-model decode attention over the models' KV pools (positions 0..pos[j])."""
    M = q.shape[0]
    k0, k1, v0, v1, L_cap, s0, s1 = _pool_args(k_pools, v_pools, n_heads)
    scale = 1.0 / math.sqrt(128) if scale is None else scale
    out = torch.empty(M, n_heads * 128, dtype=q.dtype, device=q.device) if out is None else out
    ws = workspace if workspace is not None else attention_workspace(q.device, M, n_heads, max_len, chunk)
    check(lib.ps_decode_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1), ptr(out), ptr(pos),
                                  ptr(slot), _counts_arg(counts), split_point, M, n_heads, L_cap,
                                  s0, s1, max_len, chunk, float(scale), _lib.dtype_code(q.dtype),
                                  ptr(ws), ws.numel(), ptr(_lib.status_tensor(q.device)),
                                  _lib.stream_handle(q.device)), "ps_decode_attention")
    return out


def paged_attention_workspace(device: torch.device, M: int, n_heads: int, max_len: int,
                              page_size: int, chunk: int = 0) -> torch.Tensor:
    with torch.cuda.device(device):
        nbytes = lib.ps_paged_decode_attention_workspace_bytes(M, n_heads, max_len, chunk,
                                                               page_size)
    return _lib.workspace(device, nbytes, "attn")


def paged_decode_attention(q: torch.Tensor, k_pages: tuple, v_pages: tuple, pos: torch.Tensor,
                           block_table: torch.Tensor, *, n_heads: int, max_len: int,
                           seq_rows: torch.Tensor | None = None,
                           split_point: int = 0, counts: torch.Tensor | None = None,
                           out: torch.Tensor | None = None, chunk: int = 0,
                           scale: float | None = None,
                           workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention over paged KV: pools ``[pages, n_heads, page_size, 128]`` per
    model, ``block_table`` int32 ``[M, max_pages]`` (routed rows) of page ids."""
    M = q.shape[0]
    k0, k1, v0, v1, page_size, p0, p1 = _pool_args(k_pages, v_pages, n_heads)
    if block_table.dtype != torch.int32 or block_table.dim() != 2:
        raise ValueError("block_table must be int32 [rows, max_pages]")
    if seq_rows is None and block_table.shape[0] < M:
        raise ValueError("block_table needs a row per token when seq_rows is not given")
    if not block_table.is_contiguous():
        raise ValueError("block_table must be contiguous")
    scale = 1.0 / math.sqrt(128) if scale is None else scale
    out = torch.empty(M, n_heads * 128, dtype=q.dtype, device=q.device) if out is None else out
    ws = workspace if workspace is not None else paged_attention_workspace(
        q.device, M, n_heads, max_len, page_size, chunk)
    check(lib.ps_paged_decode_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1), ptr(out),
                                        ptr(pos), ptr(block_table), block_table.shape[0],
                                        ptr(seq_rows), block_table.shape[1],
                                        page_size, _counts_arg(counts), split_point, M, n_heads,
                                        p0, p1, max_len, chunk, float(scale),
                                        _lib.dtype_code(q.dtype), ptr(ws), ws.numel(),
                                        ptr(_lib.status_tensor(q.device)),
                                        _lib.stream_handle(q.device)), "ps_paged_decode_attention")
    return out


def prefill_attention(q: torch.Tensor, k_pools: tuple, v_pools: tuple, blocks: torch.Tensor, *,
                      n_heads: int, out: torch.Tensor | None = None,
                      scale: float | None = None,
                      block_table: torch.Tensor | None = None) -> torch.Tensor:
    """Causal prefill attention on the tensor cores over the KV pools.
    ``blocks`` int32 [nblocks, 5] = (row0, nq <= 128, p0, model, slot): rows
    row0.. of q are prompt tokens at positions p0.. of that sequence. With
    ``block_table`` [rows, max_pages] the pools are page pools and `slot` is the
    sequence's block-table row."""
    T = q.shape[0]
    k0, k1, v0, v1, L_cap, s0, s1 = _pool_args(k_pools, v_pools, n_heads)
    bt_rows = max_pages = page_size = 0
    if block_table is not None:
        page_size, max_pages = L_cap, block_table.shape[1]
        bt_rows, L_cap = block_table.shape[0], max_pages * page_size
    if blocks.dtype != torch.int32 or blocks.dim() != 2 or blocks.shape[1] != 5:
        raise ValueError("blocks must be int32 [nblocks, 5]")
    scale = 1.0 / math.sqrt(128) if scale is None else scale
    out = torch.empty(T, n_heads * 128, dtype=q.dtype, device=q.device) if out is None else out
    check(lib.ps_prefill_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1), ptr(out),
                                   ptr(blocks.contiguous()), blocks.shape[0], T, n_heads, L_cap,
                                   s0, s1, ptr(block_table), bt_rows, max_pages, page_size,
                                   float(scale), _lib.dtype_code(q.dtype),
                                   ptr(_lib.status_tensor(q.device)),
                                   _lib.stream_handle(q.device)), "ps_prefill_attention")
    return out


def embed_routed(emb: torch.Tensor, tokens: torch.Tensor, perm: torch.Tensor | None,
                 counts: torch.Tensor | None, out: torch.Tensor, *,
                 out_sumsq: torch.Tensor | None = None) -> torch.Tensor:
    """out[j] = emb[m(j)][tokens[perm[j]]]; emb [2, vocab, H]. Optionally
    out_sumsq[j] = sum(out[j]^2) (fp32)."""
    M, H = out.shape
    vocab = emb.shape[1]
    check(lib.ps_embed_routed(ptr(emb), ptr(tokens), ptr(perm), _counts_arg(counts), ptr(out), M, H,
                              vocab, ptr(out_sumsq), _lib.dtype_code(emb.dtype),
                              ptr(_lib.status_tensor(emb.device)),
                              _lib.stream_handle(emb.device)), "ps_embed_routed")
    return out


def argmax_rows(logits: torch.Tensor, perm: torch.Tensor | None, next_tokens: torch.Tensor,
                seq_len: torch.Tensor | None = None) -> torch.Tensor:
    M, V = logits.shape
    check(lib.ps_argmax_rows(ptr(logits), ptr(perm), ptr(next_tokens), ptr(seq_len), M, V,
                             _lib.dtype_code(logits.dtype), _lib.stream_handle(logits.device)),
          "ps_argmax_rows")
    return next_tokens


def positions_routed(seq_len: torch.Tensor, perm: torch.Tensor | None, out: torch.Tensor) -> torch.Tensor:
    check(lib.ps_positions_routed(ptr(seq_len), ptr(perm), ptr(out), out.numel(),
                                  _lib.stream_handle(seq_len.device)), "ps_positions_routed")
    return out
