"""Two-model greedy decode loop on parallel-serve kernels (KV cache, RoPE, CUDA graphs).

This is the decode path that the reference's blocks are measured
on (kernel/benchmarks/bench_full_stack.py:161-265 times 32 stacked layers under
a CUDA graph) extended with per-sequence fp16 KV caches, RoPE, embeddings and a
routed LM head:

  partition(model_id) -> positions -> routed embedding ->
  32 x [rms_norm, QKV, RoPE + KV append, decode attention, O (+res),
        rms_norm, gate_up + SwiGLU, down (+res)] ->
  rms_norm -> routed LM head -> greedy argmax (scatter to batch order, len += 1)

With ``fused_epilogues`` (the default) a layer is 5 launches: the RMSNorm
weights are folded into the rows of W_qkv / W_gu / W_lm at load, every
producer of the residual stream (embedding, O and down GEMMs, or the
all-reduce under tensor parallelism) also writes per-row partial sums of
squares, the consuming GEMM scales its accumulator by 1/rms, and RoPE plus the
KV-cache append run in the QKV GEMM's epilogue:

  [QKV+norm+RoPE+KV append, attention, O (+res, sumsq), gate_up+norm+SwiGLU,
   down (+res, sumsq)]

Tokens stay in routed order (model 0 first) for the whole step; the split is
read on the device, so one captured graph serves any split. Each model owns
its KV pools ``[slots, heads, L_cap, 128]``; sequence slots follow the stable
routed order. ``mode="serial"`` runs the same kernels one model at a time
(every launch sees only one model's tokens): the "serial two-model decode of
the same kernels" baseline.

Tensor parallelism (``tp_group``): QKV and gate_up are column-split (by heads
and by FF), O and down row-split with an all-reduce of the layer output after
each, KV pools are split by heads, the LM head is split by vocabulary with a
(max, index) exchange for the greedy pick.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib, ops
from ._lib import check, lib, ptr


@dataclass
class DecoderConfig:
    n_layers: int = 32
    hidden: int = 4096
    n_heads: int = 32
    ffn: int = 11008
    vocab: int = 32000
    eps: float = 1e-5
    rope_theta: float = 10000.0
    dtype: torch.dtype = torch.float16

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads


def shard_columns(W: torch.Tensor, parts: int, rank: int, groups: int = 1) -> torch.Tensor:
    """Column shard of a stacked [2, K, N] weight whose N is `groups` equal
    blocks (q|k|v: 3, gate|up: 2): rank r takes the r-th slice of every block."""
    two, K, N = W.shape
    blk = N // groups
    sz = blk // parts
    cols = [W[:, :, g * blk + rank * sz: g * blk + (rank + 1) * sz] for g in range(groups)]
    return torch.cat(cols, dim=2).contiguous()


def shard_rows(W: torch.Tensor, parts: int, rank: int) -> torch.Tensor:
    """Row shard of a stacked [2, K, N] weight (K split in `parts`)."""
    K = W.shape[1]
    sz = K // parts
    return W[:, rank * sz:(rank + 1) * sz].contiguous()


def fold_norm(W: torch.Tensor, ln: torch.Tensor) -> torch.Tensor:
    """diag(ln[m]) @ W[m] for a stacked [2, K, N] weight and [2, K] RMSNorm
    weight: rms_norm(x, ln) @ W == (x / rms(x)) @ fold_norm(W, ln). Computed
    in fp32 and rounded once, a model at a time."""
    out = torch.empty_like(W)
    for m in range(W.shape[0]):
        out[m] = (W[m].float() * ln[m].float()[:, None]).to(W.dtype)
    return out


class PackedWeight:
    """A stacked [2, K, N] projection weight held only in the library's packed
    HBM layout (ps_pack_weights): every (model, weight tile, 128-k block) one
    contiguous 32 KB block in the GEMM stage's shared-memory order, so each
    pipeline stage is one sequential bulk read. The packing depends on whether
    the GEMM's epilogue is SwiGLU (gate and up columns paired)."""

    def __init__(self, W: torch.Tensor, epilogue: int):
        if W.dim() != 3 or not W.is_contiguous():
            raise ValueError("PackedWeight takes a contiguous [nmat, K, N] weight")
        self.shape = tuple(W.shape)
        self.dtype = W.dtype
        self.gated = epilogue == _lib.PS_EPI_SWIGLU
        nmat, K, N = self.shape
        nbytes = lib.ps_packed_weights_bytes(nmat, K, N, epilogue)
        self.data = torch.empty(nbytes, dtype=torch.uint8, device=W.device)
        check(lib.ps_pack_weights(ptr(W), nmat, K, N, epilogue, ptr(self.data), nbytes,
                                  _lib.stream_handle(W.device)), "ps_pack_weights")

    def attach(self, epi) -> None:
        """Point a GEMM epilogue descriptor at the packed blocks."""
        if (epi.mode == _lib.PS_EPI_SWIGLU) != self.gated:
            raise ValueError("weights were packed for another epilogue mode")
        epi.w_packed = self.data.data_ptr()


def _wargs(W, epi):
    """(W pointer, K, N) for a GEMM launch; packed weights go in the epilogue."""
    if isinstance(W, PackedWeight):
        W.attach(epi)
        return None, W.shape[-2], W.shape[-1]
    epi.w_packed = None
    return ptr(W), W.shape[-2], W.shape[-1]


def prefill_layout(prompts, perm, c0: int, chunk: int, paged: bool) -> list[dict]:
    """Host layout of a routed prefill: every prompt token of every sequence
    in routed sequence order (routed row J = original sequence perm[J]; rows
    J < c0 belong to model 0), cut into launches of at most `chunk` tokens.
    Per chunk: token ids, positions, KV rows (the sequence's slot in its
    model's pool, or its block-table row J when paged), n0 = model-0 tokens
    (they come first), last = [(row in chunk, J)] for every sequence whose
    last prompt token falls in the chunk, and qblocks = [row0, nq, p0, model,
    kv row] for each run of at most 128 consecutive tokens of one sequence
    (the work items of the tensor-core prefill attention)."""
    toks, poss, rows, seqs = [], [], [], []
    for J, s in enumerate(perm):
        p = [int(t) for t in prompts[int(s)]]
        toks += p
        poss += list(range(len(p)))
        rows += [J if paged else (J - c0 if J >= c0 else J)] * len(p)
        seqs += [J] * len(p)
    T = len(toks)
    n0_total = sum(len(prompts[int(s)]) for s in list(perm)[:c0])
    out = []
    for start in range(0, T, chunk):
        n = min(chunk, T - start)
        sl = slice(start, start + n)
        qblocks = []
        i = start
        while i < start + n:
            e = i
            while e < start + n and seqs[e] == seqs[i] and e - i < 128:
                e += 1
            J = seqs[i]
            qblocks.append([i - start, e - i, poss[i], 0 if J < c0 else 1, rows[i]])
            i = e
        out.append(dict(tok=toks[sl], pos=poss[sl], kv_rows=rows[sl],
                        n0=max(0, min(n0_total - start, n)),
                        last=[(i - start, seqs[i]) for i in range(start, start + n)
                              if i + 1 == T or seqs[i + 1] != seqs[i]],
                        qblocks=qblocks))
    return out


class TwoModelDecoder:
    """Both models' weights, KV pools and step buffers resident on one GPU (or one
    tensor-parallel rank).

    ``model_id`` (length B, values 0/1) fixes which model serves each sequence.
    ``weights`` optionally supplies full (unsharded) stacked weights as a dict
    ``{"emb": [2,V,H], "ln_f": [2,H], "W_lm": [2,H,V], "layers": [{W_qkv, W_o,
    W_gu, W_d, ln1, ln2}, ...]}``; otherwise weights are drawn N(0, 0.02) on the
    device (norm weights 1).

    ``kv_layers`` (default: one per layer) allocates that many sets of KV pools
    and gives layer i the set i % kv_layers. Every layer still appends to and
    reads a full history of its own size, so the step moves the same bytes,
    but layers that share a set overwrite each other's cache entries: it lets
    a workload whose KV caches exceed the GPU's memory (Llama-13B shapes at
    256 sequences per model and 4096 positions) be timed, and its outputs are
    not those of the model.
    """

    def __init__(self, cfg: DecoderConfig, model_id, L_cap: int, *, device="cuda",
                 weights: dict | None = None, seed: int = 0, tp_group=None,
                 allreduce: str = "nvlink", fused_epilogues: bool = True,
                 page_size: int | None = None, prefill_chunk: int = 256,
                 kv_layers: int | None = None, chain: bool = False, packed: bool = True,
                 auto_grid: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dt = cfg.dtype
        self.tp_group = tp_group
        if tp_group is not None:
            import torch.distributed as dist
            self.tp = dist.get_world_size(tp_group)
            self.rank = dist.get_rank(tp_group)
        else:
            self.tp, self.rank = 1, 0
        if cfg.n_heads % self.tp or cfg.ffn % self.tp or cfg.vocab % self.tp:
            raise ValueError("heads, ffn and vocab must divide by the tensor-parallel size")
        self.nh = cfg.n_heads // self.tp          # heads on this rank
        self.Hl = self.nh * cfg.head_dim          # q/k/v width on this rank
        self.FFl = cfg.ffn // self.tp
        self.Vl = cfg.vocab // self.tp
        if cfg.head_dim != 128:
            raise ValueError("the decode kernels support head_dim 128")
        mid = torch.as_tensor(model_id, dtype=torch.int32).flatten()
        self.B = int(mid.numel())
        self.counts_host = (int((mid == 0).sum()), int((mid == 1).sum()))
        if self.counts_host[0] + self.counts_host[1] != self.B:
            raise ValueError("model ids must be 0 or 1")
        self.L_cap = L_cap
        dev, dt = self.device, self.dt
        H, FF, V = cfg.hidden, cfg.ffn, cfg.vocab
        gen = torch.Generator(device=dev).manual_seed(seed + 1000 * self.rank)

        def rnd(*shape, std=0.02):
            return torch.empty(*shape, dtype=dt, device=dev).normal_(0.0, std, generator=gen)

        # ---------------------------------------------------------- weights
        self.layers = []
        if weights is None:
            for _ in range(cfg.n_layers):
                self.layers.append(dict(
                    W_qkv=rnd(2, H, 3 * self.Hl), W_o=rnd(2, self.Hl, H),
                    W_gu=rnd(2, H, 2 * self.FFl), W_d=rnd(2, self.FFl, H),
                    ln1=torch.ones(2, H, dtype=dt, device=dev),
                    ln2=torch.ones(2, H, dtype=dt, device=dev)))
            self.emb = rnd(2, V, H)
            self.ln_f = torch.ones(2, H, dtype=dt, device=dev)
            self.W_lm = rnd(2, H, self.Vl)
        else:
            tp, r = self.tp, self.rank
            for Lw in weights["layers"]:
                self.layers.append(dict(
                    W_qkv=shard_columns(Lw["W_qkv"], tp, r, 3).to(dev, dt),
                    W_o=shard_rows(Lw["W_o"], tp, r).to(dev, dt),
                    W_gu=shard_columns(Lw["W_gu"], tp, r, 2).to(dev, dt),
                    W_d=shard_rows(Lw["W_d"], tp, r).to(dev, dt),
                    ln1=Lw["ln1"].to(dev, dt).contiguous(), ln2=Lw["ln2"].to(dev, dt).contiguous()))
            self.emb = weights["emb"].to(dev, dt).contiguous()
            self.ln_f = weights["ln_f"].to(dev, dt).contiguous()
            self.W_lm = shard_columns(weights["W_lm"], tp, r, 1).to(dev, dt)
        # The norm statistics come from the all-reduce kernel or the GEMM
        # epilogue; a plain NCCL all-reduce produces none.
        self.fused = fused_epilogues and (self.tp == 1 or allreduce.startswith("nvlink"))
        if self.fused:
            for L in self.layers:
                L["W_qkv"] = fold_norm(L.pop("W_qkv"), L.pop("ln1"))
                L["W_gu"] = fold_norm(L.pop("W_gu"), L.pop("ln2"))
            self.W_lm = fold_norm(self.W_lm, self.ln_f)
            self.ln_f = None
        # Packed HBM layout for every projection of the fused path (the
        # unpacked copy is released as each is packed).
        self.packed = bool(packed and self.fused)
        # decode GEMMs pick their CTA count by shape (ps_gemm_epilogue_t.max_ctas = -1)
        self.auto_grid = bool(auto_grid)
        if self.packed:
            STORE, SWIGLU = _lib.PS_EPI_STORE, _lib.PS_EPI_SWIGLU
            for L in self.layers:
                for name, epi in (("W_qkv", STORE), ("W_o", STORE), ("W_gu", SWIGLU),
                                  ("W_d", STORE)):
                    L[name] = PackedWeight(L.pop(name), epi)
            self.W_lm = PackedWeight(self.W_lm, STORE)
            torch.cuda.synchronize(dev)

        # ---------------------------------------------------------- KV pools
        # contiguous: [slots, heads, L_cap, 128] per model and layer;
        # paged: [pages, heads, page_size, 128] with one block table for all layers
        s0, s1 = self.counts_host
        self.page_size = page_size
        self.block_table = None
        if page_size is not None:
            from .paged_kv import BlockTable, PageAllocator
            if not self.fused:
                raise ValueError("paged KV runs with the fused epilogues (fused_epilogues=True "
                                 "and, under tensor parallelism, allreduce='nvlink')")
            self.max_pages = -(-L_cap // page_size)
            L_cap = self.max_pages * page_size
            self.L_cap = L_cap
            n_pages = (s0 * self.max_pages, s1 * self.max_pages)
            self.block_table = BlockTable([0] * s0 + [1] * s1,
                                          tuple(PageAllocator(n, shuffle_seed=seed + m)
                                                for m, n in enumerate(n_pages)),
                                          self.max_pages, page_size, dev)
            shapes = [(n, self.nh, page_size, 128) for n in n_pages]
        else:
            shapes = [(s, self.nh, L_cap, 128) for s in (s0, s1)]
        self._host_len = 0
        self.kv_layers = cfg.n_layers if kv_layers is None else int(kv_layers)
        if kv_layers is not None and not 1 <= self.kv_layers <= cfg.n_layers:
            raise ValueError(f"kv_layers must be in [1, {cfg.n_layers}], got {kv_layers}")
        self.kpool, self.vpool = [], []
        for li in range(cfg.n_layers):
            if li >= self.kv_layers:            # aliased: share set li % kv_layers
                self.kpool.append(self.kpool[li % self.kv_layers])
                self.vpool.append(self.vpool[li % self.kv_layers])
                continue
            ks = [torch.empty(*sh, dtype=dt, device=dev) if sh[0] else None for sh in shapes]
            vs = [torch.empty(*sh, dtype=dt, device=dev) if sh[0] else None for sh in shapes]
            self.kpool.append(ks)
            self.vpool.append(vs)
        self.rope_cos, self.rope_sin = ops.rope_tables(L_cap, 128, cfg.rope_theta, dev)

        # ---------------------------------------------------------- step buffers
        B = self.B
        i32 = dict(dtype=torch.int32, device=dev)
        self.model_id = mid.to(dev)
        self.tokens = torch.zeros(B, **i32)
        self.next_tokens = torch.zeros(B, **i32)
        self.seq_len = torch.zeros(B, **i32)
        self.perm = torch.zeros(B, **i32)
        self.counts = torch.zeros(2, **i32)
        self.pos = torch.zeros(B, **i32)
        self.counts_serial = [torch.tensor([s0, 0], **i32), torch.tensor([0, s1], **i32)]
        self.x = torch.zeros(B, H, dtype=dt, device=dev)
        self.x_alt = torch.zeros(B, H, dtype=dt, device=dev)   # tensor-parallel ping-pong
        self.h = torch.zeros(B, H, dtype=dt, device=dev)
        self.qkv = torch.zeros(B, 3 * self.Hl, dtype=dt, device=dev)
        self.q = torch.zeros(B, self.Hl, dtype=dt, device=dev)
        self.attn = torch.zeros(B, self.Hl, dtype=dt, device=dev)
        self.a = torch.zeros(B, self.FFl, dtype=dt, device=dev)
        self.logits = torch.zeros(B, self.Vl, dtype=dt, device=dev)
        # folded-RMSNorm statistics: per-row partial sums of squares of the
        # residual stream (embedding: 1 part; GEMM: H/128; all-reduce: H/256)
        f32 = dict(dtype=torch.float32, device=dev)
        self.sq_emb = torch.zeros(B, 1, **f32)
        # per-launch path: GEMM epilogues write H/128 parts, the all-reduce H/256;
        # the projection chain's all-reduce writes H/64 (one per 64-column part)
        self.sq_parts = H // 128 if self.tp == 1 else H // 256
        self.use_chain = bool(chain and self.fused and self.B <= 256 and
                              max(self.counts_host) <= 128 and
                              (self.tp == 1 or allreduce.startswith("nvlink")))
        dec_parts = H // 64 if (self.use_chain and self.tp > 1) else self.sq_parts
        self.sq_a = torch.zeros(B, dec_parts, **f32)
        self.sq_b = torch.zeros(B, dec_parts, **f32)
        self.sq_last = torch.zeros(B, self.sq_parts, **f32)   # prefill: last prompt rows
        idx = self.device.index or 0
        gw = max(lib.ps_routed_gemm_workspace_bytes(B, n, e, idx)
                 for n, e in ((3 * self.Hl, 0), (H, 0), (2 * self.FFl, 1), (self.Vl, 0)))
        self.gemm_ws = torch.zeros(gw, dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            if page_size is None:
                aw = max(lib.ps_decode_attention_workspace_bytes(m, self.nh, L_cap, 0)
                         for m in (B, s0, s1) if m > 0)
            else:
                aw = max(lib.ps_paged_decode_attention_workspace_bytes(m, self.nh, L_cap, 0,
                                                                       page_size)
                         for m in (B, s0, s1) if m > 0)
        self.attn_ws = torch.zeros(max(aw, 256), dtype=torch.uint8, device=dev)
        self.status = _lib.status_tensor(dev)
        # One chain workspace for every chain launch of this rank: it carries the
        # launch epoch that the all-reduce flags of all ranks follow.
        self.chain_ws = (torch.zeros(lib.ps_routed_chain_workspace_bytes(B, 6, idx),
                                     dtype=torch.uint8, device=dev) if self.use_chain else None)
        self._chains: dict = {}
        self.ar = None
        self._slot = 0
        if self.tp > 1:
            self.lm_best = torch.zeros(B, 2, dtype=torch.float32, device=dev)
            self.lm_gather = torch.zeros(self.tp, B, 2, dtype=torch.float32, device=dev)
            algos = {"nvlink": _lib.PS_AR_AUTO, "nvlink1": _lib.PS_AR_ONE_SHOT,
                     "nvlink2": _lib.PS_AR_TWO_SHOT, "nvlink-ll": _lib.PS_AR_TWO_SHOT_LL}
            if allreduce in algos:
                from .tp import NvlinkAllReduce
                self.ar = NvlinkAllReduce(tp_group, max(B, prefill_chunk) * H, dev, dt,
                                          algo=algos[allreduce])
            elif allreduce != "nccl":
                raise ValueError("allreduce must be 'nvlink' (one-shot), "
                                 f"'nvlink1', 'nvlink2', 'nvlink-ll' or 'nccl', got {allreduce!r}")
        self.graphs: dict[str, torch.cuda.CUDAGraph] = {}
        # routed order of the fixed model ids (host copy for the prefill)
        self.prefill_chunk = prefill_chunk
        self._perm_host = torch.argsort(mid, stable=True).to(torch.int32)
        self._perm_static = self._perm_host.to(dev)
        self._counts_seq = torch.tensor(self.counts_host, **i32)
        self._pf = None      # prefill buffers, allocated on first use
        self._in_prefill = False

    # ------------------------------------------------------------------ state
    def fill_kv_random(self, length: int, seed: int = 0) -> None:
        """Synthetic prompt: KV positions [0, length) ~ N(0, 1) for every sequence."""
        gen = torch.Generator(device=self.device).manual_seed(seed + 7 + 1000 * self.rank)
        for ks, vs in zip(self.kpool[:self.kv_layers], self.vpool[:self.kv_layers]):
            for t in ks + vs:
                if t is not None:
                    t.normal_(0.0, 1.0, generator=gen)
        self.seq_len.fill_(length)
        self._host_len = length
        self.reserve(1)

    def set_state(self, tokens: torch.Tensor, seq_len) -> None:
        self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32))
        sl = torch.as_tensor(seq_len, dtype=torch.int32)
        self.seq_len.copy_(sl)
        self._host_len = int(sl.max()) if sl.numel() else 0
        self.reserve(1)

    def reset_lengths(self, length: int) -> None:
        """Every sequence back to `length` cached positions (device and host)."""
        self.seq_len.fill_(length)
        self._host_len = length
        self.reserve(1)

    def reserve(self, steps: int) -> None:
        """Paged KV: give every sequence pages for the next `steps` decode
        steps (positions < current length + steps). The length is tracked on
        the host (set_state / fill_kv_random, +1 per step()); call this before
        replaying a captured step several times. No-op for contiguous pools."""
        if self.block_table is None:
            return
        self.block_table.ensure(range(self.B), min(self._host_len + steps, self.L_cap))
        self.block_table.sync()

    def write_kv(self, layer: int, model: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Store a contiguous history k / v [slots, heads, L, 128] of one model's
        sequences (slots in routed order) into the layer's pools."""
        L = k.shape[2]
        if self.block_table is None:
            self.kpool[layer][model][:, :, :L].copy_(k)
            self.vpool[layer][model][:, :, :L].copy_(v)
            return
        ps = self.page_size
        base = 0 if model == 0 else self.counts_host[0]
        for s in range(k.shape[0]):
            pages = self.block_table.pages_of(base + s)
            if len(pages) * ps < L:
                raise ValueError("reserve pages before writing the history")
            for i in range(-(-L // ps)):
                n = min(ps, L - i * ps)
                self.kpool[layer][model][pages[i], :, :n].copy_(k[s, :, i * ps:i * ps + n])
                self.vpool[layer][model][pages[i], :, :n].copy_(v[s, :, i * ps:i * ps + n])

    def read_kv(self, layer: int, model: int, L: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The contiguous history [slots, heads, L, 128] of one model's sequences."""
        if self.block_table is None:
            return (self.kpool[layer][model][:, :, :L].clone(),
                    self.vpool[layer][model][:, :, :L].clone())
        ps = self.page_size
        base = 0 if model == 0 else self.counts_host[0]
        n = self.counts_host[model]
        k = torch.empty(n, self.nh, L, 128, dtype=self.dt, device=self.device)
        v = torch.empty_like(k)
        for s in range(n):
            pages = self.block_table.pages_of(base + s)
            for i in range(-(-L // ps)):
                c = min(ps, L - i * ps)
                k[s, :, i * ps:i * ps + c] = self.kpool[layer][model][pages[i], :, :c]
                v[s, :, i * ps:i * ps + c] = self.vpool[layer][model][pages[i], :, :c]
        return k, v

    # ------------------------------------------------------------ launches
    def _gemm(self, x, W, out, counts, *, residual=None, epilogue=0, M=None) -> None:
        Mr = x.shape[0] if M is None else M
        K, N = W.shape[-2], W.shape[-1]
        out_ptr = out if isinstance(out, int) else ptr(out)
        ws = self._ws_gemm
        check(lib.ps_routed_gemm(ptr(x), ptr(W), out_ptr, Mr, K, N, 0, ptr(counts), None,
                                 ptr(residual), epilogue, _lib.dtype_code(self.dt),
                                 ptr(ws), ws.numel(), ptr(self.status),
                                 _lib.stream_handle(self.device)), "ps_routed_gemm")

    @property
    def _rows_bound(self) -> int:
        """Rows of either model in a decode launch (0 in a prefill: unbounded)."""
        return 0 if self._in_prefill else max(self.counts_host)

    def _host_split(self, counts, M: int):
        """The decode step's split as a host value when it is known without
        reading the device (the model ids are fixed per decoder): the GEMM can
        then load its first weight stages before the preceding kernel ends.
        None for prefill chunks (their counts vary)."""
        if self._in_prefill:
            return None
        if counts is self.counts:
            return self.counts_host[0]
        if counts is self.counts_serial[0]:
            return M
        if counts is self.counts_serial[1]:
            return 0
        return None

    def _gemm_ex(self, x, W, out, counts, epi, M=None) -> None:
        Mr = x.shape[0] if M is None else M
        w_ptr, K, N = _wargs(W, epi)
        epi.max_model_rows = self._rows_bound
        out_ptr = out if isinstance(out, int) else ptr(out)
        ws = self._ws_gemm
        split = self._host_split(counts, Mr)
        cnt = None if split is not None else ptr(counts)
        epi.max_ctas = -1 if (self.auto_grid and not self._in_prefill) else 0
        check(lib.ps_routed_gemm_ex(ptr(x), w_ptr, out_ptr, Mr, K, N, split or 0, cnt,
                                    ctypes.byref(epi), _lib.dtype_code(self.dt), ptr(ws),
                                    ws.numel(), ptr(self.status),
                                    _lib.stream_handle(self.device)), "ps_routed_gemm_ex")

    @property
    def _ws_gemm(self) -> torch.Tensor:
        return self._pf["gemm_ws"] if self._in_prefill else self.gemm_ws

    def _rms(self, x, w, out, counts) -> None:
        check(lib.ps_rmsnorm_routed(ptr(x), ptr(w), ptr(out), x.shape[0], x.shape[1], 0,
                                    ptr(counts), float(self.cfg.eps), _lib.dtype_code(self.dt),
                                    ptr(self.status), _lib.stream_handle(self.device)),
              "ps_rmsnorm_routed")

    def _allreduce(self, t: torch.Tensor) -> None:
        import torch.distributed as dist
        dist.all_reduce(t, group=self.tp_group)

    def _row_split_reduce(self, inp, W, x, counts) -> None:
        """x += sum over ranks of inp @ W_shard: the GEMM writes this rank's
        partial into its NVLink slot, the all-reduce adds all ranks' partials
        and the residual in one pass (slots alternate call by call)."""
        slot = self._slot
        self._slot ^= 1
        self._gemm_ex(inp, W, self.ar.slot_ptr(slot), counts,
                      ops.gemm_epilogue(_lib.PS_EPI_STORE), M=x.shape[0])
        self.ar(slot, x.numel(), x, residual=x)

    def _layers_fused(self, rows: slice, counts: torch.Tensor) -> None:
        """All decoder layers for the token rows `rows` (routed order) under
        `counts`, 5 launches per layer (7 under tensor parallelism)."""
        bt = None if self.block_table is None else self.block_table.device[rows]
        self._run_layers(self.x[rows], self.q[rows], self.attn[rows], self.a[rows],
                         self.sq_emb[rows], self.sq_a[rows], self.sq_b[rows], self.pos[rows],
                         counts, bt, None)

    def _run_layers(self, x, q, attn, a, sq_in, sq_a, sq_b, pos, counts, bt, kv_rows) -> None:
        """The fused layer stack over rows x (routed order). sq_in: the sums of
        squares of x's rows (embedding output); kv_rows: each row's KV home
        (slot, or block-table row when paged) if rows share sequences."""
        H, eps = self.cfg.hidden, float(self.cfg.eps)
        for li, L in enumerate(self.layers):
            kp, vp = tuple(self.kpool[li]), tuple(self.vpool[li])
            e = ops.gemm_epilogue(_lib.PS_EPI_QKV_ROPE, in_sumsq=sq_in, norm_dim=H, eps=eps,
                                  k_pools=kp, v_pools=vp, pos=pos, rope_cos=self.rope_cos,
                                  rope_sin=self.rope_sin, n_heads=self.nh, block_table=bt,
                                  kv_rows=kv_rows)
            self._gemm_ex(x, L["W_qkv"], q, counts, e)
            self._attention(q, kp, vp, attn, pos, counts, bt, kv_rows)
            self._residual_proj(attn, L["W_o"], x, counts, sq_b)
            e = ops.gemm_epilogue(_lib.PS_EPI_SWIGLU, in_sumsq=sq_b, norm_dim=H, eps=eps)
            self._gemm_ex(x, L["W_gu"], a, counts, e)
            self._residual_proj(a, L["W_d"], x, counts, sq_a)
            sq_in = sq_a

    def _attention(self, q, kp, vp, attn, pos, counts, bt, kv_rows=None) -> None:
        k0, k1 = kp
        v0, v1 = vp
        s0 = 0 if k0 is None else k0.shape[0]
        s1 = 0 if k1 is None else k1.shape[0]
        M = q.shape[0]
        scale = 1.0 / math.sqrt(128)
        stream = _lib.stream_handle(self.device)
        dtc = _lib.dtype_code(self.dt)
        ws = self._pf["attn_ws"] if self._in_prefill else self.attn_ws
        if self._in_prefill:
            # prompt tokens: causal attention on the tensor cores, per run of
            # <= 128 tokens of one sequence
            paged = bt is not None
            check(lib.ps_prefill_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1), ptr(attn),
                                           ptr(self._pf["qblocks"]), self._pf_nblocks, M,
                                           self.nh, self.L_cap, s0, s1, ptr(bt),
                                           bt.shape[0] if paged else 0,
                                           self.max_pages if paged else 0,
                                           self.page_size if paged else 0, scale, dtc,
                                           ptr(self.status), stream), "ps_prefill_attention")
            return
        if bt is None:
            check(lib.ps_decode_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1), ptr(attn),
                                          ptr(pos), ptr(kv_rows), ptr(counts), 0, M, self.nh,
                                          self.L_cap, s0, s1, self.L_cap, 0, scale, dtc, ptr(ws),
                                          ws.numel(), ptr(self.status), stream),
                  "ps_decode_attention")
        else:
            check(lib.ps_paged_decode_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1),
                                                ptr(attn), ptr(pos), ptr(bt), bt.shape[0],
                                                ptr(kv_rows), self.max_pages, self.page_size,
                                                ptr(counts), 0, M, self.nh, s0, s1, self.L_cap, 0,
                                                scale, dtc, ptr(ws), ws.numel(),
                                                ptr(self.status), stream),
                  "ps_paged_decode_attention")

    def _residual_proj(self, inp, W, x, counts, sq_out) -> None:
        """x += inp @ W (summed over ranks), and the per-row sums of squares of
        the new x into sq_out."""
        if self.tp == 1:
            e = ops.gemm_epilogue(_lib.PS_EPI_STORE, residual=x, out_sumsq=sq_out)
            self._gemm_ex(inp, W, x, counts, e)
        else:
            slot = self._slot
            self._slot ^= 1
            self._gemm_ex(inp, W, self.ar.slot_ptr(slot), counts,
                          ops.gemm_epilogue(_lib.PS_EPI_STORE), M=x.shape[0])
            self.ar(slot, x.numel(), x, residual=x, out_sumsq=sq_out)

    def _layers(self, rows: slice, counts: torch.Tensor) -> None:
        """All decoder layers for the token rows `rows` (routed order) under
        `counts`, with separate norm and RoPE launches (8 per layer)."""
        if self.fused:
            return self._layers_fused(rows, counts)
        x, xa = self.x[rows], self.x_alt[rows]
        h, qkv, q, attn, a = (self.h[rows], self.qkv[rows], self.q[rows], self.attn[rows],
                              self.a[rows])
        pos = self.pos[rows]
        M = x.shape[0]
        stream = _lib.stream_handle(self.device)
        dtc = _lib.dtype_code(self.dt)
        scale = 1.0 / math.sqrt(128)
        for li, L in enumerate(self.layers):
            k0, k1 = self.kpool[li]
            v0, v1 = self.vpool[li]
            s0 = 0 if k0 is None else k0.shape[0]
            s1 = 0 if k1 is None else k1.shape[0]
            self._rms(x, L["ln1"], h, counts)
            self._gemm(h, L["W_qkv"], qkv, counts)
            check(lib.ps_rope_kv_append(ptr(qkv), ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1),
                                        ptr(self.rope_cos), ptr(self.rope_sin), ptr(pos), None,
                                        ptr(counts), 0, M, self.nh, self.L_cap, s0, s1, 1, dtc,
                                        ptr(self.status), stream), "ps_rope_kv_append")
            check(lib.ps_decode_attention(ptr(q), ptr(k0), ptr(v0), ptr(k1), ptr(v1), ptr(attn),
                                          ptr(pos), None, ptr(counts), 0, M, self.nh, self.L_cap,
                                          s0, s1, self.L_cap, 0, scale, dtc, ptr(self.attn_ws),
                                          self.attn_ws.numel(), ptr(self.status), stream),
                  "ps_decode_attention")
            if self.tp == 1:
                self._gemm(attn, L["W_o"], x, counts, residual=x)
            elif self.ar is not None:
                self._row_split_reduce(attn, L["W_o"], x, counts)
            else:
                self._gemm(attn, L["W_o"], xa, counts, residual=x if self.rank == 0 else None)
                self._allreduce(xa)
                x, xa = xa, x
            self._rms(x, L["ln2"], h, counts)
            self._gemm(h, L["W_gu"], a, counts, epilogue=_lib.PS_EPI_SWIGLU)
            if self.tp == 1:
                self._gemm(a, L["W_d"], x, counts, residual=x)
            elif self.ar is not None:
                self._row_split_reduce(a, L["W_d"], x, counts)
            else:
                self._gemm(a, L["W_d"], xa, counts, residual=x if self.rank == 0 else None)
                self._allreduce(xa)
                x, xa = xa, x
        if x.data_ptr() != self.x[rows].data_ptr():
            self.x[rows].copy_(x)

    def _layers_and_head(self, rows: slice, counts: torch.Tensor) -> None:
        if self.use_chain and self.layers:
            self._layers_chain(rows, counts)
        else:
            self._layers(rows, counts)
            self._head(rows, counts)

    def _chain_jobs(self, rows: slice, li: int, xbuf: torch.Tensor | None = None):
        """The job array of layer li's projection chain over token rows `rows`:
        O (+ residual), [all-reduce], gate_up (+ folded norm, SwiGLU), down
        (+ residual), [all-reduce], then layer li+1's QKV (+ norm, RoPE, KV
        append) or, after the last layer, the LM head (+ final norm).
        Built once per (rows, layer) and cached: every pointer is static.
        ``xbuf`` replaces the residual stream x (timing runs use a scratch copy)."""
        xb = self.x if xbuf is None else xbuf
        key = (rows.start, rows.stop, li, xb.data_ptr())
        if key in self._chains:
            return self._chains[key]
        H, eps = self.cfg.hidden, float(self.cfg.eps)
        L = self.layers[li]
        x, attn, a = xb[rows], self.attn[rows], self.a[rows]
        sq_a, sq_b, q, pos = self.sq_a[rows], self.sq_b[rows], self.q[rows], self.pos[rows]
        bt = None if self.block_table is None else self.block_table.device[rows]
        STORE, SWIGLU, QKV = _lib.PS_EPI_STORE, _lib.PS_EPI_SWIGLU, _lib.PS_EPI_QKV_ROPE
        jobs, keep = [], []

        def gemm(xx, W, y, epi, x_from=-1, norm_from=-1, res_from=-1):
            j = _lib.ChainJob()
            j.kind = _lib.PS_JOB_GEMM
            w_ptr, j.K, j.N = _wargs(W, epi)
            j.x, j.W, j.y = ptr(xx), w_ptr, (y if isinstance(y, int) else ptr(y))
            epi.max_model_rows = max(self.counts_host)
            j.epi = epi
            j.x_from, j.norm_from, j.res_from = x_from, norm_from, res_from
            j.src = j.slot = j.row_elems = 0
            keep.append(epi)
            jobs.append(j)
            return len(jobs) - 1

        def allreduce(src, slot, res_from=-1, out_sumsq=None):
            j = _lib.ChainJob()
            j.kind = _lib.PS_JOB_ALLREDUCE
            j.x_from = j.norm_from = -1
            j.res_from = res_from
            j.src, j.slot = src, slot
            j.out, j.residual, j.out_sumsq = ptr(x), ptr(x), ptr(out_sumsq)
            j.row_elems = H
            jobs.append(j)
            return len(jobs) - 1

        if self.tp == 1:
            o = gemm(attn, L["W_o"], x, ops.gemm_epilogue(STORE, residual=x, out_sumsq=sq_b))
            xo = o
            gu = gemm(x, L["W_gu"], a, ops.gemm_epilogue(SWIGLU, in_sumsq=sq_b, norm_dim=H,
                                                         eps=eps), x_from=o, norm_from=o)
            d = gemm(a, L["W_d"], x, ops.gemm_epilogue(STORE, residual=x, out_sumsq=sq_a),
                     x_from=gu, res_from=o)
            xd = d
        else:
            o = gemm(attn, L["W_o"], self.ar.slot_ptr(0), ops.gemm_epilogue(STORE))
            xo = allreduce(o, 0, out_sumsq=sq_b)
            gu = gemm(x, L["W_gu"], a, ops.gemm_epilogue(SWIGLU, in_sumsq=sq_b, norm_dim=H,
                                                         eps=eps), x_from=xo, norm_from=xo)
            d = gemm(a, L["W_d"], self.ar.slot_ptr(1), ops.gemm_epilogue(STORE), x_from=gu)
            xd = allreduce(d, 1, res_from=xo, out_sumsq=sq_a)
        if li + 1 < len(self.layers):
            nl = li + 1
            e = ops.gemm_epilogue(QKV, in_sumsq=sq_a, norm_dim=H, eps=eps,
                                  k_pools=tuple(self.kpool[nl]), v_pools=tuple(self.vpool[nl]),
                                  pos=pos, rope_cos=self.rope_cos, rope_sin=self.rope_sin,
                                  n_heads=self.nh, block_table=bt)
            gemm(x, self.layers[nl]["W_qkv"], q, e, x_from=xd, norm_from=xd)
        else:
            e = ops.gemm_epilogue(STORE, in_sumsq=sq_a, norm_dim=H, eps=eps)
            gemm(x, self.W_lm, self.logits[rows], e, x_from=xd, norm_from=xd)
        arr = (_lib.ChainJob * len(jobs))(*jobs)
        self._chains[key] = (arr, len(jobs), keep)
        return self._chains[key]

    def _layers_chain(self, rows: slice, counts: torch.Tensor, *, attention: bool = True,
                      xbuf: torch.Tensor | None = None) -> None:
        """All decoder layers and the LM head for the token rows `rows` in
        2 launches per layer: attention, then one projection chain (O, gate_up,
        down, next QKV or LM head, and the all-reduces under tensor
        parallelism); layer 0's QKV is one routed GEMM after the embedding.
        ``attention=False`` / ``xbuf`` launch the projections alone over a
        scratch residual stream (per-kernel-class timing)."""
        H, eps = self.cfg.hidden, float(self.cfg.eps)
        x = (self.x if xbuf is None else xbuf)[rows]
        q, attn, pos = self.q[rows], self.attn[rows], self.pos[rows]
        bt = None if self.block_table is None else self.block_table.device[rows]
        M = x.shape[0]
        e = ops.gemm_epilogue(_lib.PS_EPI_QKV_ROPE, in_sumsq=self.sq_emb[rows], norm_dim=H,
                              eps=eps, k_pools=tuple(self.kpool[0]), v_pools=tuple(self.vpool[0]),
                              pos=pos, rope_cos=self.rope_cos, rope_sin=self.rope_sin,
                              n_heads=self.nh, block_table=bt)
        self._gemm_ex(x, self.layers[0]["W_qkv"], q, counts, e)
        stream = _lib.stream_handle(self.device)
        if self.ar is not None:
            peers, rank, world, sb = self.ar.peers, self.ar.rank, self.ar.world, self.ar.slot_bytes
        else:
            peers, rank, world, sb = None, 0, 1, 0
        for li in range(len(self.layers)):
            if attention:
                self._attention(q, tuple(self.kpool[li]), tuple(self.vpool[li]), attn, pos,
                                counts, bt)
            arr, n, _ = self._chain_jobs(rows, li, xbuf)
            check(lib.ps_routed_chain(arr, n, M, ptr(counts), peers, rank, world, sb,
                                      _lib.dtype_code(self.dt), ptr(self.chain_ws),
                                      self.chain_ws.numel(), ptr(self.status), stream),
                  "ps_routed_chain")

    def _head(self, rows: slice, counts: torch.Tensor, sq: torch.Tensor | None = None) -> None:
        if self.fused:
            if sq is None:
                sq = self.sq_a[rows] if self.layers else self.sq_emb[rows]
            e = ops.gemm_epilogue(_lib.PS_EPI_STORE, in_sumsq=sq, norm_dim=self.cfg.hidden,
                                  eps=float(self.cfg.eps))
            self._gemm_ex(self.x[rows], self.W_lm, self.logits[rows], counts, e)
            return
        self._rms(self.x[rows], self.ln_f, self.h[rows], counts)
        self._gemm(self.h[rows], self.W_lm, self.logits[rows], counts)

    def step_device(self, mode: str = "fused") -> None:
        """Enqueue one decode step on the current stream (no host sync)."""
        stream = _lib.stream_handle(self.device)
        B = self.B
        check(lib.ps_route_partition(ptr(self.model_id), B, ptr(self.perm), ptr(self.counts),
                                     ptr(self.status), stream), "ps_route_partition")
        check(lib.ps_positions_routed(ptr(self.seq_len), ptr(self.perm), ptr(self.pos), B, stream),
              "ps_positions_routed")
        check(lib.ps_embed_routed(ptr(self.emb), ptr(self.tokens), ptr(self.perm), ptr(self.counts),
                                  ptr(self.x), B, self.cfg.hidden, self.cfg.vocab,
                                  ptr(self.sq_emb) if self.fused else None,
                                  _lib.dtype_code(self.dt), ptr(self.status), stream),
              "ps_embed_routed")
        if mode == "fused":
            self._layers_and_head(slice(0, B), self.counts)
        elif mode == "serial":
            c0 = self.counts_host[0]
            for m, rows in ((0, slice(0, c0)), (1, slice(c0, B))):
                if rows.stop > rows.start:
                    self._layers_and_head(rows, self.counts_serial[m])
        else:
            raise ValueError(mode)
        if self.tp == 1:
            check(lib.ps_argmax_rows(ptr(self.logits), ptr(self.perm), ptr(self.next_tokens),
                                     ptr(self.seq_len), B, self.cfg.vocab,
                                     _lib.dtype_code(self.dt), stream), "ps_argmax_rows")
        elif self.ar is not None:
            # one kernel: local (max, index), exchange over NVLink, pick, next
            # tokens written to both buffers, lengths += 1
            self.ar.pick(self.logits, self.perm, self.next_tokens, self.tokens, self.seq_len)
            return
        else:
            self._tp_argmax()
        self.tokens.copy_(self.next_tokens)

    def _tp_argmax(self) -> None:
        """Vocab-parallel greedy pick with NCCL (the allreduce='nccl' option):
        local (max, global index), all-gather, pick."""
        import torch.distributed as dist
        lg = self.logits.float()
        mx, ix = lg.max(dim=1)
        self.lm_best[:, 0] = mx
        self.lm_best[:, 1] = (ix + self.rank * self.Vl).float()
        dist.all_gather_into_tensor(self.lm_gather, self.lm_best, group=self.tp_group)
        vals = self.lm_gather[:, :, 0]
        best_rank = vals.argmax(dim=0)
        pick = self.lm_gather[best_rank, torch.arange(self.B, device=self.device), 1].to(torch.int32)
        self.next_tokens.index_copy_(0, self.perm.long(), pick)
        self.seq_len.add_(1)

    # ----------------------------------------------------------------- prefill
    def _prefill_buffers(self):
        if self._pf is not None:
            return self._pf
        C, H, dev, dt = self.prefill_chunk, self.cfg.hidden, self.device, self.dt
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        idx = dev.index or 0
        gw = max(lib.ps_routed_gemm_workspace_bytes(C, n, e, idx)
                 for n, e in ((3 * self.Hl, 0), (H, 0), (2 * self.FFl, 1), (self.Vl, 0)))
        with torch.cuda.device(dev):
            if self.page_size is None:
                aw = lib.ps_decode_attention_workspace_bytes(C, self.nh, self.L_cap, 0)
            else:
                aw = lib.ps_paged_decode_attention_workspace_bytes(C, self.nh, self.L_cap, 0,
                                                                   self.page_size)
        self._pf = dict(
            x=torch.zeros(C, H, dtype=dt, device=dev), q=torch.zeros(C, self.Hl, dtype=dt, device=dev),
            attn=torch.zeros(C, self.Hl, dtype=dt, device=dev),
            a=torch.zeros(C, self.FFl, dtype=dt, device=dev),
            sq_emb=torch.zeros(C, 1, **f32), sq_a=torch.zeros(C, self.sq_parts, **f32),
            sq_b=torch.zeros(C, self.sq_parts, **f32),
            tok=torch.zeros(C, **i32), pos=torch.zeros(C, **i32), kv_rows=torch.zeros(C, **i32),
            qblocks=torch.zeros(C, 5, **i32),
            counts=torch.zeros(2, **i32), pick_src=torch.zeros(self.B, **i32),
            pick_dst=torch.zeros(self.B, **i32),
            gemm_ws=torch.zeros(gw, dtype=torch.uint8, device=dev),
            attn_ws=torch.zeros(max(aw, 256), dtype=torch.uint8, device=dev))
        return self._pf

    def prefill(self, prompts) -> torch.Tensor:
        """Process every sequence's prompt (token lists in the original batch
        order, lengths 1..L_cap-1) through both models in routed launches of at
        most ``prefill_chunk`` tokens: the KV caches get positions [0, len),
        the last prompt token's logits give each sequence's first generated
        token (greedy). Afterwards ``seq_len`` = the prompt lengths and
        ``tokens`` = those first tokens, ready for ``step`` / ``step_device``.

        The reference measures decode only; this is the prefill of the
        decode loop. Each prompt token attends causally to its own
        sequence's cache (positions <= its own), written by the same fused QKV
        epilogue the decode step uses, so chunk boundaries do not change the
        result. Returns the first generated tokens (device, original order).
        """
        if not self.fused or not self.layers:
            raise ValueError("the prefill runs with the fused epilogues and at least one layer")
        B, H, dev = self.B, self.cfg.hidden, self.device
        if len(prompts) != B:
            raise ValueError(f"expected {B} prompts, got {len(prompts)}")
        pf = self._prefill_buffers()
        perm = self._perm_host.tolist()
        c0 = self.counts_host[0]
        lens = [len(prompts[s]) for s in perm]                       # routed order
        if min(lens) < 1 or max(lens) >= self.L_cap:
            raise ValueError(f"prompt lengths must be in [1, {self.L_cap - 1}]")
        if self.block_table is not None:
            self.block_table.ensure(range(B), max(lens) + 1)
            self.block_table.sync()
        chunks = prefill_layout(prompts, perm, c0, self.prefill_chunk,
                                paged=self.block_table is not None)
        stream = _lib.stream_handle(dev)
        dtc = _lib.dtype_code(self.dt)
        self._in_prefill = True
        try:
            for ch in chunks:
                n, n0 = len(ch["tok"]), ch["n0"]
                pf["tok"][:n].copy_(torch.tensor(ch["tok"], dtype=torch.int32))
                pf["pos"][:n].copy_(torch.tensor(ch["pos"], dtype=torch.int32))
                pf["kv_rows"][:n].copy_(torch.tensor(ch["kv_rows"], dtype=torch.int32))
                pf["counts"].copy_(torch.tensor([n0, n - n0], dtype=torch.int32))
                nb = len(ch["qblocks"])
                pf["qblocks"][:nb].copy_(torch.tensor(ch["qblocks"], dtype=torch.int32))
                self._pf_nblocks = nb
                x, sq_emb = pf["x"][:n], pf["sq_emb"][:n]
                check(lib.ps_embed_routed(ptr(self.emb), ptr(pf["tok"]), None, ptr(pf["counts"]),
                                          ptr(x), n, H, self.cfg.vocab, ptr(sq_emb), dtc,
                                          ptr(self.status), stream), "ps_embed_routed")
                bt = None if self.block_table is None else self.block_table.device
                self._run_layers(x, pf["q"][:n], pf["attn"][:n], pf["a"][:n], sq_emb,
                                 pf["sq_a"][:n], pf["sq_b"][:n], pf["pos"][:n], pf["counts"], bt,
                                 pf["kv_rows"][:n])
                # keep the final hidden row (and its norm statistics) of each
                # sequence whose last prompt token is in this chunk
                picks = ch["last"]
                if picks:
                    k = len(picks)
                    src = pf["pick_src"][:k]
                    dst = pf["pick_dst"][:k]
                    src.copy_(torch.tensor([a for a, _ in picks], dtype=torch.int32))
                    dst.copy_(torch.tensor([b for _, b in picks], dtype=torch.int32))
                    si, di = src.long(), dst.long()
                    self.x.index_copy_(0, di, x.index_select(0, si))
                    self.sq_last.index_copy_(0, di, pf["sq_a"][:n].index_select(0, si))
        finally:
            self._in_prefill = False
        # first generated token from the last prompt token of every sequence
        self.perm.copy_(self._perm_static)
        self.counts.copy_(self._counts_seq)
        self._head(slice(0, B), self._counts_seq, sq=self.sq_last)
        lens_orig = torch.tensor([len(p) for p in prompts], dtype=torch.int32)
        if self.tp == 1:
            check(lib.ps_argmax_rows(ptr(self.logits), ptr(self._perm_static),
                                     ptr(self.next_tokens), None, B, self.cfg.vocab, dtc, stream),
                  "ps_argmax_rows")
        elif self.ar is not None:
            self.ar.pick(self.logits, self._perm_static, self.next_tokens)
        else:
            self._tp_argmax()
        self.seq_len.copy_(lens_orig)
        self._host_len = int(lens_orig.max())
        self.tokens.copy_(self.next_tokens)
        self.reserve(1)
        return self.next_tokens

    def launches_per_step(self) -> int:
        """Kernels of this library one fused decode step launches (the torch
        copy of next -> tokens at one GPU and, with allreduce='nccl', the NCCL /
        torch ops of the greedy pick are not counted)."""
        nvlink = self.tp > 1 and self.ar is not None
        pick = 1 if (self.tp == 1 or nvlink) else 0
        if self.use_chain and self.layers:
            # layer 0's QKV, then attention + one projection chain per layer
            return 3 + 1 + 2 * len(self.layers) + pick
        if self.fused:
            per_layer, head = 5 + (2 if nvlink else 0), 1
        else:
            per_layer, head = 8 + (2 if nvlink else 0), 2
        return 3 + per_layer * len(self.layers) + head + pick

    # --------------------------------------------------------------- graphs
    def capture(self, mode: str = "fused") -> torch.cuda.CUDAGraph:
        """Capture one decode step as a CUDA graph (after an eager warm-up step
        that must be undone by the caller's state reset if it matters)."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step_device(mode)
        self.graphs[mode] = g
        return g

    def replay(self, mode: str = "fused") -> None:
        self.graphs[mode].replay()

    def release_graphs(self) -> None:
        self.graphs.clear()

    def close(self) -> None:
        """Release graphs and the NVLink all-reduce buffers (collective: every
        rank calls it)."""
        self.release_graphs()
        if self.ar is not None:
            torch.cuda.synchronize(self.device)
            import torch.distributed as dist
            dist.barrier(group=self.tp_group)
            self.ar.close()
            self.ar = None

    # --------------------------------------------------------- host-facing
    def step(self, tokens_host: torch.Tensor, out_host: torch.Tensor, mode: str = "fused") -> torch.Tensor:
        """Public decode step with host buffers: copies this step's input token
        ids (pinned int32 [B]) to the device, runs the step (graph if captured),
        and copies the greedy next tokens back into ``out_host`` (pinned int32 [B])."""
        self.reserve(1)
        self.tokens.copy_(tokens_host, non_blocking=True)
        if mode in self.graphs:
            self.graphs[mode].replay()
        else:
            self.step_device(mode)
        out_host.copy_(self.next_tokens, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self._host_len += 1
        return out_host

    def check_status(self) -> None:
        st = _lib.read_status(self.device)
        if st:
            raise _lib.PSError(f"device status bits 0x{st:x} raised during decode")
