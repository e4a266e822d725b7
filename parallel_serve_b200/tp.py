"""Tensor-parallel plumbing: NVLink peer-memory all-reduce for the row-split
projections of the decode step.

QKV / gate_up are split by columns and O / down by rows (Megatron-style), with
an all-reduce of the row-split outputs. ``NvlinkAllReduce`` keeps one symmetric
region per rank (allocated by the C library, shared with CUDA IPC; handles
exchanged once through ``torch.distributed``) and sums the ranks' partials
with ``ps_allreduce_sum``: one launch that reads every peer's slot over
NVLink (one-shot, the default) or reduces this rank's share and pushes it to
every rank (two-shot, or the low-latency two-shot whose 8-byte {data, epoch}
words need no second barrier; both on request). Ranks are summed in a fixed
order so all ranks hold identical results, and the residual is added in the
same pass. A row-split GEMM writes its partial straight into
``slot_ptr(slot)``; consecutive calls alternate the slot.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib

__all__ = ["NvlinkAllReduce"]


class NvlinkAllReduce:
    def __init__(self, group, max_elems: int, device: torch.device, dtype: torch.dtype,
                 algo: int = _lib.PS_AR_AUTO):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("NvlinkAllReduce supports up to 8 ranks (one NVLink domain)")
        self.device = torch.device(device)
        self.dtype_code = _lib.dtype_code(dtype)
        self.algo = algo
        self.slot_bytes = (max_elems * 2 + 255) // 256 * 256
        region = lib.ps_symm_region_bytes(self.slot_bytes)
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            check(lib.ps_symm_alloc(region, ctypes.byref(ptr), handle), "ps_symm_alloc")
        self._local = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        peers = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    peers.append(self._local)
                else:
                    p = ctypes.c_void_p()
                    check(lib.ps_symm_open(h, ctypes.byref(p)), "ps_symm_open")
                    self._opened.append(p.value)
                    peers.append(p.value)
        self.peers = (ctypes.c_void_p * self.world)(*peers)
        self.epochs = torch.zeros(128, dtype=torch.int32, device=self.device)
        # per-row epochs of the greedy-pick exchange (allocated here, never
        # inside a stream capture: a zero-fill captured into a graph would
        # reset them on every replay)
        self._pick_epochs = torch.zeros(4096, dtype=torch.int32, device=self.device)
        self.status = _lib.status_tensor(self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)   # every region is zeroed before anyone signals

    def slot_ptr(self, slot: int) -> int:
        return self._local + lib.ps_symm_slot_offset(slot, self.slot_bytes)

    def __call__(self, slot: int, count: int, out: torch.Tensor,
                 residual: torch.Tensor | None = None, *,
                 out_sumsq: torch.Tensor | None = None) -> None:
        """out = residual + sum over ranks of slot `slot`. With `out_sumsq`
        (fp32 [rows, out.shape[-1] // 256]) the sums of squares of each row's
        256-element parts are stored there (the next folded RMSNorm's input)."""
        check(lib.ps_allreduce_sum(self.peers, self.rank, self.world, slot, self.slot_bytes,
                                   count, out.data_ptr(),
                                   None if residual is None else residual.data_ptr(),
                                   self.epochs.data_ptr(), out.shape[-1],
                                   None if out_sumsq is None else out_sumsq.data_ptr(),
                                   self.algo, self.dtype_code,
                                   self.status.data_ptr(), _lib.stream_handle(self.device)),
              "ps_allreduce_sum")

    def pick(self, logits: torch.Tensor, perm: torch.Tensor | None, next_tokens: torch.Tensor,
             tokens_out: torch.Tensor | None = None, seq_len: torch.Tensor | None = None) -> None:
        """Vocab-parallel greedy pick (``ps_argmax_tp``): logits [M, V_local] of
        this rank's vocabulary shard (routed rows); every rank writes the same
        next_tokens[perm[j]] (and tokens_out, seq_len += 1 when given)."""
        M, V = logits.shape
        check(lib.ps_argmax_tp(logits.data_ptr(), None if perm is None else perm.data_ptr(),
                               next_tokens.data_ptr(),
                               None if tokens_out is None else tokens_out.data_ptr(),
                               None if seq_len is None else seq_len.data_ptr(), M, V,
                               self.peers, self.rank, self.world, self.slot_bytes,
                               self._pick_epochs.data_ptr(), _lib.dtype_code(logits.dtype),
                               self.status.data_ptr(), _lib.stream_handle(self.device)),
              "ps_argmax_tp")

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.ps_symm_close(p)
            self._opened = []
            if self._local:
                lib.ps_symm_free(self._local)
                self._local = None
