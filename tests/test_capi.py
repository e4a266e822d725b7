"""The C ABI library loads on CPU and exports every entry point declared in
include/parallel_serve.h, with the ctypes signatures used by the package.
No compute entry point is called (there is no GPU here)."""
from __future__ import annotations

import ctypes
import os
import re

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "parallel_serve.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ps_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    from parallel_serve_b200 import _lib
    names = declared_functions()
    assert len(names) >= 15
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(raw, n), n


def test_python_binding_covers_the_header():
    from parallel_serve_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_pure_entry_points():
    from parallel_serve_b200 import _lib
    assert b"sm_100a" in _lib.lib.ps_version()
    for code in range(6):
        assert _lib.lib.ps_error_string(code) != b"unknown error"
    assert _lib.lib.ps_error_string(99) == b"unknown error"


def test_host_argument_checks_return_before_any_cuda_call():
    from parallel_serve_b200 import _lib
    L = _lib.lib
    assert L.ps_routed_gemm(None, None, None, -1, 8, 8, 0, None, None, None, 0, 0, None, 0,
                            None, None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert L.ps_routed_gemm(None, None, None, 4, 12, 8, 0, None, None, None, 0, 0, None, 0,
                            None, None) == _lib.PS_ERR_INVALID_ARGUMENT  # K % 8
    assert L.ps_routed_gemm(None, None, None, 4, 8, 8, 5, None, None, None, 0, 0, None, 0,
                            None, None) == _lib.PS_ERR_INVALID_ARGUMENT  # split > M
    assert L.ps_rmsnorm_routed(None, None, None, 2, 12, 0, None, 1e-5, 0, None,
                               None) == _lib.PS_ERR_INVALID_ARGUMENT  # H % 8
    assert L.ps_gather_rows(None, None, None, 3, 10, None, None) == _lib.PS_ERR_INVALID_ARGUMENT
    assert L.ps_decode_attention(None, None, None, None, None, None, None, None, None, 0, 4, 2,
                                 16, 2, 2, 32, 0, 1.0, 0, None, 0, None,
                                 None) == _lib.PS_ERR_INVALID_ARGUMENT  # max_len > L_cap


def test_fused_epilogue_argument_checks():
    """ps_routed_gemm_ex rejects inconsistent epilogue descriptors on the host."""
    import ctypes
    from parallel_serve_b200 import _lib
    L = _lib.lib

    def call(e, N=3 * 256):
        return L.ps_routed_gemm_ex(None, None, None, 4, 256, N, 4, None, ctypes.byref(e), 0,
                                   None, 0, None, None)
    e = _lib.GemmEpilogue(mode=_lib.PS_EPI_QKV_ROPE, n_heads=2, L_cap=8)
    assert call(e, N=512) == _lib.PS_ERR_INVALID_ARGUMENT      # N != 3 * heads * 128
    assert call(e) == _lib.PS_ERR_INVALID_ARGUMENT             # no positions
    e = _lib.GemmEpilogue(mode=_lib.PS_EPI_SWIGLU, out_sumsq=1024)
    assert call(e, N=512) == _lib.PS_ERR_INVALID_ARGUMENT      # sumsq only after STORE
    e = _lib.GemmEpilogue(mode=_lib.PS_EPI_STORE, in_sumsq=1024, in_parts=0, norm_dim=256)
    assert call(e, N=512) == _lib.PS_ERR_INVALID_ARGUMENT      # no partial count
    e = _lib.GemmEpilogue(mode=7)
    assert call(e) == _lib.PS_ERR_INVALID_ARGUMENT
    assert L.ps_routed_gemm_ex(None, None, None, 4, 256, 512, 4, None, None, 0, None, 0, None,
                               None) == _lib.PS_ERR_INVALID_ARGUMENT
    e = _lib.GemmEpilogue(mode=_lib.PS_EPI_STORE)
    assert L.ps_routed_gemm_ex(None, None, None, 0, 256, 512, 0, None, ctypes.byref(e), 0, None,
                               0, None, None) == _lib.PS_OK


def test_new_entry_points_check_arguments_on_the_host():
    from parallel_serve_b200 import _lib
    L = _lib.lib
    bad = _lib.PS_ERR_INVALID_ARGUMENT
    # prefill attention: bad dtype / heads, and a no-op for empty input
    assert L.ps_prefill_attention(None, None, None, None, None, None, None, 1, 8, 2, 64, 1, 0,
                                  None, 0, 0, 0, 1.0, 7, None, None) == bad
    assert L.ps_prefill_attention(None, None, None, None, None, None, None, 1, 8, 0, 64, 1, 0,
                                  None, 0, 0, 0, 1.0, 0, None, None) == bad
    assert L.ps_prefill_attention(None, None, None, None, None, None, None, 0, 0, 2, 64, 1, 0,
                                  None, 0, 0, 0, 1.0, 0, None, None) == _lib.PS_OK
    # paged attention: page size must be a power of two in [8, 4096]
    assert L.ps_paged_decode_attention(None, None, None, None, None, None, None, None, 1, None, 4,
                                       12, None, 0, 1, 2, 1, 0, 32, 0, 1.0, 0, None, 0, None,
                                       None) == bad
    assert L.ps_paged_decode_attention_workspace_bytes(4, 2, 64, 0, 12) == 0
    # all-reduce: algorithm and slot range
    peers = (ctypes.c_void_p * 2)(16, 32)
    assert L.ps_allreduce_sum(peers, 0, 2, 0, 1024, 8, None, None, None, 0, None, 5, 0, None,
                              None) == bad
    assert L.ps_allreduce_sum(peers, 0, 2, 2, 1024, 8, None, None, None, 0, None, 0, 0, None,
                              None) == bad
    assert L.ps_symm_slot_offset(1, 1000) == L.ps_symm_slot_offset(0, 1000) + 1024


def test_zero_sized_calls_are_no_ops():
    from parallel_serve_b200 import _lib
    L = _lib.lib
    assert L.ps_routed_gemm(None, None, None, 0, 8, 8, 0, None, None, None, 0, 0, None, 0,
                            None, None) == _lib.PS_OK
    assert L.ps_swiglu(None, None, 0, 8, 0, None) == _lib.PS_OK


def test_later_entry_points_check_arguments_on_the_host():
    """The no-allocation GEMM, weight packing, the projection chain and the
    vocab-split pick refuse bad arguments (and treat empty work as a no-op)
    before any CUDA call."""
    from parallel_serve_b200 import _lib
    L = _lib.lib
    bad, ok = _lib.PS_ERR_INVALID_ARGUMENT, _lib.PS_OK
    STORE, SWIGLU, QKV = _lib.PS_EPI_STORE, _lib.PS_EPI_SWIGLU, _lib.PS_EPI_QKV_ROPE
    # ps_routed_gemm_noalloc(x, W, y, M, K, N, split, counts, scatter, residual, epi, dtype, st, s)
    a = (16, 32, 48)
    assert L.ps_routed_gemm_noalloc(*a, 8, 0, 64, 4, None, None, None, STORE, 0, None, None) == bad
    assert L.ps_routed_gemm_noalloc(*a, 8, 64, 64, 4, None, None, None, STORE, 5, None, None) == bad
    assert L.ps_routed_gemm_noalloc(*a, 8, 64, 64, 4, None, None, None, QKV, 0, None, None) == bad
    assert L.ps_routed_gemm_noalloc(*a, 8, 60, 64, 4, None, None, None, STORE, 0, None, None) == bad
    assert L.ps_routed_gemm_noalloc(*a, 8, 64, 72, 4, None, None, None, SWIGLU, 0, None,
                                    None) == bad                              # N % 16
    assert L.ps_routed_gemm_noalloc(*a, 8, 64, 64, 4, None, None, 64, SWIGLU, 0, None,
                                    None) == bad                              # residual
    assert L.ps_routed_gemm_noalloc(*a, 8, 64, 64, 9, None, None, None, STORE, 0, None,
                                    None) == bad                              # split > M
    assert L.ps_routed_gemm_noalloc(None, None, None, 0, 64, 64, 0, None, None, None, STORE, 0,
                                    None, None) == ok
    assert L.ps_routed_gemm_noalloc(None, 32, 48, 8, 64, 64, 4, None, None, None, STORE, 0,
                                    None, None) == bad
    assert L.ps_routed_gemm_noalloc(17, 32, 48, 8, 64, 64, 4, None, None, None, STORE, 0,
                                    None, None) == bad                        # misaligned x
    # packed weights: sizes follow the layout (128-column or 64+64 SwiGLU tiles, 128-k blocks)
    assert L.ps_packed_weights_bytes(2, 256, 384, STORE) == 2 * 3 * 2 * 32768
    assert L.ps_packed_weights_bytes(2, 384, 2 * 344, SWIGLU) == 2 * 6 * 3 * 32768
    assert L.ps_packed_weights_bytes(0, 256, 384, STORE) == 0
    need = L.ps_packed_weights_bytes(2, 256, 384, STORE)
    assert L.ps_pack_weights(16, 2, 252, 384, STORE, 32, need, None) == bad  # K % 8
    assert L.ps_pack_weights(16, 2, 256, 384, 9, 32, need, None) == bad
    assert L.ps_pack_weights(16, 2, 256, 392, SWIGLU, 32, 1 << 30, None) == bad  # N % 16
    assert L.ps_pack_weights(None, 2, 256, 384, STORE, 32, need, None) == bad
    assert L.ps_pack_weights(16, 2, 256, 384, STORE, 32, need - 16, None) == bad
    # projection chain: job count, rows, counts, dtype, ranks; no rows is a no-op
    jobs = (_lib.ChainJob * 7)()
    cnt = 64
    assert L.ps_routed_chain(None, 1, 8, cnt, None, 0, 1, 0, 0, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 0, 8, cnt, None, 0, 1, 0, 0, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 7, 8, cnt, None, 0, 1, 0, 0, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 1, 257, cnt, None, 0, 1, 0, 0, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 1, 8, None, None, 0, 1, 0, 0, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 1, 8, cnt, None, 0, 1, 0, 3, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 1, 8, cnt, None, 1, 1, 0, 0, None, 0, None, None) == bad
    assert L.ps_routed_chain(jobs, 1, 0, cnt, None, 0, 1, 0, 0, None, 0, None, None) == ok
    assert L.ps_routed_chain_workspace_bytes(0, 3, 0) == 0
    assert L.ps_routed_chain_workspace_bytes(8, 7, 0) == 0
    # vocab-split pick(logits, perm, next, tokens_out, seq_len, M, V, peers, rank, world,
    #                  slot_bytes, epochs, dtype, status, stream)
    peers = (ctypes.c_void_p * 2)(256, 512)
    args = dict(M=4, V=1000, rank=0, world=2, slot=1024, dtype=0)

    def pick(**kw):
        a = {**args, **kw}
        return L.ps_argmax_tp(kw.get("logits", 64), None, kw.get("nxt", 128), None, None,
                              a["M"], a["V"], kw.get("peers", peers), a["rank"], a["world"],
                              a["slot"], 192, a["dtype"], None, None)
    assert pick(world=0) == bad and pick(world=9) == bad and pick(rank=2) == bad
    assert pick(M=4097) == bad and pick(V=0) == bad and pick(dtype=7) == bad
    assert pick(slot=1000) == bad
    assert pick(M=0) == ok
    assert pick(logits=None) == bad and pick(nxt=None) == bad
    assert pick(peers=(ctypes.c_void_p * 2)(256, 520)) == bad             # misaligned peer
