"""ctypes binding of ``libparallel_serve.so`` (the C ABI in include/parallel_serve.h).

The product path has exactly one implementation: the sm_100a kernels in this
library. If the library is missing or cannot be loaded this module raises
immediately; there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libparallel_serve.so")

PS_OK = 0
PS_ERR_INVALID_ARGUMENT = 1
PS_ERR_WORKSPACE = 2
PS_ERR_CUDA = 3
PS_ERR_UNSUPPORTED = 4
PS_ERR_SCRATCH_LIMIT = 5

PS_ERR_TIMEOUT = 0x1
PS_ERR_BAD_MODEL_ID = 0x2
PS_ERR_BAD_INDEX = 0x4

PS_DTYPE_F16 = 0
PS_DTYPE_BF16 = 1
PS_EPI_STORE = 0
PS_EPI_SWIGLU = 1
PS_EPI_QKV_ROPE = 2
PS_AR_AUTO, PS_AR_ONE_SHOT, PS_AR_TWO_SHOT, PS_AR_TWO_SHOT_LL = 0, 1, 2, 3

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t


class GemmEpilogue(ctypes.Structure):
    """ps_gemm_epilogue_t (the fused epilogue of ps_routed_gemm_ex)."""
    _fields_ = [
        ("mode", _i), ("scatter_rows", _p), ("residual", _p), ("in_sumsq", _p),
        ("in_parts", _i), ("norm_dim", _i), ("eps", _f), ("out_sumsq", _p),
        ("k_pool0", _p), ("v_pool0", _p), ("k_pool1", _p), ("v_pool1", _p), ("pos", _p),
        ("rope_cos", _p), ("rope_sin", _p), ("n_heads", _i), ("L_cap", _i), ("slots0", _i),
        ("slots1", _i), ("apply_rope", _i), ("block_table", _p), ("max_pages", _i),
        ("page_size", _i), ("kv_rows", _p), ("table_rows", _i), ("max_model_rows", _i),
        ("w_packed", _p), ("max_ctas", _i),
    ]

PS_JOB_GEMM, PS_JOB_ALLREDUCE = 0, 1


class ChainJob(ctypes.Structure):
    """ps_chain_job_t (one job of ps_routed_chain)."""
    _fields_ = [
        ("kind", _i), ("x", _p), ("W", _p), ("y", _p), ("K", _i), ("N", _i),
        ("epi", GemmEpilogue), ("x_from", _i), ("norm_from", _i), ("res_from", _i),
        ("src", _i), ("slot", _i), ("out", _p), ("residual", _p), ("out_sumsq", _p),
        ("row_elems", _i),
    ]


# name -> (restype, argtypes); mirrors include/parallel_serve.h exactly.
SIGNATURES: dict[str, tuple] = {
    "ps_error_string": (ctypes.c_char_p, [_i]),
    "ps_version": (ctypes.c_char_p, []),
    "ps_device_sm_count": (_i, [_i]),
    "ps_route_partition": (_i, [_p, _i, _p, _p, _p, _p]),
    "ps_gather_rows": (_i, [_p, _p, _p, _i, _i, _p, _p]),
    "ps_scatter_rows": (_i, [_p, _p, _p, _i, _i, _p, _p]),
    "ps_routed_gemm_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "ps_routed_gemm": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _i, _i, _p, _sz, _p, _p]),
    "ps_routed_gemm_noalloc": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _i, _i, _p, _p]),
    "ps_routed_gemm_schedule": (_i, [_i, _i, _i, _i, _i, _i, _p]),
    "ps_routed_gemm_cta_work": (_i, [_i, _i, _i, _i, _i, _i, _i, _p, _i]),
    "ps_routed_gemm_tile": (_i, [_i, _i, _i, _i, _i, _i, _i, _p]),
    "ps_routed_gemm_ex": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, ctypes.POINTER(GemmEpilogue), _i,
                               _p, _sz, _p, _p]),
    "ps_rmsnorm_routed": (_i, [_p, _p, _p, _i, _i, _i, _p, _f, _i, _p, _p]),
    "ps_swiglu": (_i, [_p, _p, _i, _i, _i, _p]),
    "ps_rope_kv_append": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i,
                               _i, _i, _i, _p, _p]),
    "ps_decode_attention_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "ps_decode_attention": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i,
                                 _i, _f, _i, _p, _sz, _p, _p]),
    "ps_paged_decode_attention_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "ps_paged_decode_attention": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _i, _p, _i, _i, _p, _i,
                                       _i, _i, _i, _i, _i, _i, _f, _i, _p, _sz, _p, _p]),
    "ps_segment_attention": (_i, [_p, _p, _i, _i, _i, _p, _f, _i, _p, _p]),
    "ps_prefill_attention": (_i, [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _i,
                                  _i, _i, _f, _i, _p, _p]),
    "ps_deltazip_packed_bytes": (_sz, [_i, _i]),
    "ps_deltazip_workspace_bytes": (_sz, [_i, _i, _i]),
    "ps_deltazip_linear": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _p, _i, _p, _sz, _p, _p]),
    "ps_symm_region_bytes": (_sz, [_sz]),
    "ps_symm_alloc": (_i, [_sz, ctypes.POINTER(_p), _p]),
    "ps_symm_open": (_i, [_p, ctypes.POINTER(_p)]),
    "ps_symm_close": (_i, [_p]),
    "ps_symm_free": (_i, [_p]),
    "ps_allreduce_sum": (_i, [_p, _i, _i, _i, _sz, _sz, _p, _p, _p, _i, _p, _i, _i, _p, _p]),
    "ps_symm_slot_offset": (_sz, [_i, _sz]),
    "ps_argmax_tp": (_i, [_p, _p, _p, _p, _p, _i, _i, _p, _i, _i, _sz, _p, _i, _p, _p]),
    "ps_packed_weights_bytes": (_sz, [_i, _i, _i, _i]),
    "ps_pack_weights": (_i, [_p, _i, _i, _i, _i, _p, _sz, _p]),
    "ps_routed_chain_workspace_bytes": (_sz, [_i, _i, _i]),
    "ps_routed_chain": (_i, [ctypes.POINTER(ChainJob), _i, _i, _p, _p, _i, _i, _sz, _i, _p,
                             _sz, _p, _p]),
    "ps_embed_routed": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _p, _i, _p, _p]),
    "ps_argmax_rows": (_i, [_p, _p, _p, _p, _i, _i, _i, _p]),
    "ps_positions_routed": (_i, [_p, _p, _p, _i, _p]),
}


class PSError(RuntimeError):
    """A parallel-serve entry point returned a non-zero PS_* code."""


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python parallel_serve_b200/build.py` "
            "(nvcc, sm_100a). parallel-serve has no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(rc: int, what: str) -> None:
    if rc != PS_OK:
        raise PSError(f"{what}: {lib.ps_error_string(rc).decode()} (code {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | int | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return PS_DTYPE_F16
    if dtype == torch.bfloat16:
        return PS_DTYPE_BF16
    raise TypeError(f"parallel-serve kernels take float16 or bfloat16, got {dtype}")


_lock = threading.Lock()
_status: dict[int, torch.Tensor] = {}
_workspaces: dict[tuple[int, int, str], torch.Tensor] = {}


def status_tensor(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word that kernels OR their PS_ERR_* bits into."""
    idx = torch.device(device).index or 0
    with _lock:
        t = _status.get(idx)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _status[idx] = t
        return t


def read_status(device: torch.device, clear: bool = True) -> int:
    """Synchronizes, returns the device status bits and (by default) clears them."""
    t = status_tensor(device)
    torch.cuda.synchronize(t.device)
    v = int(t.item())
    if clear and v:
        t.zero_()
    return v


def workspace(device: torch.device, nbytes: int, tag: str) -> torch.Tensor:
    """Zero-initialised scratch buffer cached per (device, current stream, tag).

    Kernels that use it leave their arrival counters at zero, so it is zeroed
    only when first allocated or grown.
    """
    dev = torch.device(device)
    idx = dev.index or 0
    key = (idx, torch.cuda.current_stream(dev).cuda_stream, tag)
    with _lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[key] = buf
        return buf
