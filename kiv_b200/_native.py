"""ctypes binding of ``libkiv_b200.so`` (the C ABI declared in ``include/kiv_b200.h``).

The library is the only compute path of this package: if it is missing or
cannot be loaded, every operation raises :class:`KIVNativeError` -- there is no
CPU or PyTorch fallback.  Tensors cross the boundary as raw device pointers
(``tensor.data_ptr()``), strides in elements, and the current CUDA stream.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkiv_b200.so")

KIV_OK = 0
KIV_DTYPE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
KEEP_NONE = -1
KEEP_DIRECT = -2

STATE_WORDS = 32
ST_COLD_LEN, ST_HOT_START, ST_HOT_LEN, ST_UNION, ST_CAND, ST_SEL, ST_SEL_LOCAL, ST_ERROR = range(8)
ST_COARSE_MAX, ST_COARSE_SUM, ST_FINE_MAX, ST_FINE_SUM = 8, 9, 10, 11
ST_PAGESUM_SLOT = 21   # replicated summaries: which page_sums slot holds the carried sum

c_i32, c_i64, c_f32, c_vp, c_sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class KIVNativeError(RuntimeError):
    """A C-ABI call failed (bad argument, capacity, CUDA error) or the library is missing."""


class StoreDesc(ctypes.Structure):
    _fields_ = [("batch", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
                ("page_size", c_i32), ("dtype", c_i32), ("shard_rank", c_i32),
                ("shard_count", c_i32), ("hot_hint", c_i32), ("cold_capacity", c_i64),
                ("hot_capacity", c_i64), ("cold_k", c_vp), ("cold_v", c_vp),
                ("summaries", c_vp), ("hot_k", c_vp), ("hot_v", c_vp), ("state", c_vp),
                ("host_capacity", c_i64), ("host_k", c_vp), ("host_v", c_vp), ("stage_pages", c_i32),
                ("flags", c_i32), ("page_sums", c_vp)]


STORE_REPL_SUMMARIES = 1


class QueryDesc(ctypes.Structure):
    _fields_ = [("q", c_vp), ("stride_b", c_i64), ("stride_h", c_i64), ("stride_t", c_i64),
                ("num_query_heads", c_i32), ("query_len", c_i32), ("scaling", c_f32),
                ("softcap", c_f32), ("top_pages", c_i32), ("top_p", c_i32)]


class MaskDesc(ctypes.Structure):
    _fields_ = [("add", c_vp), ("stride_b", c_i64), ("stride_h", c_i64), ("stride_t", c_i64),
                ("causal", c_i32), ("reserved", c_i32)]


MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class ExchangeDesc(ctypes.Structure):
    _fields_ = [("world", c_i32), ("rank", c_i32), ("arena", c_vp * MAX_PEERS), ("arena_bytes", c_i64),
                ("wait_cycles", c_i64)]


class PeerRows(ctypes.Structure):
    """kiv_peer_rows: every shard's cold_k / cold_v as mapped in this process."""
    _fields_ = [("cold_k", c_vp * MAX_PEERS), ("cold_v", c_vp * MAX_PEERS)]


P = ctypes.POINTER
# name -> (restype, argtypes)
SIGNATURES = {
    "kiv_abi_version": (c_i32, []),
    "kiv_host_alloc": (c_i32, [ctypes.c_size_t, ctypes.POINTER(c_vp)]),
    "kiv_host_free": (c_i32, [c_vp]),
    "kiv_status_string": (ctypes.c_char_p, [c_i32]),
    "kiv_last_error": (ctypes.c_char_p, []),
    "kiv_workspace_bytes": (c_sz, [P(StoreDesc), P(QueryDesc)]),
    "kiv_workspace_layout": (c_i32, [P(StoreDesc), P(QueryDesc), P(c_i64)]),
    "kiv_state_reset": (c_i32, [P(StoreDesc), c_vp]),
    "kiv_append_evict": (c_i32, [P(StoreDesc), c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_i64, c_i64, c_vp]),
    "kiv_coarse_select": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, c_vp]),
    "kiv_coarse_merge": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, c_i32, c_vp]),
    "kiv_fine_select": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, c_vp]),
    "kiv_fine_score": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp]),
    "kiv_fine_topk": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, c_vp]),
    "kiv_fine_merge": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, c_i32, c_vp, c_vp, c_vp]),
    "kiv_gather_rows": (c_i32, [P(StoreDesc), c_vp, c_i32, c_i32, c_vp, c_vp, c_vp]),
    "kiv_attend": (c_i32, [P(StoreDesc), P(QueryDesc), P(MaskDesc), c_vp, c_sz, c_vp, c_i32, c_i32,
                           c_i32, c_vp, c_vp, c_vp]),
    "kiv_attend_merge": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_i32, c_vp, c_vp]),
    "kiv_retrieve_attend": (c_i32, [P(StoreDesc), P(QueryDesc), P(MaskDesc), c_vp, c_sz, c_i32, c_vp,
                                    c_vp, c_vp]),
    "kiv_retrieve_attend_noalloc": (c_i32, [P(StoreDesc), P(QueryDesc), P(MaskDesc), c_vp, c_vp, c_vp]),
    "kiv_read_state": (c_i32, [P(StoreDesc), P(c_i64), c_vp]),
    "kiv_exchange_bytes": (c_sz, [P(StoreDesc), P(QueryDesc), c_i32]),
    "kiv_peer_alloc": (c_i32, [c_sz, P(c_vp), c_vp]),
    "kiv_peer_open": (c_i32, [c_vp, P(c_vp)]),
    "kiv_peer_close": (c_i32, [c_vp]),
    "kiv_peer_free": (c_i32, [c_vp]),
    "kiv_coarse_exchange_merge": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, P(ExchangeDesc),
                                          c_vp]),
    "kiv_fine_exchange_merge": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, c_vp, c_vp, P(ExchangeDesc),
                                        c_vp, c_vp, c_vp]),
    "kiv_attend_exchange_merge": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, P(ExchangeDesc), c_vp, c_vp]),
    "kiv_fine_exchange_supported": (c_i32, [P(StoreDesc), P(QueryDesc)]),
    "kiv_peer_export": (c_i32, [c_vp, c_vp, P(c_i64)]),
    "kiv_attend_peers": (c_i32, [P(StoreDesc), P(QueryDesc), P(MaskDesc), c_vp, c_sz, c_vp, c_i32, P(PeerRows),
                                 c_vp, c_vp]),
    "kiv_fine_exchange_select": (c_i32, [P(StoreDesc), P(QueryDesc), c_vp, c_sz, P(ExchangeDesc), c_vp, c_vp,
                                         c_vp]),
}

_lib = None
_lock = threading.Lock()


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and type the C ABI.  Raises KIVNativeError if it is absent."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or os.environ.get("KIV_B200_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise KIVNativeError(
                f"libkiv_b200.so not found at {p}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (make -C kiv_b200/csrc)")
        try:
            lib = ctypes.CDLL(p)
        except OSError as e:  # pragma: no cover - depends on the machine
            raise KIVNativeError(f"cannot load {p}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load_library()


def check(rc: int, what: str) -> None:
    if rc != KIV_OK:
        L = lib()
        msg = L.kiv_last_error().decode(errors="replace")
        status = L.kiv_status_string(rc).decode()
        raise KIVNativeError(f"{what}: {status} ({rc}): {msg}")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return KIV_DTYPE[dtype]
    except KeyError:
        raise KIVNativeError(f"dtype {dtype} is not supported (float32, bfloat16, float16)") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def query_desc(query: torch.Tensor, scaling: float, top_pages: int, top_p: int,
               softcap: float | None = None) -> QueryDesc:
    """query [B, Hq, Q, D] with a contiguous last dim."""
    if query.stride(-1) != 1:
        raise KIVNativeError("query head_dim must be contiguous")
    return QueryDesc(query.data_ptr(), query.stride(0), query.stride(1), query.stride(2),
                     query.shape[1], query.shape[2], float(scaling), float(softcap or 0.0),
                     int(top_pages), int(top_p))


def mask_desc(add: torch.Tensor | None = None, causal: bool = False) -> MaskDesc:
    """add: float32 [B, Hm, Q, hot_len] view (last dim contiguous); Hm == 1 broadcasts."""
    if add is None:
        return MaskDesc(None, 0, 0, 0, int(causal), 0)
    if add.dtype != torch.float32 or add.stride(-1) != 1:
        raise KIVNativeError("mask must be float32 with a contiguous last dim")
    sh = 0 if add.shape[1] == 1 else add.stride(1)
    sb = 0 if add.shape[0] == 1 else add.stride(0)
    return MaskDesc(add.data_ptr(), sb, sh, add.stride(2), int(causal), 0)
