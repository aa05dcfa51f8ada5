"""ctypes binding of ``libdlx_b200.so`` (C ABI: include/dlx_b200.h).

There is no fallback: if the library is missing or fails to load, importing the operators raises.
Build it with ``python -m diffulex_b200.build``.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_int32, c_int64, c_uint32, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "csrc" / "libdlx_b200.so"

DLX_OK = 0
DLX_DTYPE_BF16 = 0
DLX_MASK_FULL = 0
DLX_MASK_BLOCK_CAUSAL = 1


class DlxError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(f"dlx status {status}: {message}")
        self.status = status


class DecodeAttnParams(ctypes.Structure):
    """Mirror of ``dlx_decode_attn_params`` (include/dlx_b200.h); field order and types must match."""
    _fields_ = [
        ("struct_bytes", c_uint32), ("dtype", c_int32),
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("out", c_void_p), ("block_tables", c_void_p), ("context_lens", c_void_p), ("cu_seqlens_q", c_void_p),
        ("cu_seqlens_kv", c_void_p), ("schedule", c_void_p), ("schedule_bytes", c_int64),
        ("workspace", c_void_p), ("workspace_bytes", c_int64),
        ("q_row_stride", c_int64), ("k_row_stride", c_int64), ("v_row_stride", c_int64), ("out_row_stride", c_int64),
        ("cache_page_stride", c_int64), ("cache_token_stride", c_int64), ("block_table_stride", c_int64),
        ("num_pages", c_int64),
        ("total_q", c_int32), ("num_seqs", c_int32), ("max_blocks", c_int32),
        ("num_q_heads", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32), ("page_size", c_int32),
        ("max_q_len", c_int32), ("max_kv_len", c_int32), ("mask_mode", c_int32), ("diffusion_block_size", c_int32),
        ("num_splits", c_int32), ("kernel", c_int32), ("scale", c_float), ("total_kv", c_int32),
        ("slot_mapping", c_void_p), ("slots_are_int64", c_int32), ("reserved0", c_int32),
    ]


_SIGNATURES = {
    "dlx_version": (c_int, []),
    "dlx_status_string": (c_char_p, [c_int]),
    "dlx_last_error": (c_char_p, []),
    "dlx_store_kvcache_unified": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                                          c_int64, c_int64, c_int, c_int64, c_void_p]),
    "dlx_store_kvcache_distinct": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_int,
                                           c_int64, c_int32, c_int32, c_int32, c_int32, c_int64, c_int, c_void_p]),
    "dlx_build_slot_mapping": (c_int, [c_void_p, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                       c_int64, c_int64, c_void_p, c_int, c_void_p]),
    "dlx_load_kvcache": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                 c_void_p, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_void_p, c_int64, c_int32, c_int32, c_int64, c_int64, c_int, c_void_p]),
    "dlx_decode_attn_workspace_bytes": (c_int64, [ctypes.POINTER(DecodeAttnParams)]),
    "dlx_decode_attn_num_splits": (c_int32, [ctypes.POINTER(DecodeAttnParams)]),
    "dlx_decode_attn": (c_int, [ctypes.POINTER(DecodeAttnParams), c_void_p]),
    "dlx_decode_attn_schedule_bytes": (c_int64, [ctypes.POINTER(DecodeAttnParams)]),
    "dlx_decode_attn_prepare": (c_int, [ctypes.POINTER(DecodeAttnParams), c_void_p, c_int64, c_void_p]),
    "dlx_stream_capture_id": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "dlx_static_scratch_bytes": (c_int64, []),
    "dlx_decode_attn_static_scratch": (c_int, [ctypes.POINTER(DecodeAttnParams), c_void_p]),
    "dlx_debug_device_status": (c_int, [ctypes.POINTER(c_int32)]),
}

EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises (never falls back) when it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: the CUDA extension has not been built "
                f"(run `python -m diffulex_b200.build`). There is no CPU or PyTorch fallback.")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError if the symbol is not exported
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != DLX_OK:
        handle = lib()
        msg = handle.dlx_last_error().decode() or handle.dlx_status_string(status).decode()
        raise DlxError(status, msg)
