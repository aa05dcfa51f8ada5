"""Tensor-level operators over the C ABI, registered as torch custom ops (namespace ``dlx_b200``).

Each op only reads ``data_ptr()`` / strides / sizes, launches on ``torch.cuda.current_stream()`` and
never synchronises, so all of them can be captured into a CUDA graph (the reference's
block-diffusion runner captures the whole forward, diffulex/strategy/block_diffusion/engine/
model_runner.py:206-274).  Outputs and the split-K workspace come from torch's caching allocator.
CPU tensors are rejected: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import DecodeAttnParams, DlxError, check

_DTYPES = {torch.bfloat16: _lib.DLX_DTYPE_BF16}


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream() -> int:
    """The current CUDA stream of the current device as an integer handle."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("diffulex_b200 operators run on CUDA tensors only (no CPU fallback)")


# ---- store -------------------------------------------------------------------------------------
def _store_unified_launch(key, value, k_cache, v_cache, slot_mapping) -> None:
    _need_cuda(key, value, k_cache, v_cache, slot_mapping)
    n, heads, hd = key.shape
    d = heads * hd
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise ValueError("slot_mapping must be int32 or int64")
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    num_slots = k_cache.numel() // d
    check(_lib.lib().dlx_store_kvcache_unified(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
        slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64), n, d, key.element_size(), num_slots,
        _stream()))


@torch.library.custom_op("dlx_b200::store_kvcache_unified", mutates_args=("k_cache", "v_cache"))
def store_kvcache_unified(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                          slot_mapping: torch.Tensor) -> None:
    _store_unified_launch(key, value, k_cache, v_cache, slot_mapping)


@torch.library.custom_op("dlx_b200::store_kvcache_distinct", mutates_args=("k_cache", "v_cache"))
def store_kvcache_distinct(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
    _need_cuda(key, value, k_cache, v_cache, slot_mapping)
    nb, heads, hd_x, page, x = k_cache.shape
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    check(_lib.lib().dlx_store_kvcache_distinct(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
        slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64), key.shape[0], heads, hd_x * x, page, x, nb,
        key.element_size(), _stream()))


def build_slot_mapping(block_tables: torch.Tensor, context_lens: torch.Tensor, cu_seqlens_q: torch.Tensor,
                       page_size: int, total_rows: int, num_pages: int, store_flags: Optional[torch.Tensor] = None,
                       out: Optional[torch.Tensor] = None, dtype: torch.dtype = torch.int32) -> torch.Tensor:
    """The decode step's ``slot_mapping`` computed on the device from the page tables (C ABI:
    dlx_build_slot_mapping; the reference builds it in a host loop and copies it over every step,
    diffulex/strategy/block_diffusion/engine/model_runner.py:141-156).  ``store_flags[s] == 0``: sequence s stores
    nothing this step (-1 for its rows).  Writes ``out`` (a static buffer of a captured step) when given.  No host
    sync; capturable."""
    _need_cuda(block_tables, context_lens, cu_seqlens_q, store_flags, out)
    for name, t in (("block_tables", block_tables), ("context_lens", context_lens), ("cu_seqlens_q", cu_seqlens_q),
                    ("store_flags", store_flags)):
        if t is not None and (t.dtype != torch.int32 or (t.dim() == 1 and not t.is_contiguous())):
            raise ValueError(f"{name} must be contiguous int32")
    if block_tables.dim() != 2 or (block_tables.shape[1] > 0 and block_tables.stride(1) != 1):
        raise ValueError("block_tables must be [num_seqs, max_blocks] with contiguous rows")
    if out is None:
        out = torch.empty(total_rows, dtype=dtype, device=block_tables.device)
    if out.dtype not in (torch.int32, torch.int64) or out.numel() < total_rows or not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 or int64 tensor of at least total_rows entries")
    check(_lib.lib().dlx_build_slot_mapping(
        block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1], context_lens.data_ptr(),
        cu_seqlens_q.data_ptr(), store_flags.data_ptr() if store_flags is not None else None,
        cu_seqlens_q.numel() - 1, page_size, total_rows, num_pages, out.data_ptr(), int(out.dtype == torch.int64),
        _stream()))
    return out


# ---- load --------------------------------------------------------------------------------------
@torch.library.custom_op("dlx_b200::load_kvcache", mutates_args=())
def load_kvcache(k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                 context_lens: torch.Tensor, seq_lens: torch.Tensor, cu_seqlens_q: torch.Tensor,
                 cu_seqlens_k: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                 total_rows: int) -> Tuple[torch.Tensor, torch.Tensor]:
    _need_cuda(k_cache, v_cache, block_tables, context_lens, seq_lens, cu_seqlens_q, cu_seqlens_k, k_new, v_new)
    nb, page, heads, hd = k_cache.shape
    d = heads * hd
    k_out = torch.empty((total_rows, heads, hd), device=k_cache.device, dtype=k_cache.dtype)
    v_out = torch.empty_like(k_out)
    i32 = lambda t: t if (t.dtype == torch.int32 and t.is_contiguous()) else t.to(torch.int32).contiguous()
    bt, ctx, sl, cq, ck = map(i32, (block_tables, context_lens, seq_lens, cu_seqlens_q, cu_seqlens_k))
    check(_lib.lib().dlx_load_kvcache(
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1),
        k_new.data_ptr(), k_new.stride(0), v_new.data_ptr(), v_new.stride(0),
        bt.data_ptr(), bt.stride(0), bt.shape[1], ctx.data_ptr(), sl.data_ptr(), cq.data_ptr(), ck.data_ptr(),
        k_out.data_ptr(), v_out.data_ptr(), total_rows, bt.shape[0], page, nb, d, k_cache.element_size(), _stream()))
    return k_out, v_out


@load_kvcache.register_fake
def _(k_cache, v_cache, block_tables, context_lens, seq_lens, cu_seqlens_q, cu_seqlens_k, k_new, v_new, total_rows):
    shape = (total_rows, k_cache.shape[2], k_cache.shape[3])
    return k_cache.new_empty(shape), k_cache.new_empty(shape)


# ---- decode attention --------------------------------------------------------------------------
# Which decode kernel the calls ask for: 0 auto, 1 mma.sync kernel, 2 tcgen05 kernel (one CTA per item),
# 3 tcgen05 kernel (one CTA pair per item).  Read from DLX_DECODE_KERNEL once, at import; tests set the attribute.
DECODE_KERNEL = int(os.environ.get("DLX_DECODE_KERNEL", "0"))


def _decode_params(q, k, v, k_cache, v_cache, out, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv,
                   scale, max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits,
                   schedule=None, slot_mapping=None) -> DecodeAttnParams:
    if q.dtype not in _DTYPES:
        raise ValueError(f"decode attention is built for bf16, got {q.dtype}")
    total_q, hq, hd = q.shape
    hkv = k.shape[1]
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.stride(-1) != 1 or t.stride(1) != hd:
            raise ValueError(f"{name}: heads must be contiguous ([tokens, heads, head_dim] with head stride head_dim)")
    p = DecodeAttnParams()
    p.struct_bytes = ctypes.sizeof(DecodeAttnParams)
    p.dtype = _DTYPES[q.dtype]
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.q_row_stride, p.k_row_stride, p.v_row_stride, p.out_row_stride = q.stride(0), k.stride(0), v.stride(0), out.stride(0)
    if k_cache is not None and k_cache.numel() > 0:
        if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
            raise ValueError("k_cache and v_cache must share shape and strides")
        if k_cache.stride(3) != 1 or k_cache.stride(2) != hd:
            raise ValueError("cache must be [pages, page_size, Hkv, head_dim] with contiguous heads")
        p.k_cache, p.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
        p.cache_page_stride, p.cache_token_stride = k_cache.stride(0), k_cache.stride(1)
        p.num_pages, p.page_size = k_cache.shape[0], k_cache.shape[1]
        p.block_tables = block_tables.data_ptr()
        p.block_table_stride = block_tables.stride(0)
        p.max_blocks = block_tables.shape[1]
    else:
        p.num_pages, p.page_size, p.max_blocks = 0, 1, 0
    p.context_lens = context_lens.data_ptr()
    p.cu_seqlens_q = cu_seqlens_q.data_ptr()
    p.cu_seqlens_kv = cu_seqlens_kv.data_ptr() if cu_seqlens_kv is not None else None
    if schedule is not None:
        p.schedule, p.schedule_bytes = schedule.data_ptr(), schedule.numel() * schedule.element_size()
    p.total_q, p.num_seqs = total_q, cu_seqlens_q.numel() - 1
    p.total_kv = k.shape[0]
    if slot_mapping is not None:   # the call also stores the in-flight rows
        if slot_mapping.dtype not in (torch.int32, torch.int64) or not slot_mapping.is_contiguous() \
                or slot_mapping.numel() != k.shape[0]:
            raise ValueError("slot_mapping must be a contiguous int32 or int64 tensor with one entry per row of k")
        p.slot_mapping, p.slots_are_int64 = slot_mapping.data_ptr(), int(slot_mapping.dtype == torch.int64)
    p.num_q_heads, p.num_kv_heads, p.head_dim = hq, hkv, hd
    p.max_q_len, p.max_kv_len = max_q_len, max_kv_len
    p.mask_mode, p.diffusion_block_size = mask_mode, diffusion_block_size
    p.num_splits, p.kernel = num_splits, DECODE_KERNEL
    p.scale = scale
    return p


def _check_decode_metadata(q, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, schedule=None):
    for name, t in (("block_tables", block_tables), ("context_lens", context_lens), ("cu_seqlens_q", cu_seqlens_q),
                    ("cu_seqlens_kv", cu_seqlens_kv)):
        if t is not None and t.dtype != torch.int32:
            raise ValueError(f"{name} must be int32")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise ValueError("block_tables must be [num_seqs, max_blocks] with contiguous rows")
    if schedule is not None and (schedule.dtype != torch.uint8 or not schedule.is_contiguous()):
        raise ValueError("schedule must be the uint8 buffer returned by decode_schedule")


def _decode_launch(q, k, v, k_cache, v_cache, out, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                   max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits, schedule) -> None:
    _need_cuda(q, k, v, k_cache, v_cache, out, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, schedule)
    _check_decode_metadata(q, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, schedule)
    p = _decode_params(q, k, v, k_cache, v_cache, out, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv,
                       scale, max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits, schedule)
    handle = _lib.lib()
    ws_bytes = handle.dlx_decode_attn_workspace_bytes(ctypes.byref(p))
    if ws_bytes < 0:
        check(int(-ws_bytes))
    if schedule is not None:  # the prepared schedule replaces the one the call would plan into its workspace
        ws_bytes -= handle.dlx_decode_attn_schedule_bytes(ctypes.byref(p))
    ws = None
    if ws_bytes > 0:
        ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws_bytes
    check(handle.dlx_decode_attn(ctypes.byref(p), _stream()))


class DecodePlan:
    """What every layer call of one step shares: the schedule buffer, the parameter block with everything but the
    per-layer tensors filled in, and the scratch the call needs besides the schedule."""
    __slots__ = ("schedule", "template", "workspace_bytes", "q_shape", "kv_shape", "cache_shape", "slot_mapping")


def decode_plan(q, k, v, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits, slot_mapping=None) -> DecodePlan:
    """Validates once, launches the planning kernel (``decode_schedule``) and keeps the filled parameter block, so
    that the layer calls of the step (``decode_launch_planned``) only patch their own tensors in.  With
    ``slot_mapping`` every layer call of the step also stores its in-flight K / V rows (C ABI: the ``slot_mapping``
    field of the parameter block)."""
    _need_cuda(slot_mapping)
    sched = decode_schedule(q, k, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                            max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits)
    p = _decode_params(q, k, v, k_cache, v_cache, q, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                       max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits, sched, slot_mapping)
    handle = _lib.lib()
    ws_bytes = handle.dlx_decode_attn_workspace_bytes(ctypes.byref(p))
    if ws_bytes < 0:
        check(int(-ws_bytes))
    if sched is not None:
        ws_bytes -= handle.dlx_decode_attn_schedule_bytes(ctypes.byref(p))
    plan = DecodePlan()
    plan.schedule, plan.template, plan.workspace_bytes = sched, bytes(p), int(ws_bytes)
    plan.q_shape, plan.kv_shape, plan.cache_shape = q.shape, k.shape, k_cache.shape
    plan.slot_mapping = slot_mapping   # kept alive: the parameter block points at it
    return plan


def decode_launch_planned(plan: DecodePlan, q, k, v, k_cache, v_cache, out) -> None:
    """One layer's launch over a step's plan: same shapes as the tensors the plan was made with, any pointers and
    row / page strides."""
    hd = q.shape[2]
    if q.shape != plan.q_shape or k.shape != plan.kv_shape or v.shape != plan.kv_shape or out.shape != plan.q_shape \
            or k_cache.shape != plan.cache_shape or v_cache.shape != plan.cache_shape:
        raise ValueError("tensor shapes differ from the ones this step was planned for")
    for t in (q, k, v, out):
        if not t.is_cuda or t.dtype != torch.bfloat16 or t.stride(2) != 1 or t.stride(1) != hd:
            raise ValueError("q / k / v / out: CUDA bf16 [tokens, heads, head_dim] with contiguous heads")
    p = DecodeAttnParams.from_buffer_copy(plan.template)
    p.q, p.k, p.v, p.out = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    p.q_row_stride, p.k_row_stride, p.v_row_stride, p.out_row_stride = q.stride(0), k.stride(0), v.stride(0), out.stride(0)
    if k_cache.numel() > 0:
        if not k_cache.is_cuda or k_cache.stride() != v_cache.stride() or k_cache.stride(3) != 1 or k_cache.stride(2) != hd:
            raise ValueError("cache must be CUDA [pages, page_size, Hkv, head_dim] with contiguous heads, K and V alike")
        p.k_cache, p.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
        p.cache_page_stride, p.cache_token_stride = k_cache.stride(0), k_cache.stride(1)
    if plan.workspace_bytes > 0:
        ws = torch.empty(plan.workspace_bytes, device=q.device, dtype=torch.uint8)
        p.workspace, p.workspace_bytes = ws.data_ptr(), plan.workspace_bytes
    check(_lib.lib().dlx_decode_attn(ctypes.byref(p), _stream()))


@torch.library.custom_op("dlx_b200::decode_attn", mutates_args=())
def decode_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                block_tables: torch.Tensor, context_lens: torch.Tensor, cu_seqlens_q: torch.Tensor,
                cu_seqlens_kv: Optional[torch.Tensor], scale: float, max_q_len: int, max_kv_len: int,
                mask_mode: int, diffusion_block_size: int, num_splits: int,
                schedule: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty((q.shape[0], q.shape[1], q.shape[2]), device=q.device, dtype=q.dtype)
    _decode_launch(q, k, v, k_cache, v_cache, out, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                   max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits, schedule)
    return out


@decode_attn.register_fake
def _(q, k, v, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale, max_q_len,
      max_kv_len, mask_mode, diffusion_block_size, num_splits, schedule=None):
    return q.new_empty(q.shape)


@torch.library.custom_op("dlx_b200::decode_attn_out", mutates_args=("out",))
def decode_attn_out(out: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, block_tables: torch.Tensor, context_lens: torch.Tensor,
                    cu_seqlens_q: torch.Tensor, cu_seqlens_kv: Optional[torch.Tensor], scale: float, max_q_len: int,
                    max_kv_len: int, mask_mode: int, diffusion_block_size: int, num_splits: int,
                    schedule: Optional[torch.Tensor] = None) -> None:
    """``decode_attn`` into a caller-owned ``out`` ([total_q, Hq, hd], contiguous heads, any row stride)."""
    if out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("out must have q's shape and dtype")
    _decode_launch(q, k, v, k_cache, v_cache, out, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                   max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits, schedule)


def decode_schedule(q: torch.Tensor, k: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_tables: torch.Tensor, context_lens: torch.Tensor, cu_seqlens_q: torch.Tensor,
                    cu_seqlens_kv: Optional[torch.Tensor], scale: float, max_q_len: int, max_kv_len: int,
                    mask_mode: int, diffusion_block_size: int, num_splits: int) -> Optional[torch.Tensor]:
    """The per-step half of decode attention (C ABI: dlx_decode_attn_prepare): one small launch that turns
    the step's metadata into the packed, placed work-item records every layer call of the step then reads.
    Returns the schedule buffer to pass as ``schedule``, or None when the kernel that serves these shapes
    takes none.  No host sync; capturable."""
    _need_cuda(q, k, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv)
    _check_decode_metadata(q, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv)
    p = _decode_params(q, k, k, k_cache, v_cache, q, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv,
                       scale, max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits)
    handle = _lib.lib()
    n = handle.dlx_decode_attn_schedule_bytes(ctypes.byref(p))
    if n < 0:
        check(int(-n))
    if n == 0 or p.num_seqs == 0 or p.total_q == 0:
        return None
    sched = torch.empty(n, device=q.device, dtype=torch.uint8)
    check(handle.dlx_decode_attn_prepare(ctypes.byref(p), sched.data_ptr(), n, _stream()))
    return sched


def stream_capture_id() -> int:
    """Capture sequence id of the current stream (0 when it is not being captured)."""
    if not torch.cuda.is_current_stream_capturing():
        return 0
    cid = ctypes.c_uint64(0)
    check(_lib.lib().dlx_stream_capture_id(_stream(), ctypes.byref(cid)))
    return int(cid.value)


def device_status() -> tuple:
    """(bits, site, tile, cta) of the tcgen05 kernels' status word; synchronises and clears it."""
    out = (ctypes.c_int32 * 4)()
    check(_lib.lib().dlx_debug_device_status(out))
    return tuple(int(x) for x in out)


def planned_num_splits(q, k, v, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                       max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits) -> int:
    """How many key-range splits a decode call with these arguments uses (host-side planning only)."""
    p = _decode_params(q, k, v, k_cache, v_cache, q, block_tables, context_lens, cu_seqlens_q, cu_seqlens_kv, scale,
                       max_q_len, max_kv_len, mask_mode, diffusion_block_size, num_splits)
    n = _lib.lib().dlx_decode_attn_num_splits(ctypes.byref(p))
    if n < 0:
        check(-n)
    return n


__all__ = ["store_kvcache_unified", "store_kvcache_distinct", "build_slot_mapping", "load_kvcache", "decode_attn", "decode_attn_out",
           "decode_schedule", "decode_plan", "decode_launch_planned", "DecodePlan", "stream_capture_id", "device_status", "planned_num_splits", "DlxError"]
