"""Drop-in bodies for the reference's KV-cache entry points
(diffulex_kernel/python/kv_cache_kernels.py): same names, argument order, layouts, in-place /
return conventions and assertion behaviour; the device work is the sm_100a kernels behind the
C ABI (include/dlx_b200.h).  ``attn_metadata`` is duck-typed exactly like in the reference.
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import ops


def store_kvcache_unified_layout(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                                 v_cache: torch.Tensor, slot_mapping: torch.Tensor, attn_metadata=None) -> None:
    """Scatter ``key/value [N, Hkv, hd]`` into the unified caches ``[NB, PAGE, Hkv, hd]`` at the flat
    slots of ``slot_mapping`` (int32 or int64; negative = skip).  In place, returns None.
    Mirrors store_kvcache_unified_layout (kv_cache_kernels.py:110-124) including its asserts;
    ``attn_metadata`` is unused there and here."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert N == slot_mapping.numel(), f"`N`: {N}, `slot_mapping.numel()`: {slot_mapping.numel()}"
    assert value.shape == key.shape and k_cache.dtype == key.dtype and v_cache.dtype == value.dtype
    if torch.compiler.is_compiling():   # the registered operator carries what a tracer needs
        ops.store_kvcache_unified(key, value, k_cache, v_cache, slot_mapping)
    else:                               # eager: straight to the C ABI, the dispatcher costs more than the call
        ops._store_unified_launch(key, value, k_cache, v_cache, slot_mapping)


def store_kvcache_distinct_layout(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                                  v_cache: torch.Tensor, slot_mapping: torch.Tensor, attn_metadata=None) -> None:
    """Scatter into the split layout K ``[NB, H, hd/x, PAGE, x]``, V ``[NB, H, hd, PAGE]``
    (store_kvcache_distinct_layout, kv_cache_kernels.py:86-107)."""
    NBlks, NHeads, HDim_x, Blk_sz, x = k_cache.shape
    HDim = HDim_x * x
    N = key.shape[0]
    assert HDim == key.shape[-1] and NHeads == key.shape[1]
    assert N == slot_mapping.numel()
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == HDim and value.stride(1) == HDim
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert tuple(v_cache.shape) == (NBlks, NHeads, HDim, Blk_sz)
    ops.store_kvcache_distinct(key, value, k_cache, v_cache, slot_mapping)


def load_kvcache(k_cache: torch.Tensor, v_cache: torch.Tensor, attn_metadata, k_new: torch.Tensor,
                 v_new: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Gather each sequence's cached prefix followed by its in-flight rows into fresh
    ``[sum(ctx+new), Hkv, hd]`` tensors (load_kvcache, kv_cache_kernels.py:230-279).

    Reads ``block_tables, context_lens, seq_lens_ts, cu_seqlens_q, cu_seqlens_k`` (cumulating
    ctx+new) from ``attn_metadata``.  The output row count is taken from the optional host integer
    ``attn_metadata.total_kv_rows`` when present (no host sync, graph-capturable); otherwise from
    ``cu_seqlens_k[-1]`` (one sync; the reference syncs three times, :240,248,252).  Unlike the
    reference kernel, every row is written, including the last page of a page-aligned context
    and a ragged in-flight tail (:167, :204).
    """
    assert k_cache.shape == v_cache.shape
    assert k_new.shape == v_new.shape
    md = attn_metadata
    num_seqs, _ = md.block_tables.shape
    assert md.cu_seqlens_q.shape == md.cu_seqlens_k.shape
    assert md.cu_seqlens_q.shape[0] == num_seqs + 1
    assert k_cache.stride(-1) == 1 and k_cache.stride(2) == k_cache.shape[3]
    assert k_cache.stride(1) == k_cache.shape[2] * k_cache.shape[3]
    assert k_new.stride(-1) == 1 and k_new.stride(1) == k_new.shape[2]
    total = getattr(md, "total_kv_rows", None)
    if total is None:
        total = int(md.cu_seqlens_k[-1])
    return ops.load_kvcache(k_cache, v_cache, md.block_tables, md.context_lens, md.seq_lens_ts, md.cu_seqlens_q,
                            md.cu_seqlens_k, k_new, v_new, int(total))
