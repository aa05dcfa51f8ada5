"""Drop-in body for the reference's decode attention entry point
(dllm_flash_attn_decode, diffulex_kernel/python/dllm_flash_attn.py:599-637).

One fused paged kernel serves both decode modes of the reference:

* ``decode_mode == "static"`` (block diffusion): the reference JIT-compiles a TileLang kernel per
  shape tuple (:608-631).  Here shapes are run-time arguments.  ``cu_seqlens_k`` cumulates the
  in-flight lengths.  ``scale`` is honoured (the reference kernel hard-codes head_dim**-0.5, :184;
  identical for every shipped model).
* ``decode_mode == "varlen"`` (D2F): the reference gathers the paged prefix into a contiguous
  tensor and calls a dense non-causal varlen attention (:632-637).  Here the same kernel reads the
  pages directly, so KV crosses HBM once instead of three times and no host sync happens.
  ``cu_seqlens_k`` cumulates ctx+new in this mode and is not needed: in-flight rows are addressed
  by ``cu_seqlens_q``.

One additive, optional metadata field: ``mask_mode`` in {"bd_full", "varlen_full",
"d2f_block_causal"}.  Absent, the reference behaviour (every in-flight key visible) is used.
"d2f_block_causal" hides in-flight diffusion blocks that come after the query's own block
(diffulex_legacy/engine/sequence.py:477-490).
"""
from __future__ import annotations

import os

import torch

from . import ops
from ._lib import DLX_MASK_BLOCK_CAUSAL, DLX_MASK_FULL

_SM_COUNT = 148  # B200

_MASKS = {None: DLX_MASK_FULL, "bd_full": DLX_MASK_FULL, "varlen_full": DLX_MASK_FULL,
          "d2f_block_causal": DLX_MASK_BLOCK_CAUSAL}


def dllm_flash_attn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor, scale: float, attn_metadata) -> torch.Tensor:
    """``q [sumQ, Hq, hd]``, ``k/v [sumQ, Hkv, hd]``, unified caches ``[NB, PAGE, Hkv, hd]`` ->
    new tensor ``o [sumQ, Hq, hd]`` in q's dtype."""
    md = attn_metadata
    mode = md.decode_mode
    if mode not in ("static", "varlen"):
        raise ValueError(f"unknown decode_mode {mode!r}")
    mask_name = getattr(md, "mask_mode", None)
    if mask_name not in _MASKS:
        raise ValueError(f"unknown mask_mode {mask_name!r}")
    dbs = int(getattr(md, "diffusion_block_size", 0) or 0)
    max_q = int(getattr(md, "max_seqlen_q", 0) or 0)
    if max_q <= 0:
        max_q = dbs if (mode == "static" and dbs > 0) else int(q.shape[0])
    max_kv = 0
    if mode == "varlen":
        max_kv = int(getattr(md, "max_seqlen_k", 0) or 0)  # cumulates ctx+new in this mode
    cu_kv = md.cu_seqlens_k if mode == "static" else None
    num_splits = int(getattr(md, "num_splits", 0) or os.environ.get("DLX_NUM_SPLITS", 0))
    return ops.decode_attn(q, k, v, k_cache, v_cache, md.block_tables, md.context_lens, md.cu_seqlens_q, cu_kv,
                           float(scale), max_q, max_kv, _MASKS[mask_name], dbs, num_splits, _longest_first(md, k))


def _longest_first(md, k) -> "torch.Tensor | None":
    """Sequence order for the kernel's grid: longest context first, so that the in-order CTA dispatch
    behaves like a longest-processing-time schedule when there are more (sequence, KV head) pairs than
    SMs.  One device-side argsort per metadata state (no host sync), memoised on the metadata object:
    all layers of a step share it.  The memo is keyed on the context_lens tensor and its version."""
    ctx = md.context_lens
    n = int(ctx.numel())
    if n * int(k.shape[1]) <= _SM_COUNT or os.environ.get("DLX_NO_SEQ_ORDER"):
        return None
    key = (ctx.data_ptr(), ctx._version, n)
    memo = getattr(md, "_dlx_seq_order", None)
    if memo is not None and memo[0] == key:
        return memo[1]
    order = torch.argsort(ctx, descending=True, stable=True).to(torch.int32)
    try:
        md._dlx_seq_order = (key, order)
    except AttributeError:
        pass
    return order


def dllm_flash_attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                            attn_metadata) -> torch.Tensor:
    """Prefill attention is the next operator on the build list; the name exists so that
    ``diffulex/attention/attn_impl.py:5-10`` imports.  It raises instead of silently computing
    on another backend."""
    raise NotImplementedError("dllm_flash_attn_prefill: the sm_100a prefill kernel is not built yet")
