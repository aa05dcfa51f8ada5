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

_MASKS = {None: DLX_MASK_FULL, "bd_full": DLX_MASK_FULL, "varlen_full": DLX_MASK_FULL,
          "d2f_block_causal": DLX_MASK_BLOCK_CAUSAL}


def dllm_flash_attn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                           v_cache: torch.Tensor, scale: float, attn_metadata, out: "torch.Tensor | None" = None,
                           store_slot_mapping: "torch.Tensor | None" = None) -> torch.Tensor:
    """``q [sumQ, Hq, hd]``, ``k/v [sumQ, Hkv, hd]``, unified caches ``[NB, PAGE, Hkv, hd]`` ->
    new tensor ``o [sumQ, Hq, hd]`` in q's dtype (or ``out``, additive keyword, when given).

    ``store_slot_mapping`` (additive keyword): when given, the call also stores the in-flight ``k`` / ``v`` rows
    into the caches at these flat slots, i.e. it does ``store_kvcache_unified_layout`` and the attention of
    ``Attention.forward`` (diffulex/attention/attn_impl.py:54-57, :66-67) in one call (the store kernel is launched
    first, on the same stream; one trip through Python and the C ABI instead of two); the caller then skips its own
    store.

    Optional metadata attributes (all additive): ``mask_mode``, ``num_splits``, and ``check_status``:
    when true the call synchronises afterwards, reads the kernels' status word and raises if a bounded
    wait inside a kernel gave up (debugging aid; off by default)."""
    md = attn_metadata
    mode = md.decode_mode
    if mode not in ("static", "varlen"):
        raise ValueError(f"unknown decode_mode {mode!r}")
    ops._need_cuda(q, k, v, k_cache, v_cache)
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
    num_splits = int(getattr(md, "num_splits", 0) or _ENV_NUM_SPLITS)
    args = (md.block_tables, md.context_lens, md.cu_seqlens_q, cu_kv, float(scale), max_q, max_kv, _MASKS[mask_name],
            dbs, num_splits)
    o = _run(out, q, k, v, k_cache, v_cache, args, _plan(md, q, k, v, k_cache, v_cache, args, store_slot_mapping),
             store_slot_mapping)
    if getattr(md, "check_status", False):
        bits, site, tile, cta = ops.device_status()
        if bits & 1:
            raise RuntimeError(f"decode attention: a bounded wait gave up (site {site}, tile {tile}, CTA {cta}); "
                               "the output of this call is incomplete")
    return o


def _run(out, q, k, v, k_cache, v_cache, args, plan, slots=None):
    """One launch.  Under torch.compile the registered custom operators are used (they carry the fake
    implementations a tracer needs); eager calls go straight to the C ABI with the step's prepared parameter block:
    the dispatcher and the parameter marshalling cost more host time than the rest of the call."""
    if torch.compiler.is_compiling():
        if slots is not None:   # the traced operators do not store: a separate store operator first
            ops.store_kvcache_unified(k, v, k_cache, v_cache, slots)
        if out is None:
            return ops.decode_attn(q, k, v, k_cache, v_cache, *args, plan.schedule)
        ops.decode_attn_out(out, q, k, v, k_cache, v_cache, *args, plan.schedule)
        return out
    if out is None:
        out = torch.empty((q.shape[0], q.shape[1], q.shape[2]), device=q.device, dtype=q.dtype)
    ops.decode_launch_planned(plan, q, k, v, k_cache, v_cache, out)
    return out


_ENV_NUM_SPLITS = int(os.environ.get("DLX_NUM_SPLITS", "0"))
_captured_plans = []   # plans made inside a stream capture: the graph reads their schedules on every replay


def _plan(md, q, k, v, k_cache, v_cache, args, slots=None) -> "ops.DecodePlan":
    """The step's plan (``ops.decode_plan``: schedule + prepared parameter block): built by the first layer call that
    sees a metadata state and shared by the others through a memo on the metadata object.  The memo is keyed on the
    metadata tensors (storage and in-place version), the shapes that shape the plan, and the capture id of
    the current stream: inside a CUDA-graph capture the first layer call always records a planning launch,
    so a replay after the runner refilled its static buffers (diffulex/strategy/block_diffusion/engine/
    model_runner.py:183-195) plans from the new lengths."""
    block_tables, context_lens, cu_q, cu_kv = args[0], args[1], args[2], args[3]
    cap = ops.stream_capture_id()
    key = (cap, ops.DECODE_KERNEL, q.shape, k.shape, k_cache.shape, args[4:],
           block_tables.data_ptr(), block_tables._version, block_tables.shape, block_tables.stride(0),
           context_lens.data_ptr(), context_lens._version, cu_q.data_ptr(), cu_q._version, cu_q.shape,
           None if cu_kv is None else (cu_kv.data_ptr(), cu_kv._version),
           None if slots is None else (slots.data_ptr(), slots.dtype))
    memo = getattr(md, "_dlx_plan", None)
    if memo is not None and memo[0] == key:
        return memo[1]
    plan = ops.decode_plan(q, k, v, k_cache, v_cache, *args, slots)
    try:
        md._dlx_plan = (key, plan)
    except AttributeError:
        pass
    if cap and plan.schedule is not None:
        _captured_plans.append(plan)
        del _captured_plans[:-64]
    return plan


def dllm_flash_attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                            attn_metadata, out: "torch.Tensor | None" = None) -> torch.Tensor:
    """Drop-in body for the reference's prefill attention (dllm_flash_attn_prefill,
    diffulex_kernel/python/dllm_flash_attn.py:539-596): ``q [sumQ, Hq, hd]``, ``k/v [sumK, Hkv, hd]`` of the
    prompts themselves, no cache -> ``o [sumQ, Hq, hd]``.

    ``attn_type == "full_attention"``: every key of the sequence is visible (the reference calls a dense
    non-causal varlen attention, :546-552).  ``"block_attention"``: key j is visible to query i when
    ``j < (i // diffusion_block_size + 1) * diffusion_block_size`` (the reference's TileLang kernel, :109-116,
    compiled per shape tuple and autotuned during warm-up, :554-595; here shapes are run-time arguments and
    there is no hidden ``kernel_config`` state).  ``scale`` is honoured in both modes (the reference kernel
    hard-codes head_dim**-0.5, :42).  Runs the decode kernels with an empty context: same tiles, same masks."""
    md = attn_metadata
    kind = md.attn_type
    if kind not in ("full_attention", "block_attention"):
        raise ValueError(f"unknown attn_type {kind!r}")
    ops._need_cuda(q, k, v)
    dbs = int(getattr(md, "diffusion_block_size", 0) or 0)
    if kind == "block_attention" and dbs <= 0:
        raise ValueError("block_attention needs diffusion_block_size > 0")
    num_seqs = md.cu_seqlens_q.numel() - 1
    max_q = int(getattr(md, "max_seqlen_q", 0) or 0) or int(q.shape[0])
    max_kv = int(getattr(md, "max_seqlen_k", 0) or 0)
    no_cache = q.new_empty((0, 1, k.shape[1], q.shape[2]))
    no_tables = md.cu_seqlens_q.new_empty((num_seqs, 0))
    no_context = md.cu_seqlens_q.new_empty(0)   # ignored without a cache
    mask = DLX_MASK_BLOCK_CAUSAL if kind == "block_attention" else DLX_MASK_FULL
    args = (no_tables, no_context, md.cu_seqlens_q, md.cu_seqlens_k, float(scale), max_q, max_kv, mask, dbs,
            int(getattr(md, "num_splits", 0) or 1))
    return _run(out, q, k, v, no_cache, no_cache, args, _plan(md, q, k, v, no_cache, no_cache, args))
