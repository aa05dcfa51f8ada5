"""Host-side mirror of the reference's attention layer (``Attention``, diffulex/attention/attn_impl.py:14-72):
the one caller of the three operators on the decode hot path.  Per layer call it

1. views the projections ``[s, heads * hd]`` as ``[s, heads, hd]`` (:45-47),
2. writes the step's K / V rows into the paged cache when the metadata asks for it and a cache is attached
   (:53-57; unified or split layout by ``kv_cache_layout``); in decode this is part of the attention call,
3. runs prefill or decode attention (:60-69) and
4. returns ``[s, heads * hd]`` contiguous (:72).

The reference layer takes its metadata from a module-level fetch function installed by the model runner
(diffulex/attention/__init__.py:4-15); here the fetch function is a constructor argument, so two engines in one
process do not share state.  Everything runs on the current CUDA stream without a host synchronisation, so a
whole decode step can be captured into a CUDA graph as the reference's runner does
(diffulex/strategy/block_diffusion/engine/model_runner.py:197-251).
"""
from __future__ import annotations

from typing import Callable

import torch

from .dllm_flash_attn import dllm_flash_attn_decode, dllm_flash_attn_prefill
from .kv_cache_kernels import store_kvcache_distinct_layout, store_kvcache_unified_layout


class Attention(torch.nn.Module):
    def __init__(self, num_heads: int, head_dim: int, scale: float, num_kv_heads: int,
                 fetch_attn_metadata: Callable[[], object]):
        super().__init__()
        self.num_heads, self.head_dim, self.scale, self.num_kv_heads = num_heads, head_dim, scale, num_kv_heads
        self.fetch_attn_metadata = fetch_attn_metadata
        # the runner attaches slices of its cache pool here (model_runner_base.py allocate_kv_cache)
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask=None) -> torch.Tensor:
        s = q.shape[0]
        q = q.view(s, self.num_heads, self.head_dim)
        k = k.view(k.shape[0], self.num_kv_heads, self.head_dim)
        v = v.view(v.shape[0], self.num_kv_heads, self.head_dim)
        md = self.fetch_attn_metadata()
        unified = getattr(md, "kv_cache_layout", "unified") == "unified"
        have_cache = self.k_cache.numel() > 0 and self.v_cache.numel() > 0
        store_now = have_cache and getattr(md, "need_kv_cache_store", True)
        fused = store_now and unified and not md.is_prefill   # decode: the attention call stores as well
        if store_now and not fused:
            store = store_kvcache_unified_layout if unified else store_kvcache_distinct_layout
            store(k, v, self.k_cache, self.v_cache, md.slot_mapping, md)
        if md.is_prefill:
            o = dllm_flash_attn_prefill(q, k, v, self.scale, md)
        elif unified:
            o = dllm_flash_attn_decode(q, k, v, self.k_cache, self.v_cache, self.scale, md,
                                       store_slot_mapping=md.slot_mapping if fused else None)
        else:
            # as in the reference (attn_impl.py:68-69): decode reads the unified layout only
            raise NotImplementedError("decode attention reads the unified cache layout only")
        return o.view(s, self.num_heads * self.head_dim)
