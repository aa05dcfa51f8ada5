"""CPU fp32 oracle for the dLLM paged decode attention.

TEST INFRASTRUCTURE ONLY.  This module is the checker (and the timed CPU baseline of the bench);
nothing in the product package imports it.  It restates the reference's own PyTorch check,
``naive_sdpa_with_kvcache`` (tests/python/kernel/test_dllm_flash_attn_decode_kernel.py:14-105):
per sequence, gather the cached prefix through the block table, append the in-flight K/V rows,
and run plain softmax attention with grouped query heads.  Parity is pinned: tests/golden holds
outputs of that reference function on seeded inputs (tests/golden/make_golden.py) and
tests/test_oracle_golden.py checks this oracle against them.

The block-causal mask for several in-flight diffusion blocks follows the reference's mask
builders (diffulex_legacy/engine/sequence.py:477-490; tests/python/kernel/
test_dllm_flash_attn_prefill_kernel.py:57-62): a query in diffusion block b sees the whole cached
prefix and the in-flight blocks 0..b.
"""
from __future__ import annotations

import torch

MASK_BD_FULL = 0
MASK_D2F_BLOCK_CAUSAL = 1


def gather_prefix(cache: torch.Tensor, table_row: torch.Tensor, ctx: int) -> torch.Tensor:
    """Rows 0..ctx-1 of one sequence: page j of the table holds positions j*PAGE..(j+1)*PAGE-1.
    Entries that are negative are skipped (test_dllm_flash_attn_decode_kernel.py:66-76)."""
    page = cache.shape[1]
    parts = []
    for j in range(table_row.numel()):
        pid = int(table_row[j])
        start = j * page
        if pid < 0 or start >= ctx:
            continue
        parts.append(cache[pid, : min(page, ctx - start)])
    if not parts:
        return cache.new_zeros((0,) + tuple(cache.shape[2:]))
    return torch.cat(parts, dim=0)


def decode_attention(q, k, v, k_cache, v_cache, block_tables, context_lens, cu_seqlens_q, cu_seqlens_k,
                     scale: float, mask_mode: int = MASK_BD_FULL, diffusion_block_size: int = 32,
                     kv_offsets_from_q: bool = False) -> torch.Tensor:
    """fp32 attention of every sequence's query block over [cached prefix ; in-flight rows].

    q [sumQ, Hq, hd]; k, v [sumQ, Hkv, hd]; caches [NB, PAGE, Hkv, hd]; returns fp32 [sumQ, Hq, hd].
    ``cu_seqlens_k`` addresses the in-flight rows of k/v (static decode convention,
    diffulex/strategy/block_diffusion/engine/model_runner.py:135-139); with ``kv_offsets_from_q``
    the in-flight rows are addressed by ``cu_seqlens_q`` instead (varlen convention, where
    cu_seqlens_k cumulates ctx+new).
    """
    hq, hd = q.shape[1], q.shape[2]
    hkv = k.shape[1]
    group = hq // hkv
    out = torch.zeros(q.shape, dtype=torch.float32)
    cu_kv = cu_seqlens_q if kv_offsets_from_q else cu_seqlens_k
    for s in range(context_lens.numel()):
        q0, q1 = int(cu_seqlens_q[s]), int(cu_seqlens_q[s + 1])
        k0 = int(cu_kv[s])
        n_q = q1 - q0
        if n_q <= 0:
            continue
        n_new = n_q if kv_offsets_from_q else int(cu_kv[s + 1]) - k0
        ctx = int(context_lens[s])
        keys = torch.cat([gather_prefix(k_cache, block_tables[s], ctx).float(), k[k0:k0 + n_new].float()], 0)
        vals = torch.cat([gather_prefix(v_cache, block_tables[s], ctx).float(), v[k0:k0 + n_new].float()], 0)
        ctx = keys.shape[0] - n_new  # pages listed as -1 shorten the prefix, as in the reference check
        qs = q[q0:q1].float().permute(1, 0, 2)                              # [Hq, n_q, hd]
        ks = keys.permute(1, 0, 2).repeat_interleave(group, dim=0)          # [Hq, L, hd]
        vs = vals.permute(1, 0, 2).repeat_interleave(group, dim=0)
        logits = torch.matmul(qs, ks.transpose(1, 2)) * scale              # [Hq, n_q, L]
        if mask_mode == MASK_D2F_BLOCK_CAUSAL:
            rows = torch.arange(n_q).unsqueeze(1)
            cols = torch.arange(keys.shape[0]).unsqueeze(0)
            limit = ctx + (rows // diffusion_block_size + 1) * diffusion_block_size
            logits = logits.masked_fill(~(cols < limit).unsqueeze(0), float("-inf"))
        probs = torch.softmax(logits, dim=-1)
        out[q0:q1] = torch.matmul(probs, vs).permute(1, 0, 2)
    return out


def prefill_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, scale: float, is_block_attn: bool,
                      diffusion_block_size: int = 32) -> torch.Tensor:
    """fp32 attention of every prompt over its own keys, no cache: the reference's check of its prefill
    kernel (``naive_sdpa_prefill``, tests/python/kernel/test_dllm_flash_attn_prefill_kernel.py:13-77).
    ``is_block_attn``: query i sees keys j < (i // dbs + 1) * dbs (:57-62); else every key (:46-55).
    q [sumQ, Hq, hd]; k, v [sumK, Hkv, hd]; returns fp32 [sumQ, Hq, hd]."""
    n = cu_seqlens_q.numel() - 1
    none = k.new_zeros((0, 1, k.shape[1], k.shape[2]))
    return decode_attention(q, k, v, none, none, torch.zeros((n, 0), dtype=torch.int32),
                            torch.zeros(n, dtype=torch.int32), cu_seqlens_q, cu_seqlens_k, scale,
                            MASK_D2F_BLOCK_CAUSAL if is_block_attn else MASK_BD_FULL, diffusion_block_size)
