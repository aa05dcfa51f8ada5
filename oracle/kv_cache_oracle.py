"""CPU oracle for the slot-mapped KV-cache store and the paged KV-cache load.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA kernels; nothing in the
product package imports it.  It restates, in numpy, the copy semantics of the reference's Triton
kernels in diffulex_kernel/python/kv_cache_kernels.py.  Parity is pinned: tests/golden holds
outputs of the reference's own kernels (run under the Triton interpreter by
tests/golden/make_golden.py) and tests/test_oracle_golden.py checks this oracle against them.

All functions are dtype-agnostic byte copies: pass arrays of any fixed-size dtype (bf16 tensors
are passed as their uint16 bit patterns).
"""
from __future__ import annotations

import numpy as np


def store_kvcache_unified(key, value, k_cache, v_cache, slot_mapping) -> None:
    """In place: for every token t with slot[t] >= 0, row slot[t] of the flattened cache gets
    key[t] / value[t]; tokens with a negative slot are skipped.

    Follows dllm_store_kvcache_kernel_unified (diffulex_kernel/python/kv_cache_kernels.py:22-32)
    and its launcher (:110-124): key/value are [N, Hkv, hd], caches are [NB, PAGE, Hkv, hd] seen as
    [NB*PAGE, Hkv*hd].  Later tokens win when two tokens name the same slot (sequential order; the
    reference leaves that case to a race, real slot maps never repeat a slot).
    """
    n = key.shape[0]
    d = int(np.prod(key.shape[1:]))
    assert slot_mapping.size == n
    kc = k_cache.reshape(-1, d)
    vc = v_cache.reshape(-1, d)
    kf = key.reshape(n, d)
    vf = value.reshape(n, d)
    for t in range(n):
        s = int(slot_mapping[t])
        if s < 0:
            continue
        kc[s] = kf[t]
        vc[s] = vf[t]


def store_kvcache_distinct(key, value, k_cache, v_cache, slot_mapping) -> None:
    """In place scatter into the split layout K [NB, H, hd/x, PAGE, x], V [NB, H, hd, PAGE].

    Follows dllm_store_kvcache_kernel_distinct (diffulex_kernel/python/kv_cache_kernels.py:59-83).
    """
    nb, h, hd_x, page, x = k_cache.shape
    n = key.shape[0]
    for t in range(n):
        s = int(slot_mapping[t])
        if s < 0:
            continue
        b, off = divmod(s, page)
        k_cache[b, :, :, off, :] = key[t].reshape(h, hd_x, x)
        v_cache[b, :, :, off] = value[t]


def load_kvcache(k_cache, v_cache, block_tables, context_lens, seq_lens, cu_seqlens_q, cu_seqlens_k,
                 k_new, v_new):
    """Gather every sequence's cached prefix followed by its in-flight rows.

    For sequence s: out[cu_k[s] : cu_k[s]+ctx_s] = rows 0..ctx_s-1 of the pages block_tables[s] lists
    (page j holds positions j*PAGE .. j*PAGE+PAGE-1), then out[cu_k[s]+ctx_s : +new_s] =
    k_new[cu_q[s] : cu_q[s]+new_s].  ``cu_seqlens_k`` cumulates ctx+new here
    (diffulex_kernel/python/kv_cache_kernels.py:245-248).

    This is the intended behaviour of load_kvcache_kernel (kv_cache_kernels.py:155-227) as its
    own checker states it (diffulex_legacy/layers/attention/ops/kv_cache_kernels.py:365-392).
    The reference kernel itself leaves some of these rows unwritten; see
    ``reference_written_rows``.
    """
    page = k_cache.shape[1]
    total = int(cu_seqlens_k[-1])
    k_out = np.zeros((total,) + k_cache.shape[2:], dtype=k_cache.dtype)
    v_out = np.zeros_like(k_out)
    for s in range(len(context_lens)):
        ctx, new = int(context_lens[s]), int(seq_lens[s])
        o = int(cu_seqlens_k[s])
        pos = 0
        while pos < ctx:
            j, n = pos // page, min(page, ctx - pos)
            pid = int(block_tables[s, j])
            k_out[o + pos:o + pos + n] = k_cache[pid, :n]
            v_out[o + pos:o + pos + n] = v_cache[pid, :n]
            pos += n
        qs = int(cu_seqlens_q[s])
        k_out[o + ctx:o + ctx + new] = k_new[qs:qs + new]
        v_out[o + ctx:o + ctx + new] = v_new[qs:qs + new]
    return k_out, v_out


def reference_written_rows(page, block_tables, context_lens, seq_lens, cu_seqlens_k, dbs) -> np.ndarray:
    """Boolean mask over output rows: which rows the REFERENCE kernel actually writes.

    Two documented gaps of load_kvcache_kernel: (1) a page whose window ends exactly at ctx gets
    local_ctxlen = ctx % PAGE = 0 and copies nothing (kv_cache_kernels.py:167,178-192), so the last
    full page of a page-aligned context is dropped; (2) fresh rows are copied in whole
    DIFFUSION_BLOCK_SIZE blocks, new // dbs of them (:204), so a ragged tail is dropped.  Pages
    whose block-table entry is -1 are skipped (:152).  Those rows stay uninitialised in the
    reference; parity with the reference is asserted on the rows of this mask only.
    """
    total = int(cu_seqlens_k[-1])
    m = np.zeros(total, dtype=bool)
    maxb = block_tables.shape[1]
    for s in range(len(context_lens)):
        ctx, new = int(context_lens[s]), int(seq_lens[s])
        o = int(cu_seqlens_k[s])
        for j in range(maxb):
            if int(block_tables[s, j]) == -1:
                continue
            if ctx > j * page:
                local = page if ctx > (j + 1) * page else ctx % page
                m[o + j * page:o + j * page + local] = True
        nfull = (new // dbs) * dbs
        m[o + ctx:o + ctx + nfull] = True
    return m


def build_slot_mapping(block_tables, context_lens, cu_seqlens_q, page_size, total_rows, store_flags=None) -> np.ndarray:
    """Slot of every in-flight row of a decode step: position ``ctx + i`` of its sequence through the page table,
    -1 for sequences that store nothing this step, for positions without a page and for rows of no sequence.
    The reference's runner writes ``[-1] * block`` for a sequence whose block is still active and otherwise the
    whole slot ranges of the block's pages (diffulex/strategy/block_diffusion/engine/model_runner.py:141-151);
    ``reference_bd_slot_mapping`` below restates that loop, and for page sizes that divide the diffusion block the
    two agree (tests/test_oracle_golden.py)."""
    out = np.full(total_rows, -1, dtype=np.int64)
    maxb = block_tables.shape[1]
    for s in range(len(context_lens)):
        q0, q1 = int(cu_seqlens_q[s]), int(cu_seqlens_q[s + 1])
        if q1 <= q0 or (store_flags is not None and not store_flags[s]):
            continue
        for t in range(max(q0, 0), min(q1, total_rows)):
            pos = max(int(context_lens[s]), 0) + (t - q0)
            j = pos // page_size
            if j < maxb and block_tables[s, j] >= 0:
                out[t] = int(block_tables[s, j]) * page_size + pos % page_size
    return out


def reference_bd_slot_mapping(block_table_lists, to_cache, diffusion_block_size, page_size) -> list:
    """The reference runner's own loop (model_runner.py:141-151): per sequence ``[-1] * dbs`` while its last block
    is active, else the slot ranges of the last ``dbs // page_size`` pages of its table."""
    slots = []
    for table, store in zip(block_table_lists, to_cache):
        if not store:
            slots.extend([-1] * diffusion_block_size)
            continue
        n_pages = diffusion_block_size // page_size
        for i in range(n_pages):
            start = table[len(table) - n_pages + i] * page_size
            slots.extend(range(start, start + page_size))
    return slots
