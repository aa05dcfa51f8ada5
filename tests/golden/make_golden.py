"""Generate the golden fixtures in this directory by RUNNING THE REFERENCE on seeded inputs.

Usage (in a container that has the reference checkout; it is not needed to run the tests):

    python tests/golden/make_golden.py /path/to/Diffulex

What is run, unmodified, from the reference checkout:
  * store: ``store_kvcache_unified_layout`` (diffulex_kernel/python/kv_cache_kernels.py:110-124) and
    ``store_kvcache_distinct_layout`` (:86-107), their Triton kernels executed by the Triton interpreter
    (TRITON_INTERPRET=1) on CPU tensors;
  * load: ``load_kvcache`` (kv_cache_kernels.py:230-279), same way;
  * attention: ``naive_sdpa_with_kvcache`` (tests/python/kernel/
    test_dllm_flash_attn_decode_kernel.py:14-105) in fp32 on CPU, and for the block-causal
    cases ``naive_sdpa_prefill`` (tests/python/kernel/test_dllm_flash_attn_prefill_kernel.py:13-77).

bf16 tensors are handed to the Triton interpreter as their int16 bit patterns (a copy is a
copy); attention inputs are the bf16-rounded values widened to fp32.

Outputs: store_golden.json / store_distinct_golden.json / load_golden.json (sha256 digests: bit-exact work needs no more),
load_written_rows.npz (which rows the reference wrote), attn_golden.npz (fp32 outputs of a few
heads per case), prefill_golden.npz (``naive_sdpa_prefill`` on the prefill cases: fp32 outputs of two heads
and a seeded choice of rows per case).
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import numpy as np
import torch

from tests.golden.cases import (ATTN_CASES, D2F_CASES, LOAD_CASES, PREFILL_CASES, STORE_CASES, attn_problem, bits,
                                digest, distinct_caches, load_problem, prefill_fixture_index, prefill_inputs,
                                store_inputs)

SENTINEL = 1  # int16 bit pattern of a bf16 denormal; N(0,1) draws rounded to bf16 never produce it


def as_i16(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


def gen_store(ref_kv):
    out = {}
    for name, case in STORE_CASES.items():
        key, value, k_cache, v_cache, slots = store_inputs(case)
        in_digest = digest(key.contiguous(), value.contiguous(), k_cache, v_cache, slots)
        kc, vc = as_i16(k_cache).clone(), as_i16(v_cache).clone()
        ref_kv.store_kvcache_unified_layout(as_i16(key), as_i16(value), kc, vc, slots, None)
        out[name] = dict(inputs=in_digest, k_cache=digest(kc), v_cache=digest(vc))
        print("store", name, out[name]["k_cache"][:12])
    (HERE / "store_golden.json").write_text(json.dumps(out, indent=1))


def gen_store_distinct(ref_kv):
    out = {}
    for name, case in STORE_CASES.items():
        key, value, _, _, slots = store_inputs(case)
        k_cache, v_cache = distinct_caches(case)
        in_digest = digest(key.contiguous(), value.contiguous(), k_cache, v_cache, slots)
        kc, vc = as_i16(k_cache).clone(), as_i16(v_cache).clone()
        ref_kv.store_kvcache_distinct_layout(as_i16(key), as_i16(value), kc, vc, slots, None)
        out[name] = dict(inputs=in_digest, k_cache=digest(kc), v_cache=digest(vc))
        print("store distinct", name, out[name]["k_cache"][:12])
    (HERE / "store_distinct_golden.json").write_text(json.dumps(out, indent=1))


def gen_load(ref_kv):
    out, rows = {}, {}
    real_empty = torch.empty

    def sentinel_empty(*a, **kw):
        t = real_empty(*a, **kw)
        return t.fill_(SENTINEL) if t.dtype == torch.int16 else t

    for name, case in LOAD_CASES.items():
        p = load_problem(case)
        md = SimpleNamespace(block_tables=p.block_tables, context_lens=p.context_lens, seq_lens_ts=p.seq_lens_ts,
                             seqs=[SimpleNamespace(diffusion_block_size=p.geometry.diffusion_block_size)],
                             cu_seqlens_q=p.cu_seqlens_q, cu_seqlens_k=p.cu_seqlens_k_total)
        in_digest = digest(p.k_cache, p.v_cache, p.k, p.v, p.block_tables, p.context_lens, p.seq_lens_ts)
        ref_kv.torch.empty = sentinel_empty
        ref_kv.torch.empty_like = lambda t, **kw: sentinel_empty(t.shape, dtype=t.dtype)
        try:
            k_out, v_out = ref_kv.load_kvcache(as_i16(p.k_cache), as_i16(p.v_cache), md, as_i16(p.k), as_i16(p.v))
        finally:
            ref_kv.torch.empty = real_empty
            ref_kv.torch.empty_like = torch.empty_like
        written = ~(k_out == SENTINEL).all(-1).all(-1).numpy()
        assert np.array_equal(written, ~(v_out == SENTINEL).all(-1).all(-1).numpy())
        out[name] = dict(inputs=in_digest, rows=int(written.size), rows_written=int(written.sum()),
                         k_written=digest(k_out.numpy()[written]), v_written=digest(v_out.numpy()[written]))
        rows[name] = np.packbits(written)
        print("load", name, out[name]["rows_written"], "/", out[name]["rows"])
    (HERE / "load_golden.json").write_text(json.dumps(out, indent=1))
    np.savez(HERE / "load_written_rows.npz", **rows)


def gen_attn(ref_decode_test, ref_prefill_test):
    meta, arrays = {}, {}
    for name, case in ATTN_CASES.items():
        p = attn_problem(case)
        f = lambda t: t.float()
        o = ref_decode_test.naive_sdpa_with_kvcache(
            f(p.q), f(p.k), f(p.v), f(p.k_cache), f(p.v_cache), p.block_tables, p.context_lens,
            p.cu_seqlens_q, p.cu_seqlens_k, p.scale, p.geometry.group, p.geometry.page_size)
        arrays[name] = o[:, case["heads"]].numpy().astype(np.float32)
        meta[name] = dict(inputs=digest(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens),
                          heads=case["heads"], source="naive_sdpa_with_kvcache")
        print("attn", name, arrays[name].shape)
    for name, case in D2F_CASES.items():
        p = attn_problem(case)
        g = p.geometry
        # one block-causal "prefill" per sequence over [prefix ; in-flight]; prefix query rows are
        # placeholders whose outputs are discarded
        qs, ks, vs, cu = [], [], [], [0]
        for s in range(p.num_seqs):
            ctx, new = int(p.host_context_lens[s]), int(p.host_new_lens[s])
            q0 = int(p.cu_seqlens_q[s])
            pages = [int(x) for x in p.block_tables[s] if int(x) >= 0]
            kc = torch.cat([p.k_cache[i] for i in pages])[:ctx] if ctx else p.k_cache.new_zeros((0,) + p.k.shape[1:])
            vc = torch.cat([p.v_cache[i] for i in pages])[:ctx] if ctx else p.v_cache.new_zeros((0,) + p.v.shape[1:])
            qs.append(torch.cat([torch.zeros(ctx, g.num_q_heads, g.head_dim), p.q[q0:q0 + new].float()]))
            ks.append(torch.cat([kc.float(), p.k[q0:q0 + new].float()]))
            vs.append(torch.cat([vc.float(), p.v[q0:q0 + new].float()]))
            cu.append(cu[-1] + ctx + new)
        cu_t = torch.tensor(cu, dtype=torch.int32)
        o_all = ref_prefill_test.naive_sdpa_prefill(torch.cat(qs), torch.cat(ks), torch.cat(vs), cu_t, cu_t, p.scale,
                                                    g.diffusion_block_size, True)
        keep = torch.cat([o_all[cu[s] + int(p.host_context_lens[s]):cu[s + 1]] for s in range(p.num_seqs)])
        arrays[name] = keep[:, case["heads"]].numpy().astype(np.float32)
        meta[name] = dict(inputs=digest(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens),
                          heads=case["heads"], source="naive_sdpa_prefill(is_block_attn=True)")
        print("attn", name, arrays[name].shape)
    np.savez(HERE / "attn_golden.npz", **arrays)
    (HERE / "attn_golden.json").write_text(json.dumps(meta, indent=1))


def gen_prefill(ref_prefill_test):
    meta, arrays = {}, {}
    for name, case in PREFILL_CASES.items():
        q, k, v, cu_q, cu_k = prefill_inputs(case)
        o = ref_prefill_test.naive_sdpa_prefill(q.float(), k.float(), v.float(), cu_q, cu_k, case["hd"] ** -0.5,
                                                case["dbs"], case["block"])
        rows, heads = prefill_fixture_index(case)
        arrays[name] = o[rows][:, heads].numpy().astype(np.float32)
        meta[name] = dict(inputs=digest(q, k, v, cu_q, cu_k), source="naive_sdpa_prefill")
        print("prefill", name, arrays[name].shape)
    np.savez(HERE / "prefill_golden.npz", **arrays)
    (HERE / "prefill_golden.json").write_text(json.dumps(meta, indent=1))


def main():
    ref_root = Path(sys.argv[1]).resolve()
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(ref_root / "tests" / "python" / "kernel"))
    import diffulex_kernel.python.kv_cache_kernels as ref_kv
    gen_store(ref_kv)
    gen_store_distinct(ref_kv)
    gen_load(ref_kv)
    import test_dllm_flash_attn_decode_kernel as ref_decode_test
    import test_dllm_flash_attn_prefill_kernel as ref_prefill_test
    gen_attn(ref_decode_test, ref_prefill_test)
    gen_prefill(ref_prefill_test)


if __name__ == "__main__":
    main()
