"""Pins the CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py): store / load bit-exact, attention to fp32 round-off."""
import json

import numpy as np
import pytest
import torch

from oracle import attn_oracle, kv_cache_oracle
from tests.golden.cases import (ATTN_CASES, D2F_CASES, LOAD_CASES, PREFILL_CASES, STORE_CASES, attn_problem, bits,
                                digest, distinct_caches, load_problem, prefill_fixture_index, prefill_inputs,
                                store_inputs)


@pytest.fixture(scope="module")
def store_golden(golden_dir):
    return json.loads((golden_dir / "store_golden.json").read_text())


@pytest.fixture(scope="module")
def load_golden(golden_dir):
    return json.loads((golden_dir / "load_golden.json").read_text()), np.load(golden_dir / "load_written_rows.npz")


@pytest.fixture(scope="module")
def attn_golden(golden_dir):
    return json.loads((golden_dir / "attn_golden.json").read_text()), np.load(golden_dir / "attn_golden.npz")


@pytest.mark.parametrize("name", list(STORE_CASES))
def test_store_oracle_matches_reference(name, store_golden):
    key, value, k_cache, v_cache, slots = store_inputs(STORE_CASES[name])
    g = store_golden[name]
    assert digest(key.contiguous(), value.contiguous(), k_cache, v_cache, slots) == g["inputs"], "inputs drifted"
    kc, vc = bits(k_cache).copy(), bits(v_cache).copy()
    kv_cache_oracle.store_kvcache_unified(bits(key), bits(value), kc, vc, slots.numpy())
    assert digest(kc) == g["k_cache"]
    assert digest(vc) == g["v_cache"]


@pytest.mark.parametrize("name", list(STORE_CASES))
def test_distinct_store_oracle_matches_reference(name, golden_dir):
    """The split-layout store oracle against what the reference's own Triton kernel wrote (interpreter run)."""
    g = json.loads((golden_dir / "store_distinct_golden.json").read_text())[name]
    key, value, _, _, slots = store_inputs(STORE_CASES[name])
    k_cache, v_cache = distinct_caches(STORE_CASES[name])
    assert digest(key.contiguous(), value.contiguous(), k_cache, v_cache, slots) == g["inputs"], "inputs drifted"
    kc, vc = bits(k_cache).copy(), bits(v_cache).copy()
    kv_cache_oracle.store_kvcache_distinct(bits(key), bits(value), kc, vc, slots.numpy())
    assert digest(kc) == g["k_cache"]
    assert digest(vc) == g["v_cache"]


@pytest.mark.parametrize("name", list(LOAD_CASES))
def test_load_oracle_matches_reference_on_rows_it_writes(name, load_golden):
    meta, rows = load_golden
    p = load_problem(LOAD_CASES[name])
    g = meta[name]
    assert digest(p.k_cache, p.v_cache, p.k, p.v, p.block_tables, p.context_lens, p.seq_lens_ts) == g["inputs"]
    k_out, v_out = kv_cache_oracle.load_kvcache(
        bits(p.k_cache), bits(p.v_cache), p.block_tables.numpy(), p.context_lens.numpy(), p.seq_lens_ts.numpy(),
        p.cu_seqlens_q.numpy(), p.cu_seqlens_k_total.numpy(), bits(p.k), bits(p.v))
    written = np.unpackbits(rows[name])[: g["rows"]].astype(bool)
    # the oracle's model of which rows the reference leaves unwritten agrees with what it did
    model = kv_cache_oracle.reference_written_rows(
        p.geometry.page_size, p.block_tables.numpy(), p.context_lens.numpy(), p.seq_lens_ts.numpy(),
        p.cu_seqlens_k_total.numpy(), p.geometry.diffusion_block_size)
    assert np.array_equal(model, written)
    assert int(written.sum()) == g["rows_written"]
    assert digest(k_out[written]) == g["k_written"]
    assert digest(v_out[written]) == g["v_written"]


@pytest.mark.parametrize("name", list(ATTN_CASES) + list(D2F_CASES))
def test_attention_oracle_matches_reference(name, attn_golden):
    meta, arrays = attn_golden
    case = ATTN_CASES.get(name) or D2F_CASES[name]
    p = attn_problem(case)
    assert digest(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens) == meta[name]["inputs"]
    o = attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                     p.cu_seqlens_q, p.cu_seqlens_k, p.scale, p.mask_mode,
                                     p.geometry.diffusion_block_size)
    want = torch.from_numpy(arrays[name])
    torch.testing.assert_close(o[:, meta[name]["heads"]], want, atol=2e-5, rtol=1e-5)


def test_attention_oracle_varlen_offsets():
    """cu_seqlens_k cumulating ctx+new (varlen convention) gives the same result when the
    in-flight rows are addressed through cu_seqlens_q."""
    p = attn_problem(ATTN_CASES["ragged_q"])
    a = attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                     p.cu_seqlens_q, p.cu_seqlens_k, p.scale)
    b = attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                     p.cu_seqlens_q, p.cu_seqlens_k_total, p.scale, kv_offsets_from_q=True)
    assert torch.equal(a, b)


@pytest.mark.parametrize("name", list(PREFILL_CASES))
def test_prefill_oracle_matches_reference(name, golden_dir):
    """The prefill oracle against the reference's own prefill check run on the same seeded prompts."""
    meta = json.loads((golden_dir / "prefill_golden.json").read_text())[name]
    want = torch.from_numpy(np.load(golden_dir / "prefill_golden.npz")[name])
    case = PREFILL_CASES[name]
    q, k, v, cu_q, cu_k = prefill_inputs(case)
    assert digest(q, k, v, cu_q, cu_k) == meta["inputs"], "inputs drifted"
    o = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, case["hd"] ** -0.5, case["block"], case["dbs"])
    rows, heads = prefill_fixture_index(case)
    torch.testing.assert_close(o[rows][:, heads], want, atol=2e-5, rtol=1e-5)


def test_slot_mapping_oracle_restates_the_runner_loop_and_the_workload_generator():
    """Positions through the page table == the reference runner's whole-page lists when pages divide the block
    (diffulex/strategy/block_diffusion/engine/model_runner.py:141-151), == the slots the seeded workloads carry."""
    from diffulex_b200.workload import make_problem, small_workload
    rng = np.random.default_rng(7)
    dbs, page = 32, 16
    # block-aligned contexts, tables that end with the pages of the in-flight block
    ctx = np.array([64, 0, 160, 32]); to_cache = [True, False, True, True]
    tables, nb = [], 0
    for c in ctx:
        n = (c + dbs) // page
        tables.append(list(rng.permutation(200)[:n] + 0)); nb = max(nb, n)
    bt = np.full((len(ctx), nb), -1, dtype=np.int32)
    for s, t in enumerate(tables):
        bt[s, :len(t)] = t
    cu_q = np.arange(0, (len(ctx) + 1) * dbs, dbs, dtype=np.int32)
    got = kv_cache_oracle.build_slot_mapping(bt, ctx.astype(np.int32), cu_q, page, int(cu_q[-1]),
                                             np.array(to_cache, dtype=np.int32))
    want = kv_cache_oracle.reference_bd_slot_mapping(tables, to_cache, dbs, page)
    assert got.tolist() == want
    # the seeded workloads' slot mappings (ragged contexts, 64- and 256-row pages, permuted tables)
    for name in ("ragged_q", "cfg1", "q4_gqa4"):
        p = attn_problem(ATTN_CASES[name])
        got = kv_cache_oracle.build_slot_mapping(p.block_tables.numpy(), p.context_lens.numpy(), p.cu_seqlens_q.numpy(),
                                                 p.geometry.page_size, p.q.shape[0])
        assert np.array_equal(got, p.slot_mapping.numpy().astype(np.int64))
