"""GPU parity: the CUDA path (through the reference-shaped Python entry points, i.e. through the
C ABI) against the golden vectors and the CPU oracle on the same seeded inputs.

Store / load: bit-exact.  Attention: max-abs 2e-2 / rel 1e-2 in bf16 (ATOL / RTOL below)."""
import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import attn_oracle, kv_cache_oracle
from tests.golden.cases import (ATTN_CASES, D2F_CASES, LOAD_CASES, STORE_CASES, attn_problem, bits, digest,
                                load_problem, store_inputs)

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
KERNELS = {"auto": 0, "mma": 1, "tc5": 2, "pair": 3}


@pytest.fixture(scope="module")
def dlx():
    import diffulex_b200
    assert torch.cuda.is_available(), "these tests need a CUDA device"
    return diffulex_b200


def to_dev(p):
    """Copy of a DecodeProblem with every tensor on cuda:0."""
    kw = {}
    for f in p.__dataclass_fields__:
        v = getattr(p, f)
        kw[f] = v.cuda() if isinstance(v, torch.Tensor) else v
    return type(p)(**kw)


def oracle_out(p, kv_offsets_from_q=False):
    cu_k = p.cu_seqlens_k_total if kv_offsets_from_q else p.cu_seqlens_k
    return attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                        p.cu_seqlens_q, cu_k, p.scale, p.mask_mode,
                                        p.geometry.diffusion_block_size, kv_offsets_from_q=kv_offsets_from_q)


def run_decode(dlx, pd, mode="static", num_splits=0):
    md = pd.metadata(mode)
    md.num_splits = num_splits
    return dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)


# ---- store -------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(STORE_CASES))
def test_store_bit_exact(name, dlx, golden_dir):
    golden = json.loads((golden_dir / "store_golden.json").read_text())[name]
    key, value, k_cache, v_cache, slots = store_inputs(STORE_CASES[name])
    kc_ref, vc_ref = bits(k_cache).copy(), bits(v_cache).copy()
    kv_cache_oracle.store_kvcache_unified(bits(key), bits(value), kc_ref, vc_ref, slots.numpy())
    kd, vd = key.cuda(), value.cuda()
    if not key.is_contiguous():  # keep the row padding on the device too
        n, h, d = key.shape
        wide_k = torch.zeros(n, key.stride(0), dtype=key.dtype, device="cuda")
        wide_v = torch.zeros_like(wide_k)
        wide_k[:, : h * d] = key.reshape(n, -1).cuda()
        wide_v[:, : h * d] = value.reshape(n, -1).cuda()
        kd, vd = wide_k[:, : h * d].view(n, h, d), wide_v[:, : h * d].view(n, h, d)
        assert kd.stride(0) == key.stride(0)
    kc, vc = k_cache.cuda(), v_cache.cuda()
    ret = dlx.store_kvcache_unified_layout(kd, vd, kc, vc, slots.cuda(), None)
    assert ret is None
    torch.cuda.synchronize()
    assert np.array_equal(bits(kc), kc_ref) and np.array_equal(bits(vc), vc_ref)
    assert digest(kc.cpu()) == golden["k_cache"] and digest(vc.cpu()) == golden["v_cache"]


@pytest.mark.parametrize("name", list(STORE_CASES))
def test_store_distinct_layout_bit_exact(name, dlx, golden_dir):
    """Split layout (K [NB, H, hd/x, PAGE, x], V [NB, H, hd, PAGE]): bit-exact against the oracle and against the
    digests of what the reference's own kernel wrote; int32 and int64 slots, skipped rows, strided key rows."""
    from tests.golden.cases import distinct_caches
    golden = json.loads((golden_dir / "store_distinct_golden.json").read_text())[name]
    key, value, _, _, slots = store_inputs(STORE_CASES[name])
    kc, vc = distinct_caches(STORE_CASES[name])
    kc_ref, vc_ref = bits(kc).copy(), bits(vc).copy()
    kv_cache_oracle.store_kvcache_distinct(bits(key), bits(value), kc_ref, vc_ref, slots.numpy())
    kd, vd = key.cuda(), value.cuda()
    if not key.is_contiguous():  # keep the row padding on the device too
        n, h, d = key.shape
        wide_k = torch.zeros(n, key.stride(0), dtype=key.dtype, device="cuda")
        wide_v = torch.zeros_like(wide_k)
        wide_k[:, : h * d] = key.reshape(n, -1).cuda()
        wide_v[:, : h * d] = value.reshape(n, -1).cuda()
        kd, vd = wide_k[:, : h * d].view(n, h, d), wide_v[:, : h * d].view(n, h, d)
    kcd, vcd = kc.cuda(), vc.cuda()
    assert dlx.store_kvcache_distinct_layout(kd, vd, kcd, vcd, slots.cuda(), None) is None
    torch.cuda.synchronize()
    assert np.array_equal(bits(kcd), kc_ref) and np.array_equal(bits(vcd), vc_ref)
    assert digest(kcd.cpu()) == golden["k_cache"] and digest(vcd.cpu()) == golden["v_cache"]


# ---- slot mapping built on the device ----------------------------------------------------------
@pytest.mark.parametrize("name", ["cfg1", "ragged_q", "ragged_permuted", "q4_gqa4"])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_slot_mapping_built_on_the_device_bit_exact(name, dtype, dlx):
    """Against the oracle: every sequence storing, some sequences still denoising (-1 rows), a zero-filled padded
    tail as a replayed graph's static buffers have it, and rows behind the last sequence."""
    from diffulex_b200 import ops
    p = attn_problem(ATTN_CASES[name])
    pd = to_dev(p)
    g = p.geometry
    rows, nb = p.q.shape[0], p.k_cache.shape[0]
    got = ops.build_slot_mapping(pd.block_tables, pd.context_lens, pd.cu_seqlens_q, g.page_size, rows, nb, dtype=dtype)
    want = kv_cache_oracle.build_slot_mapping(p.block_tables.numpy(), p.context_lens.numpy(), p.cu_seqlens_q.numpy(),
                                              g.page_size, rows)
    assert got.dtype == dtype and np.array_equal(got.cpu().numpy().astype(np.int64), want)
    assert np.array_equal(want, p.slot_mapping.numpy().astype(np.int64))
    flags = torch.tensor([s % 2 for s in range(p.num_seqs)], dtype=torch.int32)
    pad = 5
    z = lambda t, n: torch.cat([t, torch.zeros(n, dtype=t.dtype)])
    cu_q, ctx = z(p.cu_seqlens_q, pad), z(p.context_lens, pad)
    bt = torch.cat([p.block_tables, torch.zeros(pad, p.block_tables.shape[1], dtype=torch.int32)])
    fl = z(flags, pad)
    out = torch.full((rows + 7,), 12345, dtype=dtype, device="cuda")
    ret = ops.build_slot_mapping(bt.cuda(), ctx.cuda(), cu_q.cuda(), g.page_size, rows + 7, nb, store_flags=fl.cuda(),
                                 out=out)
    assert ret is out
    want = kv_cache_oracle.build_slot_mapping(bt.numpy(), ctx.numpy(), cu_q.numpy(), g.page_size, rows + 7, fl.numpy())
    assert (want[rows:] == -1).all()
    assert np.array_equal(out.cpu().numpy().astype(np.int64), want)


# ---- load --------------------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(LOAD_CASES))
def test_load_bit_exact(name, dlx, golden_dir):
    golden = json.loads((golden_dir / "load_golden.json").read_text())[name]
    rows = np.load(golden_dir / "load_written_rows.npz")[name]
    p = load_problem(LOAD_CASES[name])
    k_ref, v_ref = kv_cache_oracle.load_kvcache(
        bits(p.k_cache), bits(p.v_cache), p.block_tables.numpy(), p.context_lens.numpy(), p.seq_lens_ts.numpy(),
        p.cu_seqlens_q.numpy(), p.cu_seqlens_k_total.numpy(), bits(p.k), bits(p.v))
    pd = to_dev(p)
    md = pd.metadata("varlen")
    for hint in (None, int(p.cu_seqlens_k_total[-1])):
        md.total_kv_rows = hint
        k_out, v_out = dlx.load_kvcache(pd.k_cache, pd.v_cache, md, pd.k, pd.v)
        assert k_out.shape == (int(p.cu_seqlens_k_total[-1]), p.geometry.num_kv_heads, p.geometry.head_dim)
        # every row, against the oracle
        assert np.array_equal(bits(k_out), k_ref) and np.array_equal(bits(v_out), v_ref)
        # the rows the reference kernel writes, against its own output
        written = np.unpackbits(rows)[: golden["rows"]].astype(bool)
        assert digest(bits(k_out)[written]) == golden["k_written"]
        assert digest(bits(v_out)[written]) == golden["v_written"]


# ---- attention ---------------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(ATTN_CASES) + list(D2F_CASES))
@pytest.mark.parametrize("mode", ["static", "varlen"])
@pytest.mark.parametrize("num_splits", [0, 1, 3])
@pytest.mark.parametrize("kernel", ["auto", "tc5", "pair", "mma"])
def test_attention_matches_golden_and_oracle(name, mode, num_splits, kernel, dlx, golden_dir, monkeypatch):
    # "auto": head_dim 128 goes to a tcgen05 kernel (the CTA-pair kernel for more than 128 packed rows per KV head,
    # the single-CTA kernel otherwise), everything else to the mma.sync kernel; the other three force one kernel.
    # Forcing "pair" on a short query block runs the pair with an idle second CTA.
    from diffulex_b200 import ops
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    meta = json.loads((golden_dir / "attn_golden.json").read_text())[name]
    want_sel = torch.from_numpy(np.load(golden_dir / "attn_golden.npz")[name])
    p = attn_problem(ATTN_CASES.get(name) or D2F_CASES[name])
    if kernel in ("tc5", "pair") and p.geometry.head_dim != 128:
        pytest.skip("the tcgen05 kernels serve head_dim 128")
    want = oracle_out(p)
    pd = to_dev(p)
    o = run_decode(dlx, pd, mode, num_splits)
    assert o.dtype == torch.bfloat16 and o.shape == p.q.shape
    got = o.float().cpu()
    torch.testing.assert_close(got, want, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(got[:, meta["heads"]], want_sel, atol=ATOL, rtol=RTOL)


def test_attention_strided_q_and_out_of_fused_projection(dlx):
    """q/k/v as column slices of one fused projection output (row stride > heads*hd)."""
    p = attn_problem(ATTN_CASES["ragged_q"])
    want = oracle_out(p)
    pd = to_dev(p)
    g = p.geometry
    nq, nkv = g.num_q_heads * g.head_dim, g.num_kv_heads * g.head_dim
    fused = torch.zeros(p.q.shape[0], nq + 2 * nkv, dtype=torch.bfloat16, device="cuda")
    fused[:, :nq] = pd.q.reshape(-1, nq)
    fused[:, nq:nq + nkv] = pd.k.reshape(-1, nkv)
    fused[:, nq + nkv:] = pd.v.reshape(-1, nkv)
    pd.q = fused[:, :nq].view(-1, g.num_q_heads, g.head_dim)
    pd.k = fused[:, nq:nq + nkv].view(-1, g.num_kv_heads, g.head_dim)
    pd.v = fused[:, nq + nkv:].view(-1, g.num_kv_heads, g.head_dim)
    o = run_decode(dlx, pd)
    torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)


def test_attention_padded_batch_like_graph_replay(dlx):
    """CUDA-graph replay zero-fills the static metadata buffers, so padded sequences carry
    cu_seqlens of 0 (non-positive lengths) and context_lens 0 (diffulex/strategy/block_diffusion/
    engine/model_runner.py:183-195): they must be skipped and real rows must be unaffected."""
    p = attn_problem(ATTN_CASES["ragged_permuted"])
    want = oracle_out(p)
    pd = to_dev(p)
    pad = 3
    z = lambda t, n: torch.cat([t, torch.zeros(n, dtype=t.dtype, device=t.device)])
    pd.cu_seqlens_q, pd.cu_seqlens_k = z(pd.cu_seqlens_q, pad), z(pd.cu_seqlens_k, pad)
    pd.context_lens = z(pd.context_lens, pad)
    pd.block_tables = torch.cat([pd.block_tables, torch.zeros(pad, pd.block_tables.shape[1], dtype=torch.int32,
                                                              device="cuda")])
    for splits in (0, 2):
        o = run_decode(dlx, pd, "static", splits)
        torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_named_workloads_store_then_decode(name, dlx):
    """The benchmark configurations at full size (one layer): store the in-flight block, then
    decode, exactly the order of Attention.forward (diffulex/attention/attn_impl.py:53-67)."""
    from diffulex_b200.workload import make_problem, named_workload
    p = make_problem(named_workload(name), device="cpu", values="numpy")
    want = oracle_out(p)
    kc_ref, vc_ref = bits(p.k_cache).copy(), bits(p.v_cache).copy()
    kv_cache_oracle.store_kvcache_unified(bits(p.k), bits(p.v), kc_ref, vc_ref, p.slot_mapping.numpy())
    pd = to_dev(p)
    md = pd.metadata("static")
    dlx.store_kvcache_unified_layout(pd.k, pd.v, pd.k_cache, pd.v_cache, md.slot_mapping, md)
    o = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    assert np.array_equal(bits(pd.k_cache), kc_ref) and np.array_equal(bits(pd.v_cache), vc_ref)
    torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)
    # varlen convention (cu_seqlens_k cumulates ctx+new) gives the same numbers
    o2 = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, pd.metadata("varlen"))
    torch.testing.assert_close(o2.float().cpu(), want, atol=ATOL, rtol=RTOL)


def test_cuda_graph_capture_store_and_decode(dlx):
    p = attn_problem(ATTN_CASES["cfg1"])
    want = oracle_out(p)
    pd = to_dev(p)
    md = pd.metadata("static")
    md.num_splits = 2
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            dlx.store_kvcache_unified_layout(pd.k, pd.v, pd.k_cache, pd.v_cache, md.slot_mapping, md)
            dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dlx.store_kvcache_unified_layout(pd.k, pd.v, pd.k_cache, pd.v_cache, md.slot_mapping, md)
        o = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    pd.q.copy_(pd.q.flip(0))  # new contents in the captured buffers
    g.replay()
    torch.cuda.synchronize()
    p.q = p.q.flip(0)
    torch.testing.assert_close(o.float().cpu(), oracle_out(p), atol=ATOL, rtol=RTOL)
    assert not torch.equal(oracle_out(p), want)


# ---- full-size properties (sizes the oracle cannot finish in seconds) ---------------------------
@pytest.fixture(scope="module")
def cfg5_problem():
    from diffulex_b200.workload import make_problem, named_workload
    return make_problem(named_workload("cfg5"), device="cuda", values="torch")


def test_cfg5_store_load_round_trip(dlx, cfg5_problem):
    """Scaling-sweep size (4.7 M cached tokens, caches > 2^31 elements: 64-bit offsets).  Store the
    in-flight block, gather everything, and check (a) in-flight rows come back twice (from the cache
    slots and as the fresh tail), (b) a byte checksum of all gathered rows equals the checksum of
    the source rows computed by torch indexing."""
    pd = cfg5_problem
    g = pd.geometry
    assert pd.k_cache.numel() > 2 ** 31
    md = pd.metadata("varlen")
    dlx.store_kvcache_unified_layout(pd.k, pd.v, pd.k_cache, pd.v_cache, md.slot_mapping, md)
    flat_k = pd.k_cache.view(-1, g.num_kv_heads, g.head_dim)
    assert torch.equal(flat_k[pd.slot_mapping.long()], pd.k)
    # now treat the stored block as cached: ctx' = ctx + new
    md2 = pd.metadata("varlen")
    md2.context_lens = pd.context_lens + pd.seq_lens_ts
    md2.cu_seqlens_k = pd.cu_seqlens_k_total + pd.cu_seqlens_q  # cumulates ctx' + new
    md2.total_kv_rows = int(pd.host_context_lens.sum() + 2 * pd.host_new_lens.sum())
    k_out, v_out = dlx.load_kvcache(pd.k_cache, pd.v_cache, md2, pd.k, pd.v)
    cu = md2.cu_seqlens_k.cpu().numpy()
    ctx2 = (pd.host_context_lens + pd.host_new_lens)
    for s in (0, 17, 255):
        new = int(pd.host_new_lens[s])
        tail = k_out[cu[s] + ctx2[s]: cu[s] + ctx2[s] + new]
        again = k_out[cu[s] + ctx2[s] - new: cu[s] + ctx2[s]]
        assert torch.equal(tail, pd.k[int(pd.cu_seqlens_q[s]):int(pd.cu_seqlens_q[s]) + new])
        assert torch.equal(tail, again)
    # checksum of checksums over every gathered row vs torch's own gather of the same rows
    pos = torch.cat([torch.arange(int(c), device="cuda") for c in ctx2])
    seq = torch.repeat_interleave(torch.arange(len(ctx2), device="cuda"), torch.as_tensor(ctx2, device="cuda"))
    slots = pd.block_tables[seq, pos // g.page_size].long() * g.page_size + pos % g.page_size
    is_ctx = torch.ones(k_out.shape[0], dtype=torch.bool, device="cuda")
    for s in range(len(ctx2)):
        is_ctx[cu[s] + ctx2[s]: cu[s + 1]] = False
    for out, cache in ((k_out, pd.k_cache), (v_out, pd.v_cache)):
        got = out.view(torch.int16)[is_ctx].sum(dim=(1, 2), dtype=torch.int64)
        want = cache.view(-1, g.num_kv_heads, g.head_dim).view(torch.int16)[slots].sum(dim=(1, 2), dtype=torch.int64)
        assert torch.equal(got, want)


def test_cfg5_attention_properties(dlx, cfg5_problem):
    """(a) split invariance: forced 1 / planned / 7 key-range splits agree within tolerance;
    (b) rows of softmax sum to one: with V == 1 everywhere the output is 1;
    (c) the three longest-context-independent sequences picked match the fp32 oracle."""
    pd = cfg5_problem
    o_auto = run_decode(dlx, pd)
    o_1 = run_decode(dlx, pd, num_splits=1)
    o_7 = run_decode(dlx, pd, num_splits=7)
    torch.testing.assert_close(o_auto.float(), o_1.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(o_7.float(), o_1.float(), atol=ATOL, rtol=RTOL)
    ones_c, ones_n = torch.ones_like(pd.v_cache), torch.ones_like(pd.v)
    md = pd.metadata("static")
    o_ones = dlx.dllm_flash_attn_decode(pd.q, pd.k, ones_n, pd.k_cache, ones_c, pd.scale, md)
    torch.testing.assert_close(o_ones.float(), torch.ones_like(o_ones, dtype=torch.float32), atol=1e-2, rtol=0)
    del ones_c
    for s in (3, 100, 200):
        q0, q1 = int(pd.cu_seqlens_q[s]), int(pd.cu_seqlens_q[s + 1])
        ctx = int(pd.host_context_lens[s])
        pages = pd.block_tables[s][: (ctx + pd.geometry.page_size - 1) // pd.geometry.page_size].long()
        kc, vc = pd.k_cache[pages].cpu(), pd.v_cache[pages].cpu()
        bt = torch.arange(len(pages), dtype=torch.int32).unsqueeze(0)
        cu = torch.tensor([0, q1 - q0], dtype=torch.int32)
        want = attn_oracle.decode_attention(pd.q[q0:q1].cpu(), pd.k[q0:q1].cpu(), pd.v[q0:q1].cpu(), kc, vc, bt,
                                            torch.tensor([ctx], dtype=torch.int32), cu, cu, pd.scale)
        torch.testing.assert_close(o_auto[q0:q1].float().cpu(), want, atol=ATOL, rtol=RTOL)


def device_status():
    from diffulex_b200 import ops
    return list(ops.device_status())


@pytest.mark.parametrize("kernel", ["tc5", "pair"])
def test_tcgen05_kernels_are_taken_and_no_wait_expired(kernel, dlx, monkeypatch):
    """Forcing a tcgen05 kernel works on eligible shapes (head_dim 128: 7 and 4 query heads per KV head
    here), is refused on an ineligible one (head_dim 64), and the kernels' bounded waits never ran
    out during this test session."""
    from diffulex_b200 import _lib, ops
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    p = attn_problem(ATTN_CASES["cfg1"])
    for splits in (0, 2):
        o = run_decode(dlx, to_dev(p), "static", splits)
        torch.testing.assert_close(o.float().cpu(), oracle_out(p), atol=ATOL, rtol=RTOL)
    p4 = attn_problem(ATTN_CASES["q4_gqa4"])
    torch.testing.assert_close(run_decode(dlx, to_dev(p4)).float().cpu(), oracle_out(p4), atol=ATOL, rtol=RTOL)
    with pytest.raises(_lib.DlxError):
        run_decode(dlx, to_dev(attn_problem(ATTN_CASES["ref_head_dim_64"])))
    st = device_status()
    assert st == [0, 0, 0, 0], f"a bounded wait expired: {st}"


@pytest.mark.parametrize("kernel", ["tc5", "pair"])
def test_more_items_than_the_placement_sorts_and_the_item_table_holds(kernel, dlx, monkeypatch):
    """300 sequences x 32 KV heads = 9600 work items: more than the schedule kernel sorts (it deals them
    round-robin instead) and 65 / 130 rounds per persistent CTA / CTA pair: more than the kernels' shared-memory
    record tables hold, so later rounds are read from the global records."""
    from diffulex_b200 import ops
    from diffulex_b200.workload import MASK_BD_FULL, make_problem, small_workload
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    rng = np.random.default_rng(5)
    ctx = rng.integers(0, 200, size=300).tolist()
    w = small_workload("many_items", 32, 32, 128, 32, 4, ctx, [4] * 300, MASK_BD_FULL, 41)
    p = make_problem(w, device="cpu", values="numpy")
    o = run_decode(dlx, to_dev(p), "static", 1)
    torch.testing.assert_close(o.float().cpu(), oracle_out(p), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", ["tc5", "pair"])
def test_scores_far_above_the_first_tile_are_exact(kernel, dlx, monkeypatch):
    """The tcgen05 kernels scale a row's exponentials by the maximum of the item's FIRST key tile and never
    rescale.  Two keys whose scores lie ~200 and ~180 log2-units above everything else (in a later tile) leave the
    range in which that is exact; the kernels notice (row sum of the tile) and compute the item again with a
    running maximum, so the output still matches the oracle: their weights differ by 2^-20, i.e. the output
    is the higher key's V row."""
    from diffulex_b200 import ops
    from diffulex_b200.workload import MASK_BD_FULL, make_problem, small_workload
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    w = small_workload("hot_keys", 28, 4, 128, 64, 32, [300, 520], [32, 32], MASK_BD_FULL, 77)
    p = make_problem(w, device="cpu", values="numpy")
    u = p.q[0, 0].clone()
    p.q[:] = u                                         # every row asks the same question ...
    for s in range(2):                                 # ... and keys 5 and 9 of every sequence answer it loudly
        page = int(p.block_tables[s, 0])
        p.k_cache[page, 5] = (12.0 * u).to(p.k_cache.dtype)
        p.k_cache[page, 9] = (11.0 * u).to(p.k_cache.dtype)
    want = oracle_out(p)
    for splits in (1, 2):
        o = run_decode(dlx, to_dev(p), "static", splits)
        assert torch.isfinite(o).all()
        torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)
    # mixed case: only sequence 1 is out of range, sequence 0 takes the fast path
    page = int(p.block_tables[0, 0])
    p.k_cache[page, 5] = p.k_cache[page, 6]
    p.k_cache[page, 9] = p.k_cache[page, 6]
    o = run_decode(dlx, to_dev(p), "static", 1)
    torch.testing.assert_close(o.float().cpu(), oracle_out(p), atol=ATOL, rtol=RTOL)
    assert device_status() == [0, 0, 0, 0]


@pytest.mark.parametrize("kernel", ["tc5", "pair"])
def test_rows_that_see_nothing_of_the_first_tile_are_exact(kernel, dlx, monkeypatch):
    """Block-causal rows of an early in-flight block see none of the keys of the item's first tile (a late one),
    so their softmax reference comes from keys hidden to them.  Here those hidden keys score ~200 log2-units
    above the visible ones: every exponential of such a row underflows, the kernels notice (row sum ~ 0 although
    keys are visible) and recompute the item exactly."""
    from diffulex_b200 import ops
    from diffulex_b200.workload import MASK_D2F_BLOCK_CAUSAL, make_problem, small_workload
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    w = small_workload("hidden_first_tile", 28, 4, 128, 64, 32, [64, 10], [256, 224], MASK_D2F_BLOCK_CAUSAL, 78)
    p = make_problem(w, device="cpu", values="numpy")
    u = p.q[0, 0].clone()
    p.q[:] = u
    p.k[128:] = (12.0 * u).to(p.k.dtype)               # in-flight keys 128.. of sequence 0 (and all of sequence 1)
    want = oracle_out(p)
    o = run_decode(dlx, to_dev(p), "static", 1)
    assert torch.isfinite(o).all()
    torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)
    assert device_status() == [0, 0, 0, 0]


def parse_schedule(sched, bins):
    """(offsets, records) of a schedule buffer: int32 offsets[bins + 1] in a 1 KiB header, then 32-int records
    (seq, kvh, mb, split, q0, qn, ctx, kv0, nnew, t0, n, flags, first_page, n_pages, limit, -, pages[16])."""
    raw = sched.cpu().numpy().view(np.int32)
    off = raw[: bins + 1]
    recs = raw[256:].reshape(-1, 32)
    return off, recs


def test_schedule_covers_every_item_once_and_balances(dlx):
    """The device-built schedule of benchmark configuration 2: 256 (sequence, KV head) items on 74 CTA pairs, every
    item exactly once, longest first inside a pair, loads within one item of each other, page ids attached."""
    from diffulex_b200 import ops
    from diffulex_b200.workload import make_problem, named_workload
    p = make_problem(named_workload("cfg2"), device="cuda", values="torch")
    md = p.metadata("static")
    sched = ops.decode_schedule(p.q, p.k, p.k_cache, p.v_cache, p.block_tables, p.context_lens, p.cu_seqlens_q,
                                p.cu_seqlens_k, p.scale, md.max_seqlen_q, 0, p.mask_mode, 32, 0)
    off, recs = parse_schedule(sched, 74)
    assert off[0] == 0 and off[74] == 256 and np.all(np.diff(off) >= 1)
    recs = recs[:256]
    assert sorted(map(tuple, recs[:, :4])) == sorted((s, h, 0, 0) for s in range(64) for h in range(4))
    ctx = p.host_context_lens
    bt = p.block_tables.cpu().numpy()
    loads = []
    for b in range(74):
        mine = recs[off[b]:off[b + 1]]
        assert np.all(np.diff(mine[:, 10]) <= 0), "longest item first"
        loads.append(int(mine[:, 10].sum() + len(mine)))
        for r in mine:
            s = int(r[0])
            assert r[6] == ctx[s] and r[5] == 32 and r[8] == 32 and r[9] == 0 and r[11] == 1
            assert r[10] == (ctx[s] + 32 + 127) // 128 and r[14] == ctx[s] + 32
            last_page = (ctx[s] - 1) // 256
            assert r[12] == max(0, last_page - 15) and r[13] == last_page - r[12] + 1
            assert np.array_equal(r[16:16 + r[13]], bt[s, r[12]:r[12] + r[13]])
    assert max(loads) - min(loads) <= int(recs[:, 10].max()) + 1


def test_captured_step_replans_when_the_metadata_buffers_are_refilled(dlx):
    """A captured decode step holds its planning launch: after the runner refills the static metadata buffers
    in place with other lengths (diffulex/strategy/block_diffusion/engine/model_runner.py:183-195), a replay
    matches the oracle of the NEW step and its schedule follows the new lengths."""
    from diffulex_b200.workload import MASK_BD_FULL, make_problem, small_workload
    mk = lambda ctx, seed: make_problem(small_workload("replan", 28, 4, 128, 256, 32, ctx, [32] * 4, MASK_BD_FULL, seed,
                                                       spare_pages=24), device="cpu", values="numpy")
    pa, pb = mk([900, 100, 400, 30], 91), mk([60, 950, 200, 300], 92)
    assert pa.k_cache.shape == pb.k_cache.shape and pa.block_tables.shape == pb.block_tables.shape
    pd = to_dev(pa)
    md = pd.metadata("static")
    md.num_splits = 1
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        o1 = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
        o2 = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)   # second layer: same plan
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(o1.float().cpu(), oracle_out(pa), atol=ATOL, rtol=RTOL)
    for name in ("q", "k", "v", "k_cache", "v_cache", "block_tables", "context_lens"):
        getattr(pd, name).copy_(getattr(pb, name))
    g.replay()
    torch.cuda.synchronize()
    want = oracle_out(pb)
    torch.testing.assert_close(o1.float().cpu(), want, atol=ATOL, rtol=RTOL)
    assert torch.equal(o1, o2)
    bins = 16   # 4 sequences x 4 KV heads: one item per CTA pair
    off, recs = parse_schedule(md._dlx_plan[1].schedule, bins)
    recs = recs[: off[bins]]
    new_ctx = pb.host_context_lens
    assert all(r[6] == new_ctx[r[0]] for r in recs)
    assert [int(r[0]) for r in recs[:4]] == [1, 1, 1, 1], "the longest sequence of the NEW step comes first"


# ---- decode that also stores -------------------------------------------------------------------
@pytest.mark.parametrize("kernel", ["auto", "tc5", "pair", "mma"])
@pytest.mark.parametrize("num_splits", [0, 3])
@pytest.mark.parametrize("name", ["cfg1", "ragged_q", "ragged_permuted", "q4_gqa4", "ref_head_dim_64", "d2f_gqa7"])
def test_decode_that_also_stores_equals_store_then_decode(name, num_splits, kernel, dlx, monkeypatch):
    """``store_slot_mapping``: one call does the layer's store and its attention.  Caches bit-exact against the
    store oracle (some rows skipped through negative slots, int32 and int64 slots), output against the attention
    oracle; on every kernel (the ones that do not store by themselves run the store kernel first)."""
    from diffulex_b200 import ops
    case = ATTN_CASES.get(name) or D2F_CASES[name]
    p = attn_problem(case)
    if kernel in ("tc5", "pair") and p.geometry.head_dim != 128:
        pytest.skip("the tcgen05 kernels serve head_dim 128")
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    want = oracle_out(p)
    for slot_dtype, drop in ((torch.int32, 0), (torch.int64, 3)):
        slots = p.slot_mapping.clone().to(slot_dtype)
        if drop:
            slots[::drop] = -1
        kc_ref, vc_ref = bits(p.k_cache).copy(), bits(p.v_cache).copy()
        kv_cache_oracle.store_kvcache_unified(bits(p.k), bits(p.v), kc_ref, vc_ref, slots.numpy())
        pd = to_dev(p)
        md = pd.metadata("static")
        md.num_splits = num_splits
        o = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md,
                                       store_slot_mapping=slots.cuda())
        torch.cuda.synchronize()
        assert np.array_equal(bits(pd.k_cache), kc_ref) and np.array_equal(bits(pd.v_cache), vc_ref)
        torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)
    assert ops.device_status()[0] == 0


# ---- error behaviour ---------------------------------------------------------------------------
def test_errors_are_raised_before_launch(dlx):
    p = attn_problem(ATTN_CASES["ragged_q"])
    pd = to_dev(p)
    md = pd.metadata("static")
    with pytest.raises(AssertionError):  # slot count mismatch, as in the reference (:118)
        dlx.store_kvcache_unified_layout(pd.k, pd.v, pd.k_cache, pd.v_cache, md.slot_mapping[:-1], md)
    with pytest.raises(ValueError):      # CPU tensors: no fallback
        dlx.store_kvcache_unified_layout(p.k, p.v, p.k_cache, p.v_cache, p.slot_mapping, None)
    with pytest.raises(ValueError):
        dlx.dllm_flash_attn_decode(pd.q.float(), pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    bad = SimpleNamespace(**vars(md))
    bad.decode_mode = "paged"
    with pytest.raises(ValueError):
        dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, bad)
    bad.attn_type = "causal"
    with pytest.raises(ValueError):
        dlx.dllm_flash_attn_prefill(pd.q, pd.k, pd.v, pd.scale, bad)
    # a clean call still works afterwards (no sticky error, context intact)
    o = run_decode(dlx, pd)
    torch.testing.assert_close(o.float().cpu(), oracle_out(p), atol=ATOL, rtol=RTOL)
