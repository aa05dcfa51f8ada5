"""The attention layer over the three operators (host-side mirror of diffulex/attention/attn_impl.py:42-72):
one decode step and one prefill step through ``Attention.forward`` against the CPU oracle: caches bit-exact,
outputs within the attention tolerance (max-abs 2e-2 / rel 1e-2 in bf16)."""
import numpy as np
import pytest
import torch

from oracle import attn_oracle, kv_cache_oracle
from tests.golden.cases import ATTN_CASES, PREFILL_CASES, attn_problem, bits, prefill_inputs

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def to_dev(p):
    return type(p)(**{f: (getattr(p, f).cuda() if isinstance(getattr(p, f), torch.Tensor) else getattr(p, f))
                      for f in p.__dataclass_fields__})


def layer_for(g, md, k_cache=None, v_cache=None):
    from diffulex_b200.attention import Attention
    layer = Attention(g.num_q_heads, g.head_dim, g.head_dim ** -0.5, g.num_kv_heads, lambda: md)
    if k_cache is not None:
        layer.k_cache, layer.v_cache = k_cache, v_cache
    return layer


@pytest.mark.parametrize("name", ["cfg1", "ragged_q", "ragged_permuted"])
def test_decode_step_stores_then_attends(name):
    p = attn_problem(ATTN_CASES[name])
    g = p.geometry
    pd = to_dev(p)
    md = pd.metadata("static")
    layer = layer_for(g, md, pd.k_cache, pd.v_cache)
    flat = lambda t: t.reshape(t.shape[0], -1)
    out = layer(flat(pd.q), flat(pd.k), flat(pd.v))
    torch.cuda.synchronize()
    assert out.shape == (p.q.shape[0], g.num_q_heads * g.head_dim) and out.is_contiguous()
    kc, vc = bits(p.k_cache).copy(), bits(p.v_cache).copy()
    kv_cache_oracle.store_kvcache_unified(bits(p.k), bits(p.v), kc, vc, p.slot_mapping.numpy())
    assert np.array_equal(bits(pd.k_cache), kc) and np.array_equal(bits(pd.v_cache), vc)
    want = attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                        p.cu_seqlens_q, p.cu_seqlens_k, p.scale, p.mask_mode, g.diffusion_block_size)
    torch.testing.assert_close(out.view(p.q.shape).float().cpu(), want, atol=ATOL, rtol=RTOL)


def test_decode_step_replays_from_a_cuda_graph():
    """Store + decode of one layer call captured once and replayed after the inputs were refilled in place."""
    p = attn_problem(ATTN_CASES["cfg1"])
    g = p.geometry
    pd = to_dev(p)
    md = pd.metadata("static")
    layer = layer_for(g, md, pd.k_cache, pd.v_cache)
    flat = lambda t: t.reshape(t.shape[0], -1)
    q2, k2, v2 = flat(pd.q).clone(), flat(pd.k).clone(), flat(pd.v).clone()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        layer(q2, k2, v2)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = layer(q2, k2, v2)
    q_new = torch.randn_like(q2)
    q2.copy_(q_new)
    graph.replay()
    torch.cuda.synchronize()
    want = attn_oracle.decode_attention(q_new.view(p.q.shape).cpu(), p.k, p.v, p.k_cache, p.v_cache, p.block_tables,
                                        p.context_lens, p.cu_seqlens_q, p.cu_seqlens_k, p.scale, p.mask_mode,
                                        g.diffusion_block_size)
    torch.testing.assert_close(out.view(p.q.shape).float().cpu(), want, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["ref_block_attn", "ragged_block_gqa7", "ragged_full_mha"])
def test_prefill_step_stores_the_prompt_then_attends(name):
    from types import SimpleNamespace
    case = PREFILL_CASES[name]
    q, k, v, cu_q, cu_k = prefill_inputs(case)
    total, page = k.shape[0], 32
    pages = (total + page - 1) // page + 3
    rng = np.random.default_rng(5)
    slots = torch.from_numpy(rng.permutation(pages * page)[:total].astype(np.int32))
    k_cache = torch.zeros(pages, page, case["hkv"], case["hd"], dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    md = SimpleNamespace(is_prefill=True, attn_type="block_attention" if case["block"] else "full_attention",
                         cu_seqlens_q=cu_q.cuda(), cu_seqlens_k=cu_k.cuda(), max_seqlen_q=max(case["q_lens"]),
                         max_seqlen_k=max(case["kv_lens"]), diffusion_block_size=case["dbs"], block_tables=None,
                         slot_mapping=slots.cuda(), kv_cache_layout="unified", need_kv_cache_store=True)
    g = SimpleNamespace(num_q_heads=case["hq"], num_kv_heads=case["hkv"], head_dim=case["hd"])
    kcd, vcd = k_cache.cuda(), v_cache.cuda()
    layer = layer_for(g, md, kcd, vcd)
    flat = lambda t: t.reshape(t.shape[0], -1).cuda()
    out = layer(flat(q), flat(k), flat(v))
    torch.cuda.synchronize()
    kc, vc = bits(k_cache).copy(), bits(v_cache).copy()
    kv_cache_oracle.store_kvcache_unified(bits(k), bits(v), kc, vc, slots.numpy())
    assert np.array_equal(bits(kcd), kc) and np.array_equal(bits(vcd), vc)
    want = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, case["hd"] ** -0.5, case["block"], case["dbs"])
    torch.testing.assert_close(out.view(q.shape).float().cpu(), want, atol=ATOL, rtol=RTOL)


def test_layer_without_a_cache_skips_the_store():
    """Warm-up passes run before the cache pool exists (attn_impl.py:53): nothing is stored, prefill still runs."""
    from types import SimpleNamespace
    case = PREFILL_CASES["ref_single_seq"]
    q, k, v, cu_q, cu_k = prefill_inputs(case)
    md = SimpleNamespace(is_prefill=True, attn_type="full_attention", cu_seqlens_q=cu_q.cuda(), cu_seqlens_k=cu_k.cuda(),
                         max_seqlen_q=192, max_seqlen_k=192, diffusion_block_size=32, block_tables=None,
                         slot_mapping=None, kv_cache_layout="unified", need_kv_cache_store=True)
    g = SimpleNamespace(num_q_heads=case["hq"], num_kv_heads=case["hkv"], head_dim=case["hd"])
    out = layer_for(g, md)(q.reshape(192, -1).cuda(), k.reshape(192, -1).cuda(), v.reshape(192, -1).cuda())
    want = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, case["hd"] ** -0.5, False, 32)
    torch.testing.assert_close(out.view(q.shape).float().cpu(), want, atol=ATOL, rtol=RTOL)
