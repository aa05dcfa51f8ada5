"""Child process of tests/test_gpu_reference_kernels.py: the REFERENCE's attention layer
(diffulex/attention/attn_impl.py:14-72, from the copy made by baseline/make_ref.sh) constructed with this package's
shadow ``diffulex_kernel`` ahead of the reference on the path, run for one decode step and one prefill step and
checked against the CPU oracle.  Exits 0 on success."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(ROOT / "diffulex_b200" / "dropin"), str(ROOT), str(ROOT / "baseline" / "_ref")]

import torch  # noqa: E402

import diffulex_b200  # noqa: E402
from diffulex.attention import set_fetch_fn_for_attn_metadata  # noqa: E402
from diffulex.attention import attn_impl  # noqa: E402
from oracle import attn_oracle  # noqa: E402
from tests.golden.cases import ATTN_CASES, PREFILL_CASES, attn_problem, prefill_inputs  # noqa: E402

assert attn_impl.dllm_flash_attn_decode is diffulex_b200.dllm_flash_attn_decode
assert attn_impl.store_kvcache_unified_layout is diffulex_b200.store_kvcache_unified_layout
ATOL, RTOL = 2e-2, 1e-2

# ---- one decode step on benchmark configuration 1
p = attn_problem(ATTN_CASES["cfg1"])
g = p.geometry
pd = type(p)(**{f: (getattr(p, f).cuda() if isinstance(getattr(p, f), torch.Tensor) else getattr(p, f))
                for f in p.__dataclass_fields__})
md = pd.metadata("static")
set_fetch_fn_for_attn_metadata(lambda: md)
layer = attn_impl.Attention(g.num_q_heads, g.head_dim, p.scale, g.num_kv_heads)
layer.k_cache, layer.v_cache = pd.k_cache, pd.v_cache
flat = lambda t: t.reshape(t.shape[0], -1)
out = layer(flat(pd.q), flat(pd.k), flat(pd.v))
torch.cuda.synchronize()
want = attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                    p.cu_seqlens_q, p.cu_seqlens_k, p.scale, p.mask_mode, g.diffusion_block_size)
torch.testing.assert_close(out.view(p.q.shape).float().cpu(), want, atol=ATOL, rtol=RTOL)
slots = p.slot_mapping.long()
keep = slots >= 0
assert torch.equal(pd.k_cache.view(-1, g.num_kv_heads, g.head_dim)[slots[keep].cuda()].cpu(), p.k[keep])

# ---- one prefill step (block attention), no cache attached yet: the warm-up situation
case = PREFILL_CASES["ref_block_attn"]
q, k, v, cu_q, cu_k = prefill_inputs(case)
from types import SimpleNamespace  # noqa: E402
md2 = SimpleNamespace(is_prefill=True, attn_type="block_attention", cu_seqlens_q=cu_q.cuda(), cu_seqlens_k=cu_k.cuda(),
                      max_seqlen_q=max(case["q_lens"]), max_seqlen_k=max(case["kv_lens"]),
                      diffusion_block_size=case["dbs"], block_tables=None, slot_mapping=None,
                      kv_cache_layout="unified", need_kv_cache_store=True)
set_fetch_fn_for_attn_metadata(lambda: md2)
layer2 = attn_impl.Attention(case["hq"], case["hd"], case["hd"] ** -0.5, case["hkv"])
out2 = layer2(flat(q).cuda(), flat(k).cuda(), flat(v).cuda())
want2 = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, case["hd"] ** -0.5, True, case["dbs"])
torch.testing.assert_close(out2.view(q.shape).float().cpu(), want2, atol=ATOL, rtol=RTOL)
print("reference Attention.forward over the drop-in: decode and prefill agree with the oracle")
