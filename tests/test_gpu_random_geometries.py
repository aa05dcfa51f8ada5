"""Seeded random geometries against the CPU oracle: head counts, page sizes from 8 to 256 rows, diffusion blocks,
ragged contexts and in-flight lengths, both masks, both cu_seqlens conventions, every kernel, forced key-range splits;
every third case also as a prefill over the in-flight rows alone.  Tolerance: max-abs 2e-2 in bf16."""
import numpy as np
import pytest
import torch

from oracle import attn_oracle

pytestmark = pytest.mark.gpu


def draw(rng):
    from diffulex_b200.workload import MASK_BD_FULL, MASK_D2F_BLOCK_CAUSAL
    c = dict(hkv=int(rng.choice([1, 2, 4, 8])), G=int(rng.choice([1, 2, 4, 7, 8, 16])), hd=int(rng.choice([128, 128, 128, 64])),
             page=int(rng.choice([8, 16, 32, 64, 128, 256])), dbs=int(rng.choice([4, 8, 32, 64])),
             mask=int(rng.choice([MASK_BD_FULL, MASK_D2F_BLOCK_CAUSAL])), kernel=int(rng.choice([0, 0, 2, 3, 1])),
             splits=int(rng.choice([0, 0, 1, 2, 5])), mode=str(rng.choice(["static", "varlen"])))
    n = int(rng.integers(1, 7))
    if c["mask"] == MASK_D2F_BLOCK_CAUSAL:
        c["new"] = [int(c["dbs"] * rng.integers(1, 5)) for _ in range(n)]
        c["ctx"] = [int(c["dbs"] * rng.integers(0, 40)) for _ in range(n)]
    else:
        c["new"] = [int(rng.integers(1, c["dbs"] + 1)) for _ in range(n)]
        c["ctx"] = [int(rng.integers(0, 700)) for _ in range(n)]
    if c["hd"] != 128 and c["kernel"] in (2, 3):
        c["kernel"] = 0
    return c


@pytest.mark.parametrize("seed", range(4))
def test_random_geometries_match_the_oracle(seed, monkeypatch):
    import diffulex_b200 as dlx
    from diffulex_b200 import ops
    from diffulex_b200.workload import MASK_D2F_BLOCK_CAUSAL, make_problem, small_workload
    from types import SimpleNamespace
    rng = np.random.default_rng(seed)
    for i in range(12):
        c = draw(rng)
        w = small_workload("rnd", c["G"] * c["hkv"], c["hkv"], c["hd"], c["page"], c["dbs"], c["ctx"], c["new"], c["mask"],
                           100 * seed + i)
        p = make_problem(w, device="cpu", values="numpy", permute_pages=True)
        pd = type(p)(**{f: (getattr(p, f).cuda() if isinstance(getattr(p, f), torch.Tensor) else getattr(p, f))
                        for f in p.__dataclass_fields__})
        monkeypatch.setattr(ops, "DECODE_KERNEL", c["kernel"])
        md = pd.metadata(c["mode"])
        md.num_splits = c["splits"]
        o = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
        varlen = c["mode"] == "varlen"
        want = attn_oracle.decode_attention(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                            p.cu_seqlens_q, p.cu_seqlens_k_total if varlen else p.cu_seqlens_k, p.scale,
                                            p.mask_mode, c["dbs"], kv_offsets_from_q=varlen)
        err = (o.float().cpu() - want).abs().max().item()
        assert err < 2e-2, (err, c)
        if i % 3 == 0:
            monkeypatch.setattr(ops, "DECODE_KERNEL", 0 if c["kernel"] == 3 else c["kernel"])
            block = c["mask"] == MASK_D2F_BLOCK_CAUSAL
            md2 = SimpleNamespace(is_prefill=True, attn_type="block_attention" if block else "full_attention",
                                  cu_seqlens_q=pd.cu_seqlens_q, cu_seqlens_k=pd.cu_seqlens_q, max_seqlen_q=max(c["new"]),
                                  max_seqlen_k=max(c["new"]), diffusion_block_size=c["dbs"])
            o2 = dlx.dllm_flash_attn_prefill(pd.q, pd.k, pd.v, pd.scale, md2)
            want2 = attn_oracle.prefill_attention(p.q, p.k, p.v, p.cu_seqlens_q, p.cu_seqlens_q, p.scale, block, c["dbs"])
            err2 = (o2.float().cpu() - want2).abs().max().item()
            assert err2 < 2e-2, (err2, c)
    assert ops.device_status()[0] == 0
