"""GPU parity of prefill attention (no cache; full and block-causal masks): the CUDA path through the
reference-shaped entry point against the golden vectors of the reference's own prefill check and against the
CPU oracle, on the geometries of the reference's prefill-kernel tests
(tests/python/kernel/test_dllm_flash_attn_prefill_kernel.py:162-310) and on ragged prompts.

Tolerance: max-abs 2e-2 / rel 1e-2 in bf16, as for decode (the reference's own tests use 1e-2 / 1e-2, :157)."""
import json
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import attn_oracle
from tests.golden.cases import PREFILL_CASES, prefill_fixture_index, prefill_inputs

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2
KERNELS = {"auto": 0, "mma": 1, "tc5": 2}


def metadata(case, cu_q, cu_k):
    """What the reference's runner hands to the attention layer for a prefill step
    (diffulex/strategy/block_diffusion/engine/model_runner.py:45-112), as far as the entry point reads it."""
    return SimpleNamespace(is_prefill=True, attn_type="block_attention" if case["block"] else "full_attention",
                           cu_seqlens_q=cu_q, cu_seqlens_k=cu_k, max_seqlen_q=max(case["q_lens"]),
                           max_seqlen_k=max(case["kv_lens"]), diffusion_block_size=case["dbs"],
                           num_seqs=len(case["q_lens"]), block_tables=None)


@pytest.mark.parametrize("kernel", list(KERNELS))
@pytest.mark.parametrize("name", list(PREFILL_CASES))
def test_prefill_matches_reference_vectors_and_oracle(name, kernel, golden_dir, monkeypatch):
    import diffulex_b200 as dlx
    from diffulex_b200 import ops
    case = PREFILL_CASES[name]
    if kernel == "tc5" and case["hd"] != 128:
        pytest.skip("the tcgen05 kernels serve head_dim 128")
    monkeypatch.setattr(ops, "DECODE_KERNEL", KERNELS[kernel])
    q, k, v, cu_q, cu_k = prefill_inputs(case)
    md = metadata(case, cu_q.cuda(), cu_k.cuda())
    md.check_status = True
    o = dlx.dllm_flash_attn_prefill(q.cuda(), k.cuda(), v.cuda(), case["hd"] ** -0.5, md)
    torch.cuda.synchronize()
    assert ops.device_status()[0] == 0
    assert o.dtype == torch.bfloat16 and o.shape == q.shape
    o = o.float().cpu()
    rows, heads = prefill_fixture_index(case)
    golden = torch.from_numpy(np.load(golden_dir / "prefill_golden.npz")[name])
    torch.testing.assert_close(o[rows][:, heads], golden, atol=ATOL, rtol=RTOL)
    want = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, case["hd"] ** -0.5, case["block"], case["dbs"])
    torch.testing.assert_close(o, want, atol=ATOL, rtol=RTOL)


def test_prefill_honours_scale_and_out_argument():
    """``scale`` is an argument here (the reference kernel fixes head_dim ** -0.5); ``out=`` writes in place."""
    import diffulex_b200 as dlx
    case = PREFILL_CASES["ragged_block_gqa7"]
    q, k, v, cu_q, cu_k = prefill_inputs(case)
    md = metadata(case, cu_q.cuda(), cu_k.cuda())
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device="cuda")
    ret = dlx.dllm_flash_attn_prefill(q.cuda(), k.cuda(), v.cuda(), 0.05, md, out=out)
    assert ret is out
    want = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, 0.05, True, case["dbs"])
    torch.testing.assert_close(out.float().cpu(), want, atol=ATOL, rtol=RTOL)


def test_prefill_with_fewer_keys_than_queries_and_more():
    """cu_seqlens_k need not equal cu_seqlens_q: keys past a short key range do not exist, extra keys are seen
    under the full mask and follow the block rule under the block mask (dllm_flash_attn.py:101-116)."""
    import diffulex_b200 as dlx
    for block in (False, True):
        case = dict(hq=8, hkv=2, hd=128, q_lens=[64, 40], kv_lens=[32, 150], block=block, dbs=32, seed=90)
        q, k, v, cu_q, cu_k = prefill_inputs(case)
        md = metadata(case, cu_q.cuda(), cu_k.cuda())
        o = dlx.dllm_flash_attn_prefill(q.cuda(), k.cuda(), v.cuda(), case["hd"] ** -0.5, md)
        want = attn_oracle.prefill_attention(q, k, v, cu_q, cu_k, case["hd"] ** -0.5, block, case["dbs"])
        torch.testing.assert_close(o.float().cpu(), want, atol=ATOL, rtol=RTOL)


def test_prefill_rejects_unknown_attn_type():
    import diffulex_b200 as dlx
    case = PREFILL_CASES["ref_single_seq"]
    q, k, v, cu_q, cu_k = prefill_inputs(case)
    md = metadata(case, cu_q.cuda(), cu_k.cuda())
    md.attn_type = "sliding_window"
    with pytest.raises(ValueError):
        dlx.dllm_flash_attn_prefill(q.cuda(), k.cuda(), v.cuda(), 0.1, md)
