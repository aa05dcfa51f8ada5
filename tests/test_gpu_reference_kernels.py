"""The reference's OWN GPU kernels next to this package's, on the same seeded inputs, on the same GPU:
Triton store / load (diffulex_kernel/python/kv_cache_kernels.py:11-32, 36-83, 127-227), the TileLang decode kernel
(dllm_flash_attn.py:163-347 through the wrapper :599-631) and the load + dense varlen attention pair (:632-637).
They are imported, unmodified, from the copy baseline/make_ref.sh makes (git-ignored); without that copy the
tests skip.  Store / load: bit-exact.  Attention: max-abs 2e-2 / rel 1e-2 in bf16 between the two kernels."""
import importlib
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import kv_cache_oracle
from tests.golden.cases import (ATTN_CASES, LOAD_CASES, STORE_CASES, attn_problem, bits, distinct_caches, load_problem,
                                store_inputs)

ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref"
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not (REF / "diffulex_kernel").is_dir(), reason="baseline/_ref not made (baseline/make_ref.sh)")]

ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def ref():
    """The reference's kernel modules.  The path entry and the imported modules are removed again afterwards, so that
    other tests' ``diffulex_kernel`` (this package's shadow) is not affected."""
    sys.path.insert(0, str(REF))
    stale = [m for m in sys.modules if m == "diffulex_kernel" or m.startswith(("diffulex_kernel.", "diffulex."))]
    for m in stale:
        del sys.modules[m]
    try:
        kv = importlib.import_module("diffulex_kernel.python.kv_cache_kernels")
        fa = importlib.import_module("diffulex_kernel.python.dllm_flash_attn")
        assert str(REF) in kv.__file__ and str(REF) in fa.__file__
        yield kv, fa
    finally:
        sys.path.remove(str(REF))
        for m in [m for m in sys.modules if m == "diffulex_kernel" or m.startswith(("diffulex_kernel.", "diffulex."))]:
            del sys.modules[m]


def to_dev(p):
    return type(p)(**{f: (getattr(p, f).cuda() if isinstance(getattr(p, f), torch.Tensor) else getattr(p, f))
                      for f in p.__dataclass_fields__})


def dev_rows(t):
    """A device copy that keeps a strided row layout."""
    if t.is_contiguous():
        return t.cuda()
    n, h, d = t.shape
    wide = torch.zeros(n, t.stride(0), dtype=t.dtype, device="cuda")
    wide[:, : h * d] = t.reshape(n, -1).cuda()
    return wide[:, : h * d].view(n, h, d)


@pytest.mark.parametrize("name", list(STORE_CASES))
def test_store_equals_the_reference_triton_kernels(name, ref):
    import diffulex_b200 as dlx
    kv, _ = ref
    key, value, k_cache, v_cache, slots = store_inputs(STORE_CASES[name])
    kd, vd, sd = dev_rows(key), dev_rows(value), slots.cuda()
    a_k, a_v, b_k, b_v = k_cache.cuda(), v_cache.cuda(), k_cache.cuda(), v_cache.cuda()
    kv.store_kvcache_unified_layout(kd, vd, a_k, a_v, sd, None)
    dlx.store_kvcache_unified_layout(kd, vd, b_k, b_v, sd, None)
    torch.cuda.synchronize()
    assert torch.equal(a_k.view(torch.int16), b_k.view(torch.int16)) and torch.equal(a_v.view(torch.int16), b_v.view(torch.int16))
    kc, vc = distinct_caches(STORE_CASES[name])
    a_k, a_v, b_k, b_v = kc.cuda(), vc.cuda(), kc.cuda(), vc.cuda()
    kv.store_kvcache_distinct_layout(kd, vd, a_k, a_v, sd, None)
    dlx.store_kvcache_distinct_layout(kd, vd, b_k, b_v, sd, None)
    torch.cuda.synchronize()
    assert torch.equal(a_k.view(torch.int16), b_k.view(torch.int16)) and torch.equal(a_v.view(torch.int16), b_v.view(torch.int16))


@pytest.mark.parametrize("name", list(LOAD_CASES))
def test_load_equals_the_reference_triton_kernel_on_the_rows_it_writes(name, ref):
    import diffulex_b200 as dlx
    kv, _ = ref
    p = load_problem(LOAD_CASES[name])
    pd = to_dev(p)
    md = pd.metadata("varlen")
    rk, rv = kv.load_kvcache(pd.k_cache, pd.v_cache, md, pd.k, pd.v)
    mk, mv = dlx.load_kvcache(pd.k_cache, pd.v_cache, md, pd.k, pd.v)
    torch.cuda.synchronize()
    written = kv_cache_oracle.reference_written_rows(
        p.geometry.page_size, p.block_tables.numpy(), p.context_lens.numpy(), p.seq_lens_ts.numpy(),
        p.cu_seqlens_k_total.numpy(), p.geometry.diffusion_block_size)
    assert rk.shape == mk.shape
    assert np.array_equal(bits(rk)[written], bits(mk)[written]) and np.array_equal(bits(rv)[written], bits(mv)[written])


# benchmark configuration 1 and the geometries of the reference's own decode-kernel tests
STATIC_CASES = ["cfg1"] + [n for n in ATTN_CASES if n.startswith("ref_")]


@pytest.mark.parametrize("name", STATIC_CASES)
def test_static_decode_agrees_with_the_reference_tilelang_kernel(name, ref, monkeypatch):
    import diffulex_b200 as dlx
    _, fa = ref
    # the tile configuration the reference's autotuner would leave behind after a prefill warm-up
    # (dllm_flash_attn.py:20, 555-572); its kernels' defaults (:174-177)
    monkeypatch.setattr(fa, "kernel_config", dict(BLOCK_M=64, BLOCK_N=64, NUM_STAGES=1, NUM_THREADS=128))
    p = attn_problem(ATTN_CASES[name])
    pd = to_dev(p)
    md = pd.metadata("static")
    theirs = fa.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    mine = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    torch.cuda.synchronize()
    torch.testing.assert_close(mine.float(), theirs.float(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("name", ["cfg1", "ragged_q", "ragged_permuted", "q4_gqa4"])
def test_varlen_decode_agrees_with_the_reference_gather_and_dense_attention(name, ref):
    """Sequences whose gathered K / V the reference leaves partly unwritten (a page-aligned context, a ragged tail:
    see kv_cache_oracle.reference_written_rows) attend over uninitialised rows there; they are left out."""
    import diffulex_b200 as dlx
    _, fa = ref
    p = attn_problem(ATTN_CASES[name])
    pd = to_dev(p)
    md = pd.metadata("varlen")
    theirs = fa.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    mine = dlx.dllm_flash_attn_decode(pd.q, pd.k, pd.v, pd.k_cache, pd.v_cache, pd.scale, md)
    torch.cuda.synchronize()
    written = kv_cache_oracle.reference_written_rows(
        p.geometry.page_size, p.block_tables.numpy(), p.context_lens.numpy(), p.seq_lens_ts.numpy(),
        p.cu_seqlens_k_total.numpy(), p.geometry.diffusion_block_size)
    cu_q, cu_k = p.cu_seqlens_q.tolist(), p.cu_seqlens_k_total.tolist()
    compared = 0
    for s in range(p.num_seqs):
        if written[cu_k[s]:cu_k[s + 1]].all():
            torch.testing.assert_close(mine[cu_q[s]:cu_q[s + 1]].float(), theirs[cu_q[s]:cu_q[s + 1]].float(),
                                       atol=ATOL, rtol=RTOL)
            compared += 1
    assert compared > 0


def test_reference_attention_layer_runs_over_the_dropin():
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "_reference_layer_child.py")], capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
