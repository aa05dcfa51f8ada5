"""CPU-only checks: the C-ABI library builds, loads and exports every symbol the header declares;
argument validation and split planning (host code, no launch); the Python mirror's error
behaviour; the data-parallel partition and gather (gloo, world_size 2)."""
import ctypes
import os
import re
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    from diffulex_b200 import _lib
    from diffulex_b200.build import build
    build()
    return _lib.lib()


def good_params(**over):
    from diffulex_b200._lib import DecodeAttnParams
    p = DecodeAttnParams()
    p.struct_bytes = ctypes.sizeof(DecodeAttnParams)
    p.total_q, p.num_seqs, p.max_blocks, p.num_pages = 2048, 64, 9, 600
    p.q_row_stride = p.out_row_stride = 28 * 128
    p.k_row_stride = p.v_row_stride = p.cache_token_stride = 4 * 128
    p.cache_page_stride = 256 * 4 * 128
    p.num_q_heads, p.num_kv_heads, p.head_dim, p.page_size = 28, 4, 128, 256
    p.max_q_len, p.max_kv_len, p.mask_mode, p.diffusion_block_size = 32, 0, 0, 32
    p.scale = 128 ** -0.5
    for k, v in over.items():
        setattr(p, k, v)
    return p


def test_header_symbols_are_exported(lib):
    header = (ROOT / "include" / "dlx_b200.h").read_text()
    declared = set(re.findall(r"\b(dlx_[a-z0-9_]+)\s*\(", header))
    assert {"dlx_store_kvcache_unified", "dlx_load_kvcache", "dlx_decode_attn"} <= declared
    from diffulex_b200._lib import EXPORTED_SYMBOLS
    assert declared == set(EXPORTED_SYMBOLS), "ctypes binding and header disagree"
    for name in declared:
        assert getattr(lib, name) is not None
    assert lib.dlx_version() >= 100
    assert lib.dlx_status_string(0) == b"ok"


def test_decode_validation_statuses(lib):
    from diffulex_b200._lib import DecodeAttnParams
    ws = lambda p: lib.dlx_decode_attn_workspace_bytes(ctypes.byref(p))
    assert ws(good_params()) >= 0
    assert ws(good_params(struct_bytes=8)) == -1
    assert b"struct_bytes" in lib.dlx_last_error()
    assert ws(good_params(head_dim=96)) == -2
    assert ws(good_params(num_kv_heads=5)) == -1
    assert ws(good_params(mask_mode=7)) == -1
    assert ws(good_params(mask_mode=1, diffusion_block_size=0)) == -1
    assert ws(good_params(scale=0.0)) == -1
    assert ws(good_params(dtype=1)) == -2
    # null data pointers are refused before anything is launched
    assert lib.dlx_decode_attn(ctypes.byref(good_params()), None) == 1
    assert lib.dlx_decode_attn(None, None) == 1
    # an empty batch is a no-op
    assert lib.dlx_decode_attn(ctypes.byref(good_params(num_seqs=0, total_q=0)), None) == 0


def test_store_and_load_validation_statuses(lib):
    assert lib.dlx_store_kvcache_unified(None, 512, None, 512, None, None, None, 0, 0, 512, 2, 10, None) == 0
    assert lib.dlx_store_kvcache_unified(None, 512, None, 512, None, None, None, 0, 4, 512, 2, 10, None) == 1
    assert lib.dlx_store_kvcache_unified(None, 512, None, 512, None, None, None, 0, -1, 512, 2, 10, None) == 1
    buf = ctypes.create_string_buffer(64)
    a = ctypes.addressof(buf)
    # row stride smaller than a row
    assert lib.dlx_store_kvcache_unified(a, 256, a, 512, a, a, a, 0, 4, 512, 2, 10, None) == 1
    assert lib.dlx_load_kvcache(None, None, 0, 0, None, 0, None, 0, None, 0, 0, None, None, None, None, None, None,
                                0, 0, 256, 0, 512, 2, None) == 0
    assert lib.dlx_load_kvcache(None, None, 0, 0, None, 0, None, 0, None, 0, 1, None, None, None, None, None, None,
                                10, 2, 256, 4, 512, 2, None) == 1
    assert lib.dlx_store_kvcache_distinct(a, 512, a, 512, a, a, a, 0, 4, 4, 128, 256, 7, 4, 2, None) == 1


def test_split_planning_is_host_only_and_sized_right(lib):
    n = lambda p: lib.dlx_decode_attn_num_splits(ctypes.byref(p))
    ws = lambda p: lib.dlx_decode_attn_workspace_bytes(ctypes.byref(p))
    sb = lambda p: lib.dlx_decode_attn_schedule_bytes(ctypes.byref(p))
    # 64 seqs x 4 KV heads = 256 items of 224 rows (two row blocks on two CTAs) on 74 schedule bins, contexts <= 2336
    # keys: one pass; the only scratch is the schedule (1 KiB of offsets + one 128-byte record per item) when the
    # call plans itself
    p = good_params()
    assert n(p) == 1 and sb(p) == 1024 + 256 * 128 and ws(p) == sb(p)
    # both tcgen05 kernels (two neighbouring CTAs / one CTA pair per item) take the same schedule
    assert sb(good_params(kernel=2)) == sb(p) and sb(good_params(kernel=3)) == sb(p)
    # a query block of at most 128 packed rows is one item on one CTA
    assert sb(good_params(max_q_len=16, total_q=1024)) == 1024 + 256 * 128
    # the mma.sync kernel takes no schedule
    assert sb(good_params(kernel=1)) == 0 and ws(good_params(kernel=1)) == 0
    # forced splits: lse [splits, rows] (256-byte padded) + partial O [splits, rows, hd] fp32 + schedule
    p = good_params(num_splits=3)
    rows = 2048 * 28
    assert sb(p) == 1024 + 3 * 256 * 128
    assert n(p) == 3 and ws(p) == ((3 * rows * 4 + 255) // 256) * 256 + 3 * rows * 128 * 4 + sb(p)
    # preparing a schedule needs the metadata pointers and a buffer of that size
    assert lib.dlx_decode_attn_prepare(ctypes.byref(p), None, 0, None) == 1
    # few sequences: split to fill 148 SMs
    p = good_params(num_seqs=2, total_q=64)
    assert n(p) > 1
    # long contexts: the persistent tcgen05 kernel balances a long item list by itself (no split) ...
    p = good_params(num_seqs=256, total_q=8192, max_blocks=129)
    assert n(p) == 1
    # ... but cuts long contexts while there are fewer than 1.6 items per schedule bin (here 96 and 116 on 74)
    p = good_params(num_seqs=24, total_q=768, max_blocks=129)
    assert n(p) >= 3
    assert n(good_params(num_seqs=29, total_q=928, max_blocks=129)) >= 3
    assert n(good_params(num_seqs=30, total_q=960, max_blocks=129)) == 1
    # the mma.sync kernel launches one CTA per item and keeps cutting long contexts
    p = good_params(num_seqs=256, total_q=8192, max_blocks=129, kernel=1)
    assert n(p) >= 3


def test_python_mirror_rejects_bad_inputs_without_a_gpu(lib):
    import diffulex_b200 as dlx
    from diffulex_b200.workload import make_problem, small_workload
    p = make_problem(small_workload("t", 8, 2, 64, 16, 4, [10, 3], [4, 4]), device="cpu")
    md = p.metadata("static")
    with pytest.raises(AssertionError):
        dlx.store_kvcache_unified_layout(p.k, p.v, p.k_cache, p.v_cache, p.slot_mapping[:-1], md)
    with pytest.raises(AssertionError):
        dlx.store_kvcache_unified_layout(p.k.transpose(1, 2), p.v, p.k_cache, p.v_cache, p.slot_mapping, md)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        dlx.store_kvcache_unified_layout(p.k, p.v, p.k_cache, p.v_cache, p.slot_mapping, md)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md)
    md.decode_mode = "other"
    with pytest.raises(ValueError):
        dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        dlx.dllm_flash_attn_prefill(p.q, p.k, p.v, p.scale, md)
    md.attn_type = "other"
    with pytest.raises(ValueError, match="attn_type"):
        dlx.dllm_flash_attn_prefill(p.q, p.k, p.v, p.scale, md)


def test_missing_library_is_an_import_error(tmp_path, monkeypatch):
    from diffulex_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libdlx_b200.so")
    with pytest.raises(ImportError, match="no CPU or PyTorch fallback"):
        _lib.lib()


def test_dropin_package_exposes_reference_names(lib, monkeypatch):
    import importlib
    import sys
    monkeypatch.syspath_prepend(str(ROOT / "diffulex_b200" / "dropin"))
    for m in [k for k in sys.modules if k.startswith("diffulex_kernel")]:
        monkeypatch.delitem(sys.modules, m)
    mod = importlib.import_module("diffulex_kernel")
    for name in ("store_kvcache_distinct_layout", "store_kvcache_unified_layout", "dllm_flash_attn_decode",
                 "dllm_flash_attn_prefill"):
        assert callable(getattr(mod, name))
    sub = importlib.import_module("diffulex_kernel.python.kv_cache_kernels")
    assert callable(sub.load_kvcache)


REFERENCE = ROOT / "baseline" / "_ref"   # unmodified copy of the reference's kernel package (baseline/make_ref.sh)
needs_reference = pytest.mark.skipif(not (REFERENCE / "diffulex_kernel").is_dir(),
                                     reason="no copy of the reference beside the repository (baseline/make_ref.sh)")


def _reference_signature(path: Path, name: str):
    """Parameter names of a top-level function of a reference source file, read as text (no import: the file
    pulls in its JIT compilers at import time)."""
    import ast
    for node in ast.parse(path.read_text()).body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            return [a.arg for a in node.args.args]
    raise AssertionError(f"{name} not found in {path}")


@needs_reference
@pytest.mark.parametrize("module, name", [
    ("kv_cache_kernels", "store_kvcache_unified_layout"), ("kv_cache_kernels", "store_kvcache_distinct_layout"),
    ("kv_cache_kernels", "load_kvcache"), ("dllm_flash_attn", "dllm_flash_attn_decode"),
    ("dllm_flash_attn", "dllm_flash_attn_prefill")])
def test_entry_points_keep_the_reference_signatures(lib, module, name):
    """Same positional parameters, same names, same order as the reference's functions; anything this
    package adds is a keyword with a default."""
    import inspect
    import diffulex_b200 as dlx
    want = _reference_signature(REFERENCE / "diffulex_kernel" / "python" / f"{module}.py", name)
    params = list(inspect.signature(getattr(dlx, name)).parameters.values())
    assert [p.name for p in params[:len(want)]] == want
    assert all(p.default is not inspect.Parameter.empty for p in params[len(want):])


@needs_reference
def test_reference_attention_layer_binds_the_dropin(lib):
    """With the shadow package ahead of the reference checkout on the path, the reference's own attention layer
    (diffulex/attention/attn_impl.py:5-10) imports these operators.  Run in a child process: it changes what
    ``diffulex_kernel`` means."""
    import os
    import subprocess
    import sys
    code = ("import diffulex.attention.attn_impl as m, diffulex_b200 as d;"
            "assert m.dllm_flash_attn_decode is d.dllm_flash_attn_decode;"
            "assert m.dllm_flash_attn_prefill is d.dllm_flash_attn_prefill;"
            "assert m.store_kvcache_unified_layout is d.store_kvcache_unified_layout;"
            "assert m.store_kvcache_distinct_layout is d.store_kvcache_distinct_layout;"
            "import diffulex_kernel.python.kv_cache_kernels as k; assert k.load_kvcache is d.load_kvcache")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT / "diffulex_b200" / "dropin"), str(ROOT), str(REFERENCE)]))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]


# ---- workloads and partition ---------------------------------------------------------------------
def test_named_workloads_match_the_benchmark_configurations():
    from diffulex_b200.workload import named_workload
    w = named_workload("cfg2")
    assert len(w.context_lens) == 64 and w.context_lens.min() >= 512 and w.context_lens.max() <= 2048
    assert (w.geometry.num_q_heads, w.geometry.num_kv_heads, w.geometry.head_dim, w.geometry.layers) == (28, 4, 128, 28)
    w = named_workload("cfg3")
    assert (w.new_lens == 128).all() and w.mask_mode == 1 and w.geometry.num_kv_heads == 32
    w = named_workload("cfg4")
    assert w.context_lens.min() >= 128 and w.context_lens.max() <= 8192 and (w.new_lens == 4).all()
    w = named_workload("cfg5")
    assert len(w.context_lens) == 256 and w.context_lens.min() >= 4096 and w.context_lens.max() <= 32768
    assert np.array_equal(named_workload("cfg5").context_lens, w.context_lens), "seeded"


def test_lpt_partition_is_exact_and_balanced():
    from diffulex_b200.workload import named_workload, partition_lpt, shard_workload
    w = named_workload("cfg5")
    costs = (w.context_lens + w.new_lens).tolist()
    for ws in (2, 4, 8):
        parts = partition_lpt(costs, ws)
        assert sorted(sum(parts, [])) == list(range(len(costs)))
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) / (sum(loads) / ws) < 1.01
        sub, owned = shard_workload(w, 1, ws)
        assert owned == parts[1] and np.array_equal(sub.context_lens, w.context_lens[owned])


def test_page_tables_are_disjoint_permuted_and_padded():
    from diffulex_b200.workload import make_problem, named_workload
    p = make_problem(named_workload("cfg1"), device="cpu")
    bt = p.block_tables.numpy()
    used = bt[bt >= 0]
    assert len(set(used.tolist())) == len(used) and (bt == -1).any()
    assert used.max() < p.k_cache.shape[0]
    assert not np.array_equal(np.sort(used), used), "physical pages are not handed out in order"
    # slots of the in-flight rows land in the right page at the right offset
    s, pos = 2, int(p.host_context_lens[2]) + 5
    slot = int(p.slot_mapping[int(p.cu_seqlens_q[2]) + 5])
    assert slot == bt[s, pos // 256] * 256 + pos % 256


# ---- data-parallel gather over gloo ----------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, world_size, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        from diffulex_b200 import dp
        from diffulex_b200.workload import partition_lpt
        q_lens = [3, 5, 2, 7, 1, 4]
        costs = [100, 900, 50, 700, 20, 300]
        parts = partition_lpt(costs, world_size)
        cu = np.concatenate([[0], np.cumsum(q_lens)])
        # a rank's "attention output": row value = global query row index
        rows = np.concatenate([np.arange(cu[s], cu[s + 1]) for s in parts[rank]])
        local = torch.from_numpy(rows).float().view(-1, 1, 1).expand(-1, 2, 3).contiguous()
        full = dp.gather_outputs(local, parts, q_lens)
        ok = torch.equal(full[:, 0, 0], torch.arange(int(cu[-1])).float()) and full.shape == (int(cu[-1]), 2, 3)
        t = dp.max_over_ranks(1.0 + rank)
        ts = dp.gather_timings(1.0 + rank)
        tot = dp.sum_over_ranks(10.0)
        q.put((rank, bool(ok), t, ts, tot))
    finally:
        dist.destroy_process_group()


def test_dp_gather_world_size_2_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, t, ts, tot in results:
        assert ok and t == 2.0 and ts == [1.0, 2.0] and tot == 20.0


# ---- a rank that leaves between steps -------------------------------------------------------------
def _leaving_worker(rank, world_size, port, q):
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world_size, timeout=datetime.timedelta(seconds=8))
    from diffulex_b200 import dp
    q_lens, parts = [2, 3], [[0], [1]]
    local = torch.full((q_lens[rank], 1, 4), float(rank))
    full = dp.gather_outputs(local, parts, q_lens)            # step 1: both ranks are there
    first_ok = full.shape[0] == 5 and float(full[:, 0, 0].sum()) == 3.0
    if rank == 1:
        q.put((rank, first_ok, "left"))
        q.close(); q.join_thread()
        os._exit(0)                                           # leaves between steps, nothing in flight
    time.sleep(1.0)
    t0 = time.time()
    try:
        dp.gather_outputs(local, parts, q_lens)               # step 2: the peer is gone
        outcome = "no error"
    except Exception as e:   # the process group reports the missing rank (closed connection or timeout)
        outcome = type(e).__name__
    q.put((rank, first_ok, outcome, time.time() - t0))
    q.close(); q.join_thread()
    os._exit(0)   # the group cannot be torn down cleanly without its peer


def test_gather_reports_a_rank_that_left_instead_of_hanging():
    """Failure detection on the host: a data-parallel rank exits between two steps; the survivor's next output
    gather raises within the process group's (short) timeout instead of waiting forever."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        item = q.get(timeout=90)
        got[item[0]] = item
    for p in procs:
        p.join(timeout=30)
    assert got[1][1] and got[1][2] == "left"
    assert got[0][1], "the first gather (both ranks present) must work"
    assert got[0][2] != "no error", "the second gather must fail once the peer is gone"
    assert got[0][3] < 60.0
