#!/usr/bin/env python
"""Benchmark of the decode hot path: per layer, slot-mapped KV store of the in-flight block and
paged block-diffusion decode attention, over all layers of the model shape.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N ... bench.py --gpus N ...

One JSON line on rank 0.  ``value`` is the attention's algorithmic KV-read rate, summed over ranks:
(valid cached + in-flight tokens) x 2 x Hkv x hd x 2 B per layer call, each byte counted once.

* a step = L layers x (store + decode), L distinct caches (4.8 GB for cfg2, far above the 126 MB
  L2, so nothing is reused between layer calls or steps);
* ``value``: the step is captured once into a CUDA graph (the reference's block-diffusion runner
  replays its decode step the same way) and K replays are timed with CUDA events between
  barriers; inputs are resident in HBM;
* ``e2e``: the same step through the Python entry points with HOST inputs: q/k/v and all
  metadata copied from pinned memory, outputs copied back, every step, inside the timed region;
* ``roofline``: the decode kernel alone (a graph of the L decode launches, CUDA events around each
  replay, divided by L), against the measured HBM copy bandwidth;
* ``cpu_baseline`` / ``--impl reference``: the PyTorch fp32 CPU restatement of the reference's
  attention check (oracle/attn_oracle.py) on the host cores, on a bounded sample (one layer).

N > 1 is weak scaling: every rank runs its own batch of the workload (rank-specific seed) on its own
GPU with no data-path collective; NCCL only reduces timings.  ``--scaling strong`` instead shards
one global batch by sequences (LPT on KV tokens).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np
import torch

FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum per decode launch of the workload, from an ncu capture of this
# command on two resident layer caches; None where no capture has been taken.
NCU_TRAFFIC_BYTES = {"cfg2": 178475008 + 7841024}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg2", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"])
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (0 = the model's)")
    ap.add_argument("--num-splits", type=int, default=0)
    ap.add_argument("--separate-store", action="store_true",
                    help="one store launch and one attention launch per layer (default: the attention call stores too)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-group", type=int, default=2, help="layers per host<->device copy group of the e2e step")
    ap.add_argument("--no-strong", action="store_true", help="skip the cfg5 strong-scaling side measurement")
    ap.add_argument("--no-splitk", action="store_true", help="skip the split-K side measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill side measurement")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU kernels (needs baseline/_ref)")
    ap.add_argument("--no-store-load", action="store_true", help="skip the store / load bandwidth side measurement")
    ap.add_argument("--only-store-load", action="store_true",
                    help="run only the store / load side measurement and print its object (for profiler captures)")
    ap.add_argument("--only-prefill", action="store_true",
                    help="run only the prefill side measurement and print its object (for profiler captures)")
    ap.add_argument("--store-load-seqs", type=int, default=256,
                    help="sequences of the cfg5-shaped layer used by the store / load measurement (256 = all)")
    return ap.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak_tflops():
    """Measured dense bf16 peak (burst figure: the decode kernel is timed launch by launch), if the file gives one."""
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["bf16_tflops"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled while the timed region runs."""
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.rows, self.proc = [], None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), line.strip()))

    def window(self, t0, t1):
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, line in self.rows:
            if ts < t0 - 0.15 or ts > t1 + 0.15:
                continue
            parts = [x.strip() for x in line.split(",")]
            try:
                sm.append(float(parts[0])); smax = max(smax, float(parts[1]))
            except Exception:
                continue
            for n, v in zip(names, parts[2:]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax or None,
                "reasons": sorted(reasons), "samples": len(sm)}

    def stop(self):
        if self.proc:
            self.proc.terminate()


def cpu_attention_baseline(w, budget_s=12.0):
    """Oracle port on the host cores: one layer of the workload (all sequences), repeated within a
    time budget.  Returns (GB/s of bf16-equivalent KV, query tok/s, cores, sample description)."""
    from diffulex_b200.workload import make_problem
    from oracle import attn_oracle
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    p = make_problem(w, device="cpu", values="numpy")
    f = lambda t: t.float()
    args = (f(p.q), f(p.k), f(p.v), f(p.k_cache), f(p.v_cache), p.block_tables, p.context_lens, p.cu_seqlens_q,
            p.cu_seqlens_k, p.scale, p.mask_mode, p.geometry.diffusion_block_size)
    attn_oracle.decode_attention(*args)  # warm-up
    times, t_start = [], time.time()
    while len(times) < 3 or (time.time() - t_start < budget_s and len(times) < 50):
        t = time.time(); attn_oracle.decode_attention(*args); times.append(time.time() - t)
    dt = statistics.median(times)
    return (p.kv_bytes() / dt / 1e9, int(p.host_new_lens.sum()) / dt, cores,
            f"1 of {w.geometry.layers} layers, all {p.num_seqs} sequences, fp32, {len(times)} runs, median", dt * 1e3)


def store_load_bandwidth(dlx, dev, peak, num_seqs=256):
    """Store and load kernels on one cfg5-shaped layer (256 sequences, ctx U[4096, 32768]: 9.7 GB of KV, far
    larger than L2).  Algorithmic bytes: store N_valid * row * 2 (K and V) * 2 (read + write) + N * sizeof(slot);
    load rows * row * 2 * 2.  Three cases: the per-step store of the in-flight blocks (N = 8192), a prefill-sized
    store (every cached token of the layer) and the load of every sequence's [prefix ; in-flight] rows."""
    from diffulex_b200.workload import make_problem, named_workload, small_workload
    w5 = named_workload("cfg5")
    if num_seqs < len(w5.context_lens):   # a prefix of the same sequences: smaller footprint for profiler captures
        g5 = w5.geometry
        w5 = small_workload("cfg5_prefix", g5.num_q_heads, g5.num_kv_heads, g5.head_dim, g5.page_size,
                            g5.diffusion_block_size, list(w5.context_lens[:num_seqs]), list(w5.new_lens[:num_seqs]),
                            w5.mask_mode, w5.seed)
    p = make_problem(w5, device=dev, values="torch")
    geo = p.geometry
    row = geo.num_kv_heads * geo.head_dim * 2
    md = p.metadata("varlen")

    def timed(fn, iters):
        fn(); torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record(); torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters * 1e-3

    n_step = p.k.shape[0]
    # the per-step store is a 35 MB copy: replayed from a CUDA graph (20 launches) so that host launch time is out
    store_step = lambda: dlx.store_kvcache_unified_layout(p.k, p.v, p.k_cache, p.v_cache, md.slot_mapping, md)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        store_step()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(20):
            store_step()
    t_step = timed(g.replay, 5) / 20
    # prefill-sized: one row per cached token, written to the slot it already occupies
    slots = []
    bt, ctx = p.block_tables.cpu(), p.host_context_lens
    for s in range(p.num_seqs):
        pos = torch.arange(int(ctx[s]))
        slots.append(bt[s][pos // geo.page_size].long() * geo.page_size + pos % geo.page_size)
    slots = torch.cat(slots).to(torch.int32).to(dev)
    n_big = slots.numel()
    kb = torch.empty(n_big, geo.num_kv_heads, geo.head_dim, dtype=p.k.dtype, device=dev).normal_()
    vb = torch.empty_like(kb).normal_()
    t_big = timed(lambda: dlx.store_kvcache_unified_layout(kb, vb, p.k_cache, p.v_cache, slots, md), 3)
    del kb, vb
    rows = int(p.host_context_lens.sum() + p.host_new_lens.sum())
    md.total_kv_rows = rows
    t_load = timed(lambda: dlx.load_kvcache(p.k_cache, p.v_cache, md, p.k, p.v), 3)
    gb = lambda b, t: b / t / 1e9
    out = {
        "workload": f"cfg5-shaped layer: {p.num_seqs} seqs, ctx U[4096,32768], 28q/4kv x 128, page 256",
        "store_step": {"tokens": n_step, "us": t_step * 1e6, "gbps": gb(n_step * (row * 4 + 4), t_step)},
        "store_prefill_sized": {"tokens": n_big, "ms": t_big * 1e3, "gbps": gb(n_big * (row * 4 + 4), t_big)},
        "load": {"rows": rows, "ms": t_load * 1e3, "gbps": gb(rows * row * 4, t_load)},
        "peak_gbps": peak,
    }
    for k in ("store_step", "store_prefill_sized", "load"):
        out[k]["frac_of_peak"] = out[k]["gbps"] / peak
    return out


def pin_cpus(local_rank: int, world: int) -> None:
    """Give every rank of a multi-GPU run its own slice of the host cores this process may use (the launcher
    starts all ranks with the same affinity mask, so eight ranks would otherwise share the same cores for
    their copy and launch loops).  Pinned host buffers are then first touched from those cores."""
    if world <= 1:
        return
    try:
        cores = sorted(os.sched_getaffinity(0))
        per = max(1, len(cores) // world)
        mine = cores[local_rank * per:(local_rank + 1) * per] or cores
        os.sched_setaffinity(0, mine)
        torch.set_num_threads(max(1, min(per, 8)))
    except (AttributeError, OSError):
        pass


def strong_cfg5(dlx, dp, dev, rank, world, peak):
    """Strong scaling of the scaling-sweep configuration: its 256 sequences (seed fixed) are sharded over the ranks
    by longest-processing-time on KV tokens, every rank stores and decodes its shard (one layer), and the outputs
    are gathered over the process group.  Reported: per-rank time, imbalance, aggregate KV GB/s of the slowest rank,
    the gather's time, and a bit checksum of the gathered tensor against the sum of the ranks' own checksums."""
    from diffulex_b200.workload import make_problem, named_workload, partition_lpt, shard_workload
    w_global = named_workload("cfg5")
    w, owned = shard_workload(w_global, rank, world)
    parts = (partition_lpt((w_global.context_lens + w_global.new_lens).tolist(), world) if world > 1
             else [list(range(len(w_global.context_lens)))])
    p = make_problem(w, device=dev, values="torch")
    md = p.metadata("static")
    out = torch.empty_like(p.q)

    def step():   # one layer call: store the in-flight rows and attend
        dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md, out=out,
                                   store_slot_mapping=md.slot_mapping)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 5
    ea.record()
    for _ in range(n):
        step()
    eb.record()
    torch.cuda.synchronize()
    ms_local = ea.elapsed_time(eb) / n
    per_rank = dp.gather_timings(ms_local, dev)
    bytes_local = float(p.kv_bytes())
    per_rank_bytes = dp.gather_timings(bytes_local, dev)
    total_bytes = sum(per_rank_bytes)
    slowest = max(per_rank)
    # gather of the outputs (59 MB in total) over the process group, timed on the device
    q_lens = w_global.new_lens.tolist()
    full = dp.gather_outputs(out, parts, q_lens)
    torch.cuda.synchronize()
    gather_ms = float("inf")
    for _ in range(3):   # best of three: the first gathers also pay for NCCL's channel set-up
        ea.record()
        full = dp.gather_outputs(out, parts, q_lens)
        eb.record()
        torch.cuda.synchronize()
        gather_ms = min(gather_ms, dp.max_over_ranks(ea.elapsed_time(eb), dev))
    bits_sum = lambda t: float(t.contiguous().view(torch.int16).to(torch.int64).sum().item())
    local_sum = bits_sum(out)
    return {
        "workload": "cfg5: 256 seqs, ctx U[4096,32768], one layer, sequences LPT-sharded over the ranks",
        "n_gpus": world, "per_rank_ms": per_rank, "imbalance_max_over_mean": slowest / (sum(per_rank) / len(per_rank)),
        "ms": slowest, "value": total_bytes / (slowest * 1e-3) / 1e9, "unit": "GB/s",
        "per_gpu_frac_of_hbm_peak": [b / (t * 1e-3) / 1e9 / peak for b, t in zip(per_rank_bytes, per_rank)],
        "gather_ms": gather_ms, "gather_bytes": full.numel() * full.element_size(),
        "gather_checksum_ok": bits_sum(full) == dp.sum_over_ranks(local_sum, dev),
        "gather_backend": torch.distributed.get_backend() if world > 1 else "none (one rank)",
    }


def splitk_side(dlx, ops, dev, peak):
    """A few long sequences (the first 8 of the scaling-sweep configuration: 32 work items for 74 CTA pairs), where
    the planner cuts every sequence into key-range splits and the combine kernel merges them."""
    from diffulex_b200.workload import make_problem, named_workload, small_workload
    w5 = named_workload("cfg5")
    g = w5.geometry
    w = small_workload("cfg5_first8", g.num_q_heads, g.num_kv_heads, g.head_dim, g.page_size, g.diffusion_block_size,
                       list(w5.context_lens[:8]), list(w5.new_lens[:8]), w5.mask_mode, w5.seed)
    p = make_problem(w, device=dev, values="torch")
    md = p.metadata("static")
    splits = ops.planned_num_splits(p.q, p.k, p.v, p.k_cache, p.v_cache, p.block_tables, p.context_lens,
                                    p.cu_seqlens_q, p.cu_seqlens_k, p.scale, md.max_seqlen_q, 0, p.mask_mode,
                                    g.diffusion_block_size, 0)
    out = torch.empty_like(p.q)
    fn = lambda: dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md, out=out)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(10):
            fn()
    graph.replay()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(3):
        graph.replay()
    eb.record()
    torch.cuda.synchronize()
    us = ea.elapsed_time(eb) / 30 * 1e3
    gbps = p.kv_bytes() / (us * 1e-6) / 1e9
    return {"workload": "8 sequences, ctx 4k..32k (cfg5's first 8), 28q/4kv x 128", "num_splits": splits,
            "launches_per_call": 2 if splits > 1 else 1, "us_per_call": us, "gbps": gbps, "frac_of_peak": gbps / peak,
            "kernels": "decode attention (key-range splits) + combine_splits"}


def _graph_us(fn, calls=10, replays=3):
    """Device time per call of ``fn``, from CUDA-graph replays (events on the current stream)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(calls):
            fn()
    graph.replay()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(replays):
        graph.replay()
    eb.record()
    torch.cuda.synchronize()
    return ea.elapsed_time(eb) / (calls * replays) * 1e3


def _eager_us(fn, calls=20):
    """Device time per call of ``fn`` launched eagerly (for code that cannot be captured: it synchronises)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(calls):
        fn()
    eb.record()
    torch.cuda.synchronize()
    return ea.elapsed_time(eb) / calls * 1e3


def prefill_side(dlx, dev):
    """Prefill attention (no cache) on prompts of the headline geometry: 8 prompts of 4096 tokens, block-causal
    with 32-token diffusion blocks and full.  FLOPs = 4 * head_dim * visible (query, key) pairs * query heads."""
    from types import SimpleNamespace as NS
    geo = dict(hq=28, hkv=4, hd=128, seqs=8, qlen=4096, dbs=32)
    tq = geo["seqs"] * geo["qlen"]
    gen = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn(tq, geo["hq"], geo["hd"], device=dev, dtype=torch.bfloat16, generator=gen)
    k = torch.randn(tq, geo["hkv"], geo["hd"], device=dev, dtype=torch.bfloat16, generator=gen)
    v = torch.randn(tq, geo["hkv"], geo["hd"], device=dev, dtype=torch.bfloat16, generator=gen)
    cu = torch.arange(0, tq + 1, geo["qlen"], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    res = {"workload": f"{geo['seqs']} prompts x {geo['qlen']} tokens, {geo['hq']}q/{geo['hkv']}kv x {geo['hd']}, "
                       f"diffusion block {geo['dbs']}", "peak_tflops": tensor_peak_tflops() or 1590.0}
    for kind in ("block_attention", "full_attention"):
        md = NS(is_prefill=True, attn_type=kind, cu_seqlens_q=cu, cu_seqlens_k=cu, max_seqlen_q=geo["qlen"],
                max_seqlen_k=geo["qlen"], diffusion_block_size=geo["dbs"])
        us = _graph_us(lambda: dlx.dllm_flash_attn_prefill(q, k, v, geo["hd"] ** -0.5, md, out=out), calls=3, replays=3)
        n, b = geo["qlen"], geo["dbs"]
        pairs = n * n if kind == "full_attention" else sum(b * (i + 1) * b for i in range(n // b))
        flops = 4.0 * geo["hd"] * pairs * geo["hq"] * geo["seqs"]
        res[kind] = {"us_per_call": us, "tflops": flops / (us * 1e-6) / 1e12,
                     "frac_of_peak": flops / (us * 1e-6) / 1e12 / res["peak_tflops"],
                     "query_tokens_per_s": tq / (us * 1e-6)}
    return res


def reference_gpu_side(dlx, dev, w):
    """The reference's OWN GPU kernels (copied unmodified by baseline/make_ref.sh into baseline/_ref) on one layer of
    the headline workload, next to this package's kernels on the same tensors: Triton store (K4), Triton gather +
    dense varlen attention (K6 + K7, the reference's varlen decode), TileLang decode kernel (K1, its static decode).
    A side measurement: the `--impl reference` arm stays the CPU port."""
    ref_root = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "diffulex_kernel")):
        return {"unavailable": "baseline/_ref not made (baseline/make_ref.sh)"}
    import importlib
    from diffulex_b200.workload import make_problem
    sys.path.insert(0, ref_root)
    res = {"workload": f"one layer of {w.name}", "versions": {}}
    try:
        for name in ("triton", "tilelang", "flash_attn"):
            try:
                res["versions"][name] = getattr(importlib.import_module(name), "__version__", "?")
            except Exception as e:  # noqa: BLE001
                res["versions"][name] = f"import failed: {type(e).__name__}: {str(e)[:120]}"
        kv = importlib.import_module("diffulex_kernel.python.kv_cache_kernels")
        fa = importlib.import_module("diffulex_kernel.python.dllm_flash_attn")
        p = make_problem(w, device=dev, values="torch")
        kvb = p.kv_bytes()
        out = torch.empty_like(p.q)
        md_s, md_v = p.metadata("static"), p.metadata("varlen")

        def entry(us):
            return {"us": us, "kv_gbps": kvb / (us * 1e-6) / 1e9}
        ours = {"store_us": _graph_us(lambda: dlx.store_kvcache_unified_layout(p.k, p.v, p.k_cache, p.v_cache, p.slot_mapping, md_s)),
                "decode_static": entry(_graph_us(lambda: dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md_s, out=out))),
                "decode_varlen": entry(_graph_us(lambda: dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md_v, out=out)))}
        theirs = {}
        try:
            theirs["store_us"] = _graph_us(lambda: kv.store_kvcache_unified_layout(p.k, p.v, p.k_cache, p.v_cache, p.slot_mapping, md_s))
        except Exception as e:  # noqa: BLE001
            theirs["store_us"] = f"failed: {type(e).__name__}: {str(e)[:200]}"
        try:   # its gather sizes the output from a device value (a host sync): eager launches, device-timed
            theirs["decode_varlen"] = entry(_eager_us(lambda: fa.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md_v)))
            theirs["decode_varlen"]["kernels"] = "Triton load_kvcache + flash_attn_varlen_func"
        except Exception as e:  # noqa: BLE001
            theirs["decode_varlen"] = f"failed: {type(e).__name__}: {str(e)[:200]}"
        best = None
        tried = {}
        # the reference autotunes 54 tile configurations during warm-up; a few of them here, best kept
        for cfg in ((64, 64, 1, 128), (64, 128, 2, 128), (128, 64, 2, 256), (128, 128, 2, 256)):
            fa.kernel_config = dict(BLOCK_M=cfg[0], BLOCK_N=cfg[1], NUM_STAGES=cfg[2], NUM_THREADS=cfg[3])
            try:
                o = fa.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md_s)
                ok = bool(torch.allclose(o.float(), dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md_s).float(),
                                         atol=2e-2, rtol=1e-2))
                us = _eager_us(lambda: fa.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md_s))
                tried["x".join(map(str, cfg))] = {"us": us, "agrees_with_ours": ok}
                if ok and (best is None or us < best):
                    best = us
            except Exception as e:  # noqa: BLE001
                tried["x".join(map(str, cfg))] = f"failed: {type(e).__name__}: {str(e)[:160]}"
        theirs["decode_static"] = dict(entry(best), kernels="TileLang dllm_flash_attn_decode_kernel",
                                       configs=tried) if best else {"configs": tried}
        res["ours"], res["reference"] = ours, theirs
        if best:
            res["decode_static_speedup"] = best / ours["decode_static"]["us"]
        if isinstance(theirs.get("decode_varlen"), dict):
            res["decode_varlen_speedup"] = theirs["decode_varlen"]["us"] / ours["decode_varlen"]["us"]
    except Exception as e:  # noqa: BLE001
        res["unavailable"] = f"{type(e).__name__}: {str(e)[:300]}"
    finally:
        sys.path.remove(ref_root)
    return res


def run_reference(args, w, rank, world):
    """The reference's CPU implementation of the path (its PyTorch attention check, restated in
    oracle/attn_oracle.py; the reference itself is Python and cannot travel) on the host cores."""
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        pass  # warm-up happens inside cpu_attention_baseline
    gbs, toks, cores, sample, sample_ms = cpu_attention_baseline(w, budget_s=max(5.0, min(60.0, 3.0 * args.steps)))
    line = {
        "impl": "reference", "metric": "decode_attn_kv_read_gbps", "value": gbs, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sample_ms, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "query_tokens_per_s": toks,
        "config": {"workload": f"{w.name}: {w.note}", "sample": sample},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line))


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    from diffulex_b200.workload import make_problem, named_workload, shard_workload

    w_global = named_workload(args.workload)
    if args.impl == "reference":
        run_reference(args, w_global, rank, world)
        return

    import torch.distributed as dist
    assert torch.cuda.is_available(), "bench.py needs a CUDA device (there is no CPU fallback)"
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pin_cpus(local_rank, world)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    import diffulex_b200 as dlx
    from diffulex_b200 import dp, ops

    if args.only_store_load:
        print(json.dumps(store_load_bandwidth(dlx, dev, peaks()[0], args.store_load_seqs)))
        return
    if args.only_prefill:
        print(json.dumps(prefill_side(dlx, dev)))
        return

    # ---- this rank's batch ----
    if args.scaling == "strong":
        w, owned = shard_workload(w_global, rank, world)
    else:
        w = named_workload(args.workload, seed=w_global.seed + 100 * rank) if world > 1 else w_global
    geo = w.geometry
    L = args.layers or geo.layers
    base = make_problem(w, device=dev, values="torch")
    layers = [base]
    gen = torch.Generator(device=dev); gen.manual_seed(w.seed + 1)
    for _ in range(1, L):
        rnd = lambda t: torch.empty_like(t).normal_(0, 1, generator=gen)
        layers.append(type(base)(**{**{f: getattr(base, f) for f in base.__dataclass_fields__},
                                    "q": rnd(base.q), "k": rnd(base.k), "v": rnd(base.v),
                                    "k_cache": rnd(base.k_cache), "v_cache": rnd(base.v_cache)}))
    md = base.metadata("static")
    md.num_splits = args.num_splits
    kv_bytes_layer = base.kv_bytes()
    kv_tokens_layer = int(base.host_context_lens.sum() + base.host_new_lens.sum())
    query_block, seqs_per_gpu = int(base.host_new_lens.max()), base.num_seqs
    q_tokens = int(base.host_new_lens.sum())
    flops_layer = base.flops()
    splits = ops.planned_num_splits(base.q, base.k, base.v, base.k_cache, base.v_cache, base.block_tables,
                                    base.context_lens, base.cu_seqlens_q, base.cu_seqlens_k, base.scale,
                                    md.max_seqlen_q, 0, base.mask_mode, geo.diffusion_block_size, args.num_splits)
    fused = not args.separate_store   # the attention call also stores the layer's in-flight K / V rows
    launches_per_layer = 2 + (1 if splits > 1 else 0)   # store kernel + attention kernel either way

    def layer_call(q, k, v, p, m, out=None):
        """What the attention layer does per decode call: store the in-flight rows, attend."""
        if fused:
            return dlx.dllm_flash_attn_decode(q, k, v, p.k_cache, p.v_cache, p.scale, m, out=out,
                                              store_slot_mapping=m.slot_mapping)
        dlx.store_kvcache_unified_layout(k, v, p.k_cache, p.v_cache, m.slot_mapping, m)
        return dlx.dllm_flash_attn_decode(q, k, v, p.k_cache, p.v_cache, p.scale, m, out=out)

    def step(outs=None):
        for i, p in enumerate(layers):
            o = layer_call(p.q, p.k, p.v, p, md)
            if outs is not None:
                outs[i] = o
        return o

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- value: CUDA-graph replay of the step ----
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(); step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    sampler = ClockSampler(local_rank) if rank == 0 else None
    time.sleep(0.25)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    barrier()
    t_wall1 = time.time()
    ms_local = e0.elapsed_time(e1)
    ms_total = dp.max_over_ranks(ms_local, dev)
    clocks = sampler.window(t_wall0, t_wall1) if sampler else None
    total_kv_bytes = dp.sum_over_ranks(float(kv_bytes_layer) * L * args.steps, dev)
    total_q_tokens = dp.sum_over_ranks(float(q_tokens) * args.steps, dev)
    value = total_kv_bytes / (ms_total * 1e-3) / 1e9
    per_rank_ms = dp.gather_timings(ms_local, dev)

    # ---- roofline: the decode kernel alone ----
    # A second CUDA graph holds only the L decode launches (no store); each replay is bracketed by CUDA
    # events on the launching stream, so the average launch duration is (replay time / L) with no host
    # launch gaps inside.  Same caches as above: every launch reads its own layer's 163 MB (cfg2).
    peak, peak_kind = peaks()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for p in layers:
            dlx.dllm_flash_attn_decode(p.q, p.k, p.v, p.k_cache, p.v_cache, p.scale, md)
    torch.cuda.current_stream().wait_stream(side)
    # The step's schedule is planned once, outside this graph (in the step graph above the planning launch is inside):
    # what is timed here is the attention kernel (and the combine kernel when the plan splits), nothing else.
    from diffulex_b200._lib import DLX_MASK_BLOCK_CAUSAL, DLX_MASK_FULL
    p0 = layers[0]
    dec_args = (md.block_tables, md.context_lens, md.cu_seqlens_q, md.cu_seqlens_k, float(p0.scale),
                int(md.max_seqlen_q), 0, DLX_MASK_BLOCK_CAUSAL if md.mask_mode == "d2f_block_causal" else DLX_MASK_FULL,
                int(md.diffusion_block_size), int(getattr(md, "num_splits", 0) or 0))
    sched = ops.decode_schedule(p0.q, p0.k, p0.k_cache, p0.v_cache, *dec_args)
    dec_outs = [torch.empty_like(p.q) for p in layers]
    g_dec = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_dec):
        for p, o in zip(layers, dec_outs):
            ops.decode_attn_out(o, p.q, p.k, p.v, p.k_cache, p.v_cache, *dec_args, sched)
    for _ in range(3):
        g_dec.replay()
    evs = []
    for it in range(min(max(args.steps, 5), 20)):
        ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ea.record(); g_dec.replay(); eb.record()
        evs.append((ea, eb))
    torch.cuda.synchronize()
    launch_ms = [ea.elapsed_time(eb) / L for ea, eb in evs]
    avg_launch_ms = sum(launch_ms) / len(launch_ms)
    achieved = kv_bytes_layer / (avg_launch_ms * 1e-3) / 1e9
    traffic = NCU_TRAFFIC_BYTES.get(args.workload)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "peak_kind": f"of {peak_kind}", "kernel": "decode attention (+ combine if split)",
                "algorithmic_bytes_per_launch": kv_bytes_layer, "avg_launch_us": avg_launch_ms * 1e3,
                "min_launch_us": min(launch_ms) * 1e3, "tflops": flops_layer / (avg_launch_ms * 1e-3) / 1e12}
    tensor_peak = tensor_peak_tflops()   # the second fraction asked for on cfg2 / cfg5: tensor-pipe use of the kernel
    if tensor_peak:
        roofline["tensor_frac"] = roofline["tflops"] / tensor_peak
        roofline["tensor_peak_tflops"] = tensor_peak

    # ---- e2e: host buffers in, host buffers out, every step ----
    e2e = None
    host_cost = None
    if not args.no_e2e:
        pin = lambda t: t.cpu().pin_memory()
        h_q = torch.stack([p.q for p in layers]).cpu().pin_memory()
        h_k = torch.stack([p.k for p in layers]).cpu().pin_memory()
        h_v = torch.stack([p.v for p in layers]).cpu().pin_memory()
        h_meta = {n: pin(getattr(base, n)) for n in ("block_tables", "context_lens", "cu_seqlens_q", "cu_seqlens_k",
                                                     "slot_mapping")}
        h_out = torch.empty((L,) + tuple(base.q.shape), dtype=base.q.dtype).pin_memory()
        d_q, d_k, d_v = (torch.empty_like(t, device=dev) for t in (h_q, h_k, h_v))
        d_out = torch.empty_like(h_out, device=dev)
        from types import SimpleNamespace
        h2d = sum(t.numel() * t.element_size() for t in (h_q, h_k, h_v, *h_meta.values()))
        d2h = h_out.numel() * h_out.element_size()
        # Copies go in groups of layers: few, large transfers (one cudaMemcpyAsync per tensor per group), while the
        # host->device copies of group g+1 and the device->host copy of group g-1 still run under the kernels of
        # group g (three streams; PCIe is full duplex).
        groups = [list(range(i, min(i + args.e2e_group, L))) for i in range(0, L, args.e2e_group)]
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        ev_in = [torch.cuda.Event() for _ in groups]
        ev_c = [torch.cuda.Event() for _ in groups]

        def e2e_step(copies=True, kernels=True):
            cur = torch.cuda.current_stream()
            s_in.wait_stream(cur)
            m = SimpleNamespace(**vars(md))
            m.__dict__.pop("_dlx_plan", None)          # a new step: the schedule is planned again from the copied metadata
            with torch.cuda.stream(s_in):
                if copies:
                    for n_, t in h_meta.items():
                        setattr(m, n_, t.to(dev, non_blocking=True))
                for gi, g in enumerate(groups):
                    if copies:
                        sl = slice(g[0], g[-1] + 1)
                        d_q[sl].copy_(h_q[sl], non_blocking=True)
                        d_k[sl].copy_(h_k[sl], non_blocking=True)
                        d_v[sl].copy_(h_v[sl], non_blocking=True)
                    ev_in[gi].record(s_in)
            for gi, g in enumerate(groups):
                cur.wait_event(ev_in[gi])
                if kernels:
                    for i in g:
                        p = layers[i]
                        layer_call(d_q[i], d_k[i], d_v[i], p, m, out=d_out[i])
                ev_c[gi].record(cur)
                s_out.wait_event(ev_c[gi])
                if copies:
                    with torch.cuda.stream(s_out):
                        sl = slice(g[0], g[-1] + 1)
                        h_out[sl].copy_(d_out[sl], non_blocking=True)
            cur.wait_stream(s_out)
            cur.synchronize()  # the caller holds the result on the host

        def timed_e2e(n, **kw):
            for _ in range(2):
                e2e_step(**kw)
            barrier()
            e0.record()
            for _ in range(n):
                e2e_step(**kw)
            e1.record()
            barrier()
            return dp.max_over_ranks(e0.elapsed_time(e1), dev) / n

        for _ in range(max(1, min(args.warmup, 3))):
            e2e_step()
        n_e2e = max(3, min(args.steps, 10))
        ms_e2e = timed_e2e(n_e2e)
        tot = dp.sum_over_ranks(float(kv_bytes_layer) * L, dev)
        e2e = {"value": tot / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": n_e2e, "ms_per_step": ms_e2e,
               # the same step with the kernels left out (what the copies alone cost: PCIe / host memory ceiling) and
               # with the copies left out (resident inputs through the same Python loop: launch cost + device time)
               "copy_only_ms": timed_e2e(3, kernels=False), "launch_only_ms": timed_e2e(3, copies=False),
               "layers_per_copy_group": args.e2e_group, "cpu_affinity": sorted(os.sched_getaffinity(0))[:4] + ["..."]}
        e2e["host_link_gbps"] = (h2d + d2h) * world / (e2e["copy_only_ms"] * 1e-3) / 1e9   # all ranks, both directions

        # host time per eager call (device-resident inputs): what a runner that never captures a graph pays per layer
        p0 = layers[0]
        m = SimpleNamespace(**vars(md))
        def host_us(fn, n=300):
            fn(); torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            dt = time.perf_counter() - t0
            torch.cuda.synchronize()
            return dt / n * 1e6
        host_cost = {
            "store_us": host_us(lambda: dlx.store_kvcache_unified_layout(p0.k, p0.v, p0.k_cache, p0.v_cache, m.slot_mapping, m)),
            "decode_us": host_us(lambda: dlx.dllm_flash_attn_decode(p0.q, p0.k, p0.v, p0.k_cache, p0.v_cache, p0.scale, m,
                                                                     out=d_out[0])),
            "calls": 300, "note": "wall time per call of the Python entry point, launches queue on the device",
        }

    # ---- side measurements: the cfg2 state is released first ----
    del layers, graph, g_dec, base, dec_outs
    if e2e is not None:
        del h_q, h_k, h_v, h_out, d_q, d_k, d_v, d_out
    torch.cuda.empty_cache()
    strong = None
    if not args.no_strong:   # every rank takes part: sequences sharded over the ranks, outputs gathered
        strong = strong_cfg5(dlx, dp, dev, rank, world, peak)
        torch.cuda.empty_cache()
    splitk = None
    if rank == 0 and world == 1 and not args.no_splitk:
        splitk = splitk_side(dlx, ops, dev, peak)
        torch.cuda.empty_cache()
    # store and load bandwidth on a cfg5-shaped layer (rank 0, one GPU)
    store_load = None
    if rank == 0 and world == 1 and not args.no_store_load:
        store_load = store_load_bandwidth(dlx, dev, peak, args.store_load_seqs)

    prefill = None
    if rank == 0 and world == 1 and not args.no_prefill:
        prefill = prefill_side(dlx, dev)
        torch.cuda.empty_cache()
    reference_gpu = None
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        reference_gpu = reference_gpu_side(dlx, dev, w_global)
        torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, toks, cores, sample, _ = cpu_attention_baseline(w_global)
        cpu = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample,
               "query_tokens_per_s": toks}
    if sampler:
        sampler.stop()

    if rank == 0:
        line = {
            "metric": "decode_attn_kv_read_gbps", "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_total / args.steps,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "query_tokens_per_s": total_q_tokens / (ms_total * 1e-3),
            "config": {"workload": f"{w_global.name}: {w_global.note}", "layers": L, "seqs_per_gpu": seqs_per_gpu,
                       "heads": f"{geo.num_q_heads}q/{geo.num_kv_heads}kv x {geo.head_dim}", "page_size": geo.page_size,
                       "query_block": query_block, "kv_tokens_per_layer_per_gpu":
                       kv_tokens_layer, "num_splits": splits,
                       "step": ("L x (one call: store kernel + decode attention kernel), CUDA-graph replay" if fused
                                else "L x (store_kvcache_unified + decode attention), CUDA-graph replay"),
                       "l2": f"inputs larger than L2: {L} distinct layer caches, "
                             f"{kv_bytes_layer * L / 1e9:.2f} GB of KV per step",
                       "parallelism": f"dp{world}" + ("" if world == 1 else f" ({args.scaling})")},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "host_us_per_call": host_cost,
            "strong_cfg5": strong, "splitk": splitk, "store_load": store_load, "prefill": prefill,
            "reference_gpu": reference_gpu,
            # per step: L x (store + decode [+ combine]) + the one planning launch of the step's schedule
            "gpu_launches": args.steps * (L * launches_per_layer + 1), "clocks": clocks, "per_rank_ms": per_rank_ms,
        }
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
