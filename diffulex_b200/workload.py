"""Seeded synthetic inputs for the dLLM decode hot path (store -> decode attention, and load).

Every problem is the input set one ``Attention.forward`` call of the reference sees in decode
(diffulex/attention/attn_impl.py:42-72): fresh ``q/k/v`` rows for the in-flight diffusion blocks,
a paged unified-layout KV cache ``[NB, PAGE, Hkv, hd]`` (diffulex/engine/model_runner.py:229-243),
``block_tables`` padded with -1 (diffulex/engine/model_runner.py:251-255), ``context_lens``,
``cu_seqlens_q/k`` and the per-token ``slot_mapping`` of the rows being cached.

Lengths and page tables always come from a numpy ``Generator`` (host side, tiny).  Tensor values
are N(0,1) rounded to bf16; they come from numpy for the small golden/parity cases (stable bit
patterns wherever the fixture is checked) and from a torch generator on the target device for
the bench-sized cases, which never leave the GPU.

The five named workloads restate the five benchmark configurations this project is measured on;
they stand in for real engine traffic (no dataset is involved on this path).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from types import SimpleNamespace
from typing import List, Optional, Sequence

import numpy as np
import torch

MASK_BD_FULL = 0          # every query row sees all cached keys and every fresh key
MASK_D2F_BLOCK_CAUSAL = 1  # fresh key j visible to row i iff j < (i // dbs + 1) * dbs

MASK_MODES = {"bd_full": MASK_BD_FULL, "varlen_full": MASK_BD_FULL, "d2f_block_causal": MASK_D2F_BLOCK_CAUSAL}


@dataclass
class Geometry:
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    page_size: int = 256
    diffusion_block_size: int = 32
    layers: int = 1

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads

    @property
    def kv_row_elems(self) -> int:
        return self.num_kv_heads * self.head_dim


@dataclass
class Workload:
    name: str
    geometry: Geometry
    context_lens: np.ndarray            # [S] cached prefix tokens
    new_lens: np.ndarray                # [S] in-flight (query == fresh key) tokens
    mask_mode: int = MASK_BD_FULL
    seed: int = 1234
    spare_pages: int = 16
    note: str = ""


def named_workload(name: str, seed: Optional[int] = None) -> Workload:
    """The five benchmark configurations, by short name ("cfg1".."cfg5")."""
    idx = {"cfg1": 0, "cfg2": 1, "cfg3": 2, "cfg4": 3, "cfg5": 4}[name]
    seed = 1234 + idx if seed is None else seed
    rng = np.random.default_rng(seed)
    if name == "cfg1":
        g = Geometry(28, 4, 128, 256, 32, layers=1)
        ctx = np.array([128, 256, 384, 512]); new = np.full(4, 32)
        return Workload(name, g, ctx, new, MASK_BD_FULL, seed, note="CPU-runnable op test")
    if name == "cfg2":
        g = Geometry(28, 4, 128, 256, 32, layers=28)
        ctx = rng.integers(512, 2049, size=64); new = np.full(64, 32)
        return Workload(name, g, ctx, new, MASK_BD_FULL, seed, note="Dream-7B-shaped, 64 seqs, ctx U[512,2048]")
    if name == "cfg3":
        g = Geometry(32, 32, 128, 256, 32, layers=32)
        ctx = rng.integers(256, 1025, size=32); new = np.full(32, 128)
        return Workload(name, g, ctx, new, MASK_D2F_BLOCK_CAUSAL, seed,
                        note="LLaDA-8B-shaped MHA, 4 in-flight 32-token blocks, D2F block-causal")
    if name == "cfg4":
        g = Geometry(32, 8, 128, 256, 4, layers=36)
        # The configuration names a log-normal with median 1024 but no sigma; sigma = 1.0 is used.
        ctx = np.clip(np.exp(rng.normal(math.log(1024.0), 1.0, size=128)), 128, 8192).astype(np.int64)
        new = np.full(128, 4)
        return Workload(name, g, ctx, new, MASK_BD_FULL, seed, note="SDAR-8B-shaped, 4-token blocks, log-normal ctx")
    if name == "cfg5":
        g = Geometry(28, 4, 128, 256, 32, layers=1)
        ctx = rng.integers(4096, 32769, size=256); new = np.full(256, 32)
        return Workload(name, g, ctx, new, MASK_BD_FULL, seed, note="Fast-dLLM-v2-7B-shaped scaling sweep")
    raise KeyError(name)


def partition_lpt(costs: Sequence[int], world_size: int) -> List[List[int]]:
    """Longest-processing-time assignment of sequences to data-parallel ranks.

    Sequences are independent units (each owns its page table and cache pages); the reference's DP
    splits requests across replicas with no collective (diffulex/engine/dp_worker.py:285-312).
    Cost is the sequence's KV token count.  Deterministic: ties break on the sequence index.
    Returns, per rank, the sorted list of global sequence indices it owns.
    """
    order = sorted(range(len(costs)), key=lambda i: (-int(costs[i]), i))
    load = [0] * world_size
    owned: List[List[int]] = [[] for _ in range(world_size)]
    for i in order:
        r = min(range(world_size), key=lambda j: (load[j], j))
        owned[r].append(i)
        load[r] += int(costs[i])
    return [sorted(o) for o in owned]


def shard_workload(w: Workload, rank: int, world_size: int) -> "tuple[Workload, List[int]]":
    """The sub-workload rank ``rank`` owns, plus the global sequence indices it covers."""
    if world_size == 1:
        return w, list(range(len(w.context_lens)))
    owned = partition_lpt((w.context_lens + w.new_lens).tolist(), world_size)[rank]
    sub = Workload(w.name, w.geometry, w.context_lens[owned], w.new_lens[owned], w.mask_mode,
                   w.seed * 1000 + rank, w.spare_pages, w.note)
    return sub, owned


@dataclass
class DecodeProblem:
    """One layer's decode inputs. Tensors live on ``device``; K/V caches are bf16 unless stated."""
    geometry: Geometry
    mask_mode: int
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_tables: torch.Tensor      # [S, MAXB] int32, -1 padded
    context_lens: torch.Tensor      # [S] int32
    seq_lens_ts: torch.Tensor       # [S] int32 in-flight tokens per sequence
    cu_seqlens_q: torch.Tensor      # [S+1] int32
    cu_seqlens_k: torch.Tensor      # [S+1] int32, cumulates the FRESH lengths (static decode convention)
    cu_seqlens_k_total: torch.Tensor  # [S+1] int32, cumulates ctx+new (load_kvcache / varlen convention)
    slot_mapping: torch.Tensor      # [sum new] int32 flat slots of the in-flight rows
    scale: float = 0.0
    host_context_lens: np.ndarray = field(default=None, repr=False)
    host_new_lens: np.ndarray = field(default=None, repr=False)

    @property
    def num_seqs(self) -> int:
        return int(self.context_lens.numel())

    def kv_bytes(self) -> int:
        """Algorithmic KV bytes one decode call must read: every valid K and V row exactly once."""
        g = self.geometry
        toks = int(self.host_context_lens.sum() + self.host_new_lens.sum())
        return toks * 2 * g.num_kv_heads * g.head_dim * self.k_cache.element_size()

    def flops(self) -> float:
        """4 * Hq * hd * sum over query rows of visible keys."""
        g = self.geometry
        total = 0.0
        for c, n in zip(self.host_context_lens.tolist(), self.host_new_lens.tolist()):
            if self.mask_mode == MASK_D2F_BLOCK_CAUSAL:
                d = g.diffusion_block_size
                vis = sum(c + min(n, (i // d + 1) * d) for i in range(n))
            else:
                vis = n * (c + n)
            total += vis
        return 4.0 * g.num_q_heads * g.head_dim * total

    def metadata(self, decode_mode: str = "static") -> SimpleNamespace:
        """A duck-typed stand-in for the reference's attention metadata dataclasses
        (diffulex/attention/metadata.py:7-24 and the two strategy subclasses)."""
        g = self.geometry
        varlen = decode_mode == "varlen"
        return SimpleNamespace(
            is_prefill=False,
            cu_seqlens_q=self.cu_seqlens_q,
            cu_seqlens_k=self.cu_seqlens_k_total if varlen else self.cu_seqlens_k,
            max_seqlen_q=int(self.host_new_lens.max()),
            max_seqlen_k=int((self.host_context_lens + self.host_new_lens).max()) if varlen
            else int(self.host_new_lens.max()),
            slot_mapping=self.slot_mapping,
            context_lens=self.context_lens,
            block_tables=self.block_tables,
            page_block_size=g.page_size,
            attn_type="block_attention" if self.mask_mode == MASK_D2F_BLOCK_CAUSAL else "full_attention",
            diffusion_block_size=g.diffusion_block_size,
            decode_mode=decode_mode,
            num_seqs=self.num_seqs,
            seq_lens_ts=self.seq_lens_ts,
            seqs=[SimpleNamespace(diffusion_block_size=g.diffusion_block_size)],
            kv_cache_layout="unified",
            need_kv_cache_store=True,
            mask_mode={MASK_BD_FULL: "bd_full", MASK_D2F_BLOCK_CAUSAL: "d2f_block_causal"}[self.mask_mode],
        )


def build_page_tables(ctx: np.ndarray, new: np.ndarray, page: int, spare: int, rng: np.random.Generator,
                      permute: bool = True):
    """Random non-contiguous page assignment: physical ids are a permutation of the free list."""
    pages = (ctx + new + page - 1) // page
    nb = int(pages.sum()) + spare
    ids = rng.permutation(nb) if permute else np.arange(nb)
    maxb = max(int(pages.max()), 1)
    bt = np.full((len(ctx), maxb), -1, dtype=np.int32)
    p = 0
    for s, n in enumerate(pages.tolist()):
        bt[s, :n] = ids[p:p + n]
        p += n
    return bt, nb


def slots_for_new_tokens(bt: np.ndarray, ctx: np.ndarray, new: np.ndarray, page: int) -> np.ndarray:
    out = []
    for s in range(len(ctx)):
        pos = ctx[s] + np.arange(new[s])
        out.append(bt[s, pos // page].astype(np.int64) * page + pos % page)
    return np.concatenate(out) if out else np.zeros(0, np.int64)


def _normal_bf16(shape, *, device, values: str, rng: np.random.Generator, tgen: Optional[torch.Generator],
                 dtype=torch.bfloat16) -> torch.Tensor:
    if values == "numpy":
        a = rng.standard_normal(size=shape, dtype=np.float32)
        return torch.from_numpy(a).to(dtype).to(device)
    t = torch.empty(shape, dtype=dtype, device=device)
    t.normal_(0.0, 1.0, generator=tgen)
    return t


def make_problem(w: Workload, device="cpu", values: str = "numpy", dtype=torch.bfloat16,
                 permute_pages: bool = True, slot_dtype=torch.int32,
                 share_cache_with: Optional[DecodeProblem] = None) -> DecodeProblem:
    """Materialise one layer of ``w`` on ``device``.

    ``values="numpy"``: bit patterns depend only on (workload, seed).  ``values="torch"``: values
    are drawn by a torch generator on ``device`` (fast for multi-GB caches; not bit-stable across
    devices, so used only where outputs are compared within one run).
    """
    g = w.geometry
    rng = np.random.default_rng(w.seed)
    # Page tables use their own stream so that lengths drawn in named_workload stay independent.
    prng = np.random.default_rng([w.seed, 7])
    ctx = np.asarray(w.context_lens, dtype=np.int64)
    new = np.asarray(w.new_lens, dtype=np.int64)
    bt, nb = build_page_tables(ctx, new, g.page_size, w.spare_pages, prng, permute_pages)
    slots = slots_for_new_tokens(bt, ctx, new, g.page_size)
    tq = int(new.sum())
    tgen = None
    if values == "torch":
        tgen = torch.Generator(device=device)
        tgen.manual_seed(w.seed)
    mk = lambda shape: _normal_bf16(shape, device=device, values=values, rng=rng, tgen=tgen, dtype=dtype)
    q = mk((tq, g.num_q_heads, g.head_dim))
    k = mk((tq, g.num_kv_heads, g.head_dim))
    v = mk((tq, g.num_kv_heads, g.head_dim))
    if share_cache_with is not None:
        k_cache, v_cache = share_cache_with.k_cache, share_cache_with.v_cache
    else:
        k_cache = mk((nb, g.page_size, g.num_kv_heads, g.head_dim))
        v_cache = mk((nb, g.page_size, g.num_kv_heads, g.head_dim))
    i32 = lambda a: torch.from_numpy(np.asarray(a, dtype=np.int32)).to(device)
    cu_q = np.concatenate([[0], np.cumsum(new)])
    cu_tot = np.concatenate([[0], np.cumsum(ctx + new)])
    return DecodeProblem(
        geometry=g, mask_mode=w.mask_mode, q=q, k=k, v=v, k_cache=k_cache, v_cache=v_cache,
        block_tables=i32(bt), context_lens=i32(ctx), seq_lens_ts=i32(new),
        cu_seqlens_q=i32(cu_q), cu_seqlens_k=i32(cu_q), cu_seqlens_k_total=i32(cu_tot),
        slot_mapping=torch.from_numpy(slots).to(slot_dtype).to(device),
        scale=1.0 / math.sqrt(g.head_dim), host_context_lens=ctx, host_new_lens=new,
    )


def small_workload(name: str, num_q_heads: int, num_kv_heads: int, head_dim: int, page: int, dbs: int,
                   ctx: Sequence[int], new: Sequence[int], mask_mode: int = MASK_BD_FULL, seed: int = 0,
                   spare_pages: int = 3) -> Workload:
    g = Geometry(num_q_heads, num_kv_heads, head_dim, page, dbs)
    return Workload(name, g, np.asarray(ctx, dtype=np.int64), np.asarray(new, dtype=np.int64), mask_mode, seed,
                    spare_pages)
