"""Data-parallel plumbing: sequences are the unit of parallelism.

Each rank owns a subset of the sequences together with their page tables and cache pages
(``workload.shard_workload``: longest-processing-time by KV tokens) and runs the hot path on its
own GPU with no data-path collective -- the reference's DP replicas never talk to each other
either (diffulex/engine/dp_worker.py:97-146, 285-312).  The only collectives are the ones a
measurement or a caller that wants all outputs in one place needs: an all-gather of the padded
per-rank outputs followed by an inverse permutation, and a MAX all-reduce of per-rank timings.
Works on any ``torch.distributed`` backend (NCCL over NVLink on GPUs, gloo on CPU).
"""
from __future__ import annotations

from typing import List, Sequence

import numpy as np
import torch
import torch.distributed as dist


def world() -> "tuple[int, int]":
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def max_over_ranks(value: float, device="cpu") -> float:
    """MAX all-reduce of one float (a per-rank time): the job is as slow as its slowest rank."""
    rank, ws = world()
    if ws == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device="cpu") -> float:
    rank, ws = world()
    if ws == 1:
        return float(value)
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_timings(value: float, device="cpu") -> List[float]:
    rank, ws = world()
    if ws == 1:
        return [float(value)]
    t = torch.tensor([value], dtype=torch.float64, device=device)
    out = torch.empty(ws, dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(out, t)
    return out.cpu().tolist()


def gather_outputs(local_out: torch.Tensor, owned_per_rank: Sequence[Sequence[int]],
                   q_lens: Sequence[int]) -> torch.Tensor:
    """Assemble the global ``[sum q, Hq, hd]`` output from per-rank outputs.

    ``local_out`` holds this rank's sequences in ascending global sequence order
    (``owned_per_rank[rank]``); ``q_lens[s]`` is the query length of global sequence s.  Every rank
    returns the full tensor.  One all_gather of rank-padded buffers, then an index_select.
    """
    rank, ws = world()
    q_lens = np.asarray(q_lens, dtype=np.int64)
    rows_per_rank = [int(q_lens[list(o)].sum()) for o in owned_per_rank]
    assert local_out.shape[0] == rows_per_rank[rank], "local output does not match the partition"
    if ws == 1:
        return local_out
    pad = max(rows_per_rank)
    buf = local_out.new_zeros((pad,) + tuple(local_out.shape[1:]))
    buf[: local_out.shape[0]] = local_out
    gathered = local_out.new_empty((ws * pad,) + tuple(local_out.shape[1:]))
    dist.all_gather_into_tensor(gathered, buf)
    # row index, in the gathered buffer, of every global query row
    cu = np.concatenate([[0], np.cumsum(q_lens)])
    src = np.empty(int(cu[-1]), dtype=np.int64)
    for r, owned in enumerate(owned_per_rank):
        o = r * pad
        for s in owned:
            n = int(q_lens[s])
            src[cu[s]:cu[s] + n] = np.arange(o, o + n)
            o += n
    return gathered.index_select(0, torch.from_numpy(src).to(gathered.device))
