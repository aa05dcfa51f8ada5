"""Seeded case definitions shared by the golden-vector generator and the tests that read the
fixtures.  Every case rebuilds its inputs from (geometry, lengths, seed) through
``diffulex_b200.workload`` with numpy-drawn values, so a fixture stores only parameters, an input
digest and the reference's outputs."""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from diffulex_b200.workload import (MASK_BD_FULL, MASK_D2F_BLOCK_CAUSAL, make_problem, named_workload,
                                    small_workload)


def bits(t: torch.Tensor) -> np.ndarray:
    """Bit pattern of a tensor as a numpy integer array of the same item size."""
    t = t.detach().cpu().contiguous()
    view = {1: torch.uint8, 2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.view(view).numpy()


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = bits(a) if isinstance(a, torch.Tensor) else np.ascontiguousarray(a)
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


# ---- attention ---------------------------------------------------------------------------------
# name -> (workload factory, sequential pages?, heads stored in the fixture)
def _ref_geom(name, seqs, hq, hkv, hd, ctx, page, dbs, seed):
    return small_workload(name, hq, hkv, hd, page, dbs, [ctx] * seqs, [dbs] * seqs, MASK_BD_FULL, seed)


ATTN_CASES = {
    # benchmark configuration 1: 28/4 heads, hd 128, page 256, ctx 128..512, one 32-token block
    "cfg1": dict(w=lambda: named_workload("cfg1"), permute=True, heads=[0, 6, 7, 13, 20, 27]),
    # geometries of the reference's own decode-kernel tests
    # (tests/python/kernel/test_dllm_flash_attn_decode_kernel.py:223-391): sequential page tables,
    # uniform context; drawn here from a seed instead of unseeded randn
    "ref_single_seq": dict(w=lambda: _ref_geom("ref_single_seq", 1, 32, 8, 128, 128, 32, 32, 11), permute=False,
                           heads=[0, 3, 4, 17, 31]),
    "ref_multi_seq": dict(w=lambda: _ref_geom("ref_multi_seq", 4, 32, 8, 128, 256, 32, 32, 12), permute=False,
                          heads=[0, 5, 30]),
    "ref_gqa_8": dict(w=lambda: _ref_geom("ref_gqa_8", 2, 32, 4, 128, 128, 32, 32, 13), permute=False,
                      heads=[0, 7, 8, 15, 31]),
    "ref_head_dim_64": dict(w=lambda: _ref_geom("ref_head_dim_64", 2, 32, 8, 64, 128, 32, 32, 14), permute=False,
                            heads=[0, 1, 2, 3, 4, 12, 31]),
    "ref_large_context": dict(w=lambda: _ref_geom("ref_large_context", 2, 32, 8, 128, 512, 32, 32, 15),
                              permute=False, heads=[1, 10, 29]),
    "ref_page_block_64": dict(w=lambda: _ref_geom("ref_page_block_64", 2, 32, 8, 128, 256, 64, 32, 16),
                              permute=False, heads=[2, 11, 28]),
    "ref_diffusion_block_64": dict(w=lambda: _ref_geom("ref_diffusion_block_64", 2, 32, 8, 128, 128, 32, 64, 17),
                                   permute=False, heads=[0, 9, 31]),
    # cases the reference's tests do not pin: ragged contexts (incl. 0 and non-multiples of the
    # page), permuted page tables, -1 padded table columns, 4-token blocks
    "ragged_permuted": dict(w=lambda: small_workload("ragged_permuted", 32, 8, 128, 32, 32,
                                                      [5, 40, 64, 0, 129], [32] * 5, MASK_BD_FULL, 21),
                            permute=True, heads=[0, 3, 4, 16, 31]),
    "q4_gqa4": dict(w=lambda: small_workload("q4_gqa4", 32, 8, 128, 256, 4, [130, 700, 17, 256], [4] * 4,
                                             MASK_BD_FULL, 22), permute=True, heads=[0, 1, 2, 3, 13, 31]),
    "ragged_q": dict(w=lambda: small_workload("ragged_q", 28, 4, 128, 64, 32, [100, 33, 300], [32, 7, 19],
                                              MASK_BD_FULL, 23), permute=True, heads=[0, 6, 7, 27]),
}

# Block-causal decode over several in-flight blocks.  Golden outputs come from the reference's
# block-causal prefill check (tests/python/kernel/test_dllm_flash_attn_prefill_kernel.py:13-77)
# run over [prefix ; in-flight] as one sequence, keeping the in-flight rows; that function lines
# its diffusion blocks up from position 0, so contexts are multiples of the diffusion block.
D2F_CASES = {
    "d2f_mha": dict(w=lambda: small_workload("d2f_mha", 8, 8, 128, 32, 32, [64, 256, 96], [128, 128, 64],
                                             MASK_D2F_BLOCK_CAUSAL, 31), permute=True, heads=[0, 3, 7]),
    "d2f_gqa7": dict(w=lambda: small_workload("d2f_gqa7", 28, 4, 128, 256, 32, [512, 32], [128, 96],
                                              MASK_D2F_BLOCK_CAUSAL, 32), permute=True, heads=[0, 6, 7, 27]),
    "d2f_hd64_dbs4": dict(w=lambda: small_workload("d2f_hd64_dbs4", 16, 4, 64, 16, 4, [8, 20, 0], [16, 12, 8],
                                                   MASK_D2F_BLOCK_CAUSAL, 33), permute=True, heads=[0, 5, 15]),
}


def attn_problem(case: dict):
    return make_problem(case["w"](), device="cpu", values="numpy", permute_pages=case["permute"])


# ---- prefill ----------------------------------------------------------------------------------
def _ref_prefill(seqs, hq, hkv, hd, qlen, block, dbs, seed):
    return dict(hq=hq, hkv=hkv, hd=hd, q_lens=[qlen] * seqs, kv_lens=[qlen] * seqs, block=block, dbs=dbs, seed=seed)


PREFILL_CASES = {
    # geometries of the reference's own prefill-kernel tests
    # (tests/python/kernel/test_dllm_flash_attn_prefill_kernel.py:162-310), drawn from a seed
    "ref_single_seq": _ref_prefill(1, 32, 8, 128, 192, False, 32, 61),
    "ref_multi_seq": _ref_prefill(4, 32, 8, 128, 256, False, 32, 62),
    "ref_block_attn": _ref_prefill(2, 32, 8, 128, 256, True, 32, 63),
    "ref_block_attn_long": _ref_prefill(3, 32, 8, 128, 320, True, 32, 64),
    "ref_block_attn_dbs64": _ref_prefill(2, 32, 8, 128, 256, True, 64, 65),
    "ref_gqa_4": _ref_prefill(2, 32, 8, 128, 192, False, 32, 66),
    "ref_gqa_8": _ref_prefill(2, 32, 4, 128, 192, False, 32, 67),
    "ref_block_attn_gqa_8": _ref_prefill(2, 32, 4, 128, 256, True, 32, 68),
    "ref_head_dim_64": _ref_prefill(2, 32, 8, 64, 192, False, 32, 69),
    "ref_varied_stages": _ref_prefill(2, 32, 8, 128, 192, False, 32, 70),
    # cases the reference's tests do not pin: ragged prompts (shorter than a key tile, not multiples of the
    # diffusion block), 7 query heads per KV head, one query head per KV head
    "ragged_block_gqa7": dict(hq=28, hkv=4, hd=128, q_lens=[100, 33, 257, 1], kv_lens=[100, 33, 257, 1], block=True,
                              dbs=32, seed=71),
    "ragged_full_mha": dict(hq=8, hkv=8, hd=128, q_lens=[129, 5, 300], kv_lens=[129, 5, 300], block=False, dbs=32,
                            seed=72),
}
PREFILL_FIXTURE_HEADS = 2     # heads per case kept in the fixture (first and last)
PREFILL_FIXTURE_ROWS = 192    # rows per case kept in the fixture (seeded choice)


def prefill_inputs(case: dict):
    """(q, k, v, cu_seqlens_q, cu_seqlens_k) of a prefill case: bf16 values drawn with numpy from the seed."""
    rng = np.random.default_rng([case["seed"], 7])
    tq, tk = sum(case["q_lens"]), sum(case["kv_lens"])
    mk = lambda n, h: torch.from_numpy(rng.standard_normal(size=(n, h, case["hd"]), dtype=np.float32)).to(torch.bfloat16)
    q, k, v = mk(tq, case["hq"]), mk(tk, case["hkv"]), mk(tk, case["hkv"])
    cu = lambda lens: torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    return q, k, v, cu(case["q_lens"]), cu(case["kv_lens"])


def prefill_fixture_index(case: dict):
    """(rows, heads) of a case's outputs that the fixture holds."""
    tq = sum(case["q_lens"])
    rng = np.random.default_rng([case["seed"], 8])
    rows = np.sort(rng.choice(tq, size=min(tq, PREFILL_FIXTURE_ROWS), replace=False))
    return rows, [0, case["hq"] - 1]


# ---- store -------------------------------------------------------------------------------------
STORE_CASES = {
    "cfg1": dict(w=lambda: named_workload("cfg1"), slot_dtype="int32", drop_every=0, row_pad=0),
    "neg_slots_int64": dict(w=lambda: small_workload("neg_slots_int64", 32, 8, 128, 32, 32, [5, 40, 64],
                                                     [32, 32, 64], MASK_BD_FULL, 41),
                            slot_dtype="int64", drop_every=3, row_pad=0),
    "strided_rows": dict(w=lambda: small_workload("strided_rows", 28, 4, 128, 64, 32, [100, 33], [32, 32],
                                                  MASK_BD_FULL, 42), slot_dtype="int32", drop_every=5, row_pad=1536),
    "hd64_all_skipped_tail": dict(w=lambda: small_workload("hd64", 32, 8, 64, 64, 32, [0, 64, 7], [32, 32, 32],
                                                           MASK_BD_FULL, 43), slot_dtype="int32", drop_every=2,
                                  row_pad=0),
}


def store_inputs(case: dict):
    """(key, value, k_cache, v_cache, slot_mapping).  ``row_pad`` makes key/value strided views of a
    wider buffer (as slices of a fused projection would be); ``drop_every`` sets every n-th slot
    to -1 (rows of still-active blocks, diffulex/strategy/block_diffusion/engine/
    model_runner.py:141-142)."""
    p = make_problem(case["w"](), device="cpu", values="numpy",
                     slot_dtype=getattr(torch, case["slot_dtype"]))
    key, value = p.k, p.v
    if case["row_pad"]:
        n, h, d = key.shape
        wide = torch.zeros(n, h * d + case["row_pad"], dtype=key.dtype)
        wide2 = torch.zeros_like(wide)
        wide[:, : h * d] = key.reshape(n, -1)
        wide2[:, : h * d] = value.reshape(n, -1)
        key = wide[:, : h * d].view(n, h, d)
        value = wide2[:, : h * d].view(n, h, d)
    slots = p.slot_mapping.clone()
    if case["drop_every"]:
        slots[:: case["drop_every"]] = -1
    return key, value, p.k_cache, p.v_cache, slots


DISTINCT_X = 8   # elements of head_dim kept together in the split K layout (Config.k_cache_hdim_split_factor_x)


def distinct_caches(case: dict):
    """Seeded caches in the split ("distinct") layout for a store case: K ``[NB, H, hd/x, PAGE, x]``, V ``[NB, H, hd,
    PAGE]`` (diffulex_kernel/python/kv_cache_kernels.py:86-91), bf16, same page count and geometry as the case's
    unified caches."""
    _, _, k_cache, _, _ = store_inputs(case)
    nb, page, h, hd = k_cache.shape
    rng = np.random.default_rng([case["w"]().seed, 99])
    mk = lambda shape: torch.from_numpy(rng.standard_normal(size=shape, dtype=np.float32)).to(torch.bfloat16)
    return mk((nb, h, hd // DISTINCT_X, page, DISTINCT_X)), mk((nb, h, hd, page))


# ---- load --------------------------------------------------------------------------------------
LOAD_CASES = {
    # page-aligned contexts 256 and 512: the reference leaves their last page unwritten
    "cfg1": dict(w=lambda: named_workload("cfg1")),
    "ragged_p32": dict(w=lambda: small_workload("ragged_p32", 32, 8, 128, 32, 32, [5, 40, 64, 0], [32, 64, 32, 32],
                                                MASK_BD_FULL, 51)),
    # 48 in-flight rows with 32-row blocks: the reference drops the 16-row tail
    "ragged_tail": dict(w=lambda: small_workload("ragged_tail", 28, 4, 128, 64, 32, [100, 33], [64, 48],
                                                 MASK_BD_FULL, 52)),
    "hd64_p64": dict(w=lambda: small_workload("hd64_p64", 16, 4, 64, 64, 32, [130, 64, 1], [32, 32, 32],
                                              MASK_BD_FULL, 53)),
}


def load_problem(case: dict):
    return make_problem(case["w"](), device="cpu", values="numpy")
