"""B200-native (sm_100a) implementation of Diffulex's decode hot path: slot-mapped KV-cache store,
paged KV-cache load and dLLM paged decode attention, behind the reference's ``diffulex_kernel``
entry points.

The operator names resolve lazily so that ``diffulex_b200.build`` (which creates the CUDA
library) and ``diffulex_b200.workload`` (host-side input generation) import without it.  Touching
any operator loads ``csrc/libdlx_b200.so`` and raises ImportError if it has not been built: there
is no CPU or PyTorch fallback.
"""
_OPERATORS = {
    "store_kvcache_unified_layout": "kv_cache_kernels",
    "store_kvcache_distinct_layout": "kv_cache_kernels",
    "load_kvcache": "kv_cache_kernels",
    "dllm_flash_attn_decode": "dllm_flash_attn",
    "dllm_flash_attn_prefill": "dllm_flash_attn",
}

__all__ = list(_OPERATORS)


def __getattr__(name):
    if name in _OPERATORS:
        import importlib

        from . import _lib
        _lib.lib()  # fail loudly if the CUDA extension is missing
        return getattr(importlib.import_module(f".{_OPERATORS[name]}", __name__), name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
