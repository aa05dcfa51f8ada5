"""``from diffulex_kernel.python.kv_cache_kernels import load_kvcache`` keeps working
(the reference imports it this way in diffulex_kernel/python/dllm_flash_attn.py:9)."""
from diffulex_b200.kv_cache_kernels import (load_kvcache, store_kvcache_distinct_layout,  # noqa: F401
                                            store_kvcache_unified_layout)
