"""Shadow package: put ``diffulex_b200/dropin`` ahead of the Diffulex checkout on PYTHONPATH and
``from diffulex_kernel import ...`` (diffulex/attention/attn_impl.py:5-10) resolves to the
sm_100a kernels.  Imports eagerly: a missing CUDA library is an ImportError here."""
from diffulex_b200 import (dllm_flash_attn_decode, dllm_flash_attn_prefill, load_kvcache,  # noqa: F401
                           store_kvcache_distinct_layout, store_kvcache_unified_layout)
