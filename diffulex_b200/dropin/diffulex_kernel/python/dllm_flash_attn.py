"""Module path of the reference's attention entry points, re-exported."""
from diffulex_b200.dllm_flash_attn import dllm_flash_attn_decode, dllm_flash_attn_prefill  # noqa: F401
